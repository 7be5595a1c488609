"""Worker-side weight manager: parameter walk, CPU backups and the delta switch.

Drop-in for the worker half of the reference's ``warpshift/weights.py``
(lines 27-137): ``_collect_tensors``, ``_update_worker_weights``,
``_validate_delta_restore`` and the SGLang custom-loader entry point
``model_weight_loader``. These run inside each tensor-parallel worker process
and keep the reference's two-phase agreement: every rank validates before any
rank writes, and the model identity is committed only after every rank reports
success. For delta restores each rank additionally all-reduces its apply
outcome and shard checksums over the worker's device process group (NCCL under
SGLang), which confirms the switch on the GPUs themselves.

The HTTP control client of the reference (weights.py:140-261) is control plane
and is not part of this package.
"""

from __future__ import annotations

import json
import logging
from collections.abc import Iterable
from typing import TYPE_CHECKING, Any, Literal

if TYPE_CHECKING:
    import torch

WeightSource = Literal["disk", "pageable", "pinned", "delta"]

LOADER = "warpshift_b200.weights.model_weight_loader"
_STATE = "_warpshift_weights"


def _collect_tensors(model: torch.nn.Module) -> dict[str, torch.Tensor]:
    """Registered parameters and buffers, non-persistent ones included (weights.py:27-36).

    Names are prefixed ``parameter:``/``buffer:``; aliases are dropped by
    (device, pointer, dtype, shape, stride), so a same-pointer view of a
    different shape is kept; empty tensors are skipped.
    """
    tensors: dict[str, torch.Tensor] = {}
    seen: set[tuple[Any, ...]] = set()
    for prefix, named in (("parameter", model.named_parameters()), ("buffer", model.named_buffers())):
        for name, tensor in named:
            key = (tensor.device, tensor.data_ptr(), tensor.dtype, tuple(tensor.shape), tuple(tensor.stride()))
            if tensor.numel() and key not in seen:
                seen.add(key)
                tensors[f"{prefix}:{name}"] = tensor
    return tensors


def _update_worker_weights(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Backup or restore one model on this rank (weights.py:39-84)."""
    import torch

    target = command["model"]
    operation = command["operation"]
    if operation == "backup":
        if command.get("reset"):
            setattr(model, _STATE, {"cpu_backups": {}})
        state = getattr(model, _STATE)
        gpu_tensors = _collect_tensors(model)
        layout = {name: (tuple(t.shape), t.dtype) for name, t in gpu_tensors.items()}
        if not gpu_tensors or layout != state.get("layout", layout):
            raise ValueError("Model tensor layout changed")
        state["gpu_tensors"], state["layout"] = gpu_tensors, layout
        state["pinned"] = command["source"] == "pinned"
        if command["source"] == "delta" and state["cpu_backups"]:
            from warpshift_b200.delta import DeltaWeights

            base_model, cpu_base = next(iter(state["cpu_backups"].items()))
            if base_model == target or "delta" in state:
                raise ValueError("Delta prepare requires exactly two distinct models")
            logging.getLogger(__name__).info("Building delta package: %s <-> %s", base_model, target)
            state["delta"] = DeltaWeights(cpu_base, gpu_tensors)
            state["delta_models"] = (base_model, target)
            state["cpu_backups"].clear()  # the package keeps no full CPU copy
            logging.getLogger(__name__).info("Delta package ready: %s", json.dumps(state["delta"].stats))
            return
        backup = {}
        for name, gpu_tensor in gpu_tensors.items():
            cpu_tensor = torch.empty_like(gpu_tensor, device="cpu", pin_memory=state["pinned"])
            cpu_tensor.copy_(gpu_tensor.detach())
            backup[name] = cpu_tensor
        state["cpu_backups"][target] = backup
    elif operation == "restore":
        state = getattr(model, _STATE)
        if command["source"] == "delta":
            base_model = state["delta_models"][0]
            state["delta"].apply(reverse=target == base_model)
            return  # identity is committed only after every rank succeeds
        backup = state["cpu_backups"][target]
        with torch.no_grad():
            for name, gpu_tensor in state["gpu_tensors"].items():
                gpu_tensor.copy_(backup[name], non_blocking=state["pinned"])
        for device in {t.device for t in state["gpu_tensors"].values() if t.is_cuda}:
            torch.cuda.synchronize(device)
    else:
        raise ValueError(f"Unknown operation: {operation}")


def _validate_delta_restore(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Reject a stale source or changed GPU storage before any rank writes (weights.py:87-103)."""
    if command["source"] != "delta" or command["operation"] != "restore":
        return
    state = getattr(model, _STATE)
    if "delta" not in state:
        raise ValueError("Prepare the delta package before restoring")
    if command.get("from_model") != state["current"]:
        raise ValueError("Delta source model does not match resident weights")
    if command["model"] not in state["delta_models"] or command["model"] == state["current"]:
        raise ValueError("Delta target must be the other model in the prepared pair")
    current = _collect_tensors(model)
    if current.keys() != state["gpu_tensors"].keys() or any(
        tensor is not state["gpu_tensors"][name] for name, tensor in current.items()
    ):
        raise ValueError("Delta model tensors were replaced; prepare again")
    state["delta"].validate_bindings()


def _tp_groups() -> tuple[Any, Any]:
    """SGLang's TP CPU (gloo) group and device (NCCL) group of this worker."""
    from sglang.srt.distributed import get_tp_group

    tp = get_tp_group()
    return tp.cpu_group, getattr(tp, "device_group", None)


def _confirm_delta(model: torch.nn.Module, device_group: Any, failed_locally: bool) -> str | None:
    """NCCL all-reduce of the apply outcome and shard checksums; every rank calls it."""
    state = getattr(model, _STATE, {})
    delta = state.get("delta")
    if delta is None or device_group is None:
        return None
    if failed_locally and delta.last_apply is not None:
        delta.last_apply = {**delta.last_apply, "ok": False}
    try:
        delta.confirm(device_group)
    except RuntimeError as exc:
        return str(exc)
    return None


def model_weight_loader(model: torch.nn.Module, named_tensors: Iterable[tuple[str, torch.Tensor]]) -> None:
    """Agree before writes and acknowledge GPU completion on every TP rank (weights.py:106-137)."""
    import torch.distributed as dist

    cpu_group, device_group = _tp_groups()
    rank, size = dist.get_rank(cpu_group), dist.get_world_size(cpu_group)
    command, error = None, None
    try:
        ((payload, _),) = named_tensors
        command = json.loads(payload)
        _validate_delta_restore(model, command)
    except Exception as exc:
        error = f"rank {rank}: {type(exc).__name__}: {exc}"
    proposals: list[tuple[dict[str, Any] | None, str | None]] = [(None, None)] * size
    dist.all_gather_object(proposals, (command, error), group=cpu_group)
    errors = [failure for _, failure in proposals if failure]
    if errors:
        raise RuntimeError("; ".join(errors))
    if any(proposal != command for proposal, _ in proposals):
        raise RuntimeError("TP ranks received different weight commands")

    try:
        _update_worker_weights(model, command)
    except Exception as exc:
        error = f"rank {rank}: {type(exc).__name__}: {exc}"
    if command["source"] == "delta" and command["operation"] == "restore":
        # Every rank reaches this collective: the command was agreed above.
        unconfirmed = _confirm_delta(model, device_group, error is not None)
        if unconfirmed and error is None:
            error = f"rank {rank}: RuntimeError: {unconfirmed}"
    completions: list[str | None] = [None] * size
    dist.all_gather_object(completions, error, group=cpu_group)
    if any(completions):
        raise RuntimeError("; ".join(failure for failure in completions if failure))
    if command["source"] == "delta":
        getattr(model, _STATE)["current"] = command["model"]
