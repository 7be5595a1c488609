"""Worker-side weight manager: parameter walk, CPU backups and the delta switch.

Drop-in for the worker half of the reference's ``warpshift/weights.py``
(lines 27-137). SGLang loads ``model_weight_loader`` by name (``LOADER``) and
drives it with JSON commands ``{operation, model, source, from_model, reset}``;
the per-model state lives on the model object under ``_STATE`` with the keys
the reference uses (``cpu_backups``, ``gpu_tensors``, ``layout``, ``pinned``,
``delta``, ``delta_models``, ``current``), and the functions keep the
reference's names, exception types and messages.

How a command runs on one tensor-parallel rank (``model_weight_loader``):

1. **propose** — decode the command and check it locally
   (``_validate_delta_restore``); every rank shares its (command, error) on
   the TP CPU group, and nothing is written unless all ranks hold the same
   command and none failed;
2. **execute** — ``_update_worker_weights`` dispatches to the backup or
   restore handler;
3. **confirm** (delta restores) — every rank contributes one flag, "my switch
   wrote the expected bytes", to an all-reduce over the TP device group (NCCL
   under SGLang) through ``DeltaWeights.confirm``. If any rank's flag is down,
   the ranks whose own switch succeeded switch back, so the whole group holds
   the source model again;
4. **acknowledge** — every rank shares its outcome on the CPU group; the
   model identity (``current``) changes only if all ranks succeeded.

The HTTP control client of the reference (weights.py:140-261) is control plane
and is not part of this package.
"""

from __future__ import annotations

import json
import logging
from collections.abc import Callable, Iterable
from typing import TYPE_CHECKING, Any, Literal

if TYPE_CHECKING:
    import torch

WeightSource = Literal["disk", "pageable", "pinned", "delta"]

LOADER = "warpshift_b200.weights.model_weight_loader"
_STATE = "_warpshift_weights"

_log = logging.getLogger(__name__)


# --------------------------------------------------------------------------- tensor set
def _identity(tensor: torch.Tensor) -> tuple[Any, ...]:
    """Two registrations are the same tensor when they view the same bytes the same way."""
    return tensor.device, tensor.data_ptr(), tensor.dtype, tuple(tensor.shape), tuple(tensor.stride())


def _collect_tensors(model: torch.nn.Module) -> dict[str, torch.Tensor]:
    """Every registered parameter and buffer, non-persistent buffers included (weights.py:27-36).

    Names carry a ``parameter:`` or ``buffer:`` prefix. The first registration of
    a tensor wins (tied weights appear once); a view that starts at the same
    address but has another shape or stride is a different tensor; empty
    tensors are left out.
    """
    first: dict[tuple[Any, ...], tuple[str, torch.Tensor]] = {}
    for kind, named in (("parameter", model.named_parameters()), ("buffer", model.named_buffers())):
        for name, tensor in named:
            if tensor.numel():
                first.setdefault(_identity(tensor), (f"{kind}:{name}", tensor))
    return dict(first.values())


# --------------------------------------------------------------------------- operations
def _state(model: torch.nn.Module) -> dict[str, Any]:
    return getattr(model, _STATE)


def _snapshot(tensors: dict[str, torch.Tensor], pinned: bool) -> dict[str, torch.Tensor]:
    """Host copies of ``tensors`` (page-locked when ``pinned``), weights.py:65-70."""
    import torch

    copies = {}
    for name, tensor in tensors.items():
        host = torch.empty_like(tensor, device="cpu", pin_memory=pinned)
        host.copy_(tensor.detach())
        copies[name] = host
    return copies


def _backup(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Record the resident model under ``command["model"]``; with source "delta"
    and one model already recorded, build the pair's delta package instead."""
    if command.get("reset"):
        setattr(model, _STATE, {"cpu_backups": {}})
    state = _state(model)
    tensors = _collect_tensors(model)
    layout = {name: (tuple(t.shape), t.dtype) for name, t in tensors.items()}
    if not tensors or state.get("layout", layout) != layout:
        raise ValueError("Model tensor layout changed")
    state.update(gpu_tensors=tensors, layout=layout, pinned=command["source"] == "pinned")
    name = command["model"]
    if command["source"] == "delta" and state["cpu_backups"]:
        _build_delta(state, name)
    else:
        state["cpu_backups"][name] = _snapshot(tensors, state["pinned"])


def _build_delta(state: dict[str, Any], second: str) -> None:
    """Replace the single recorded backup by the delta package between it (A) and
    the resident model (B); the package keeps no full host copy (weights.py:53-64)."""
    from warpshift_b200.delta import DeltaWeights

    first, cpu_base = next(iter(state["cpu_backups"].items()))
    if "delta" in state or first == second:
        raise ValueError("Delta prepare requires exactly two distinct models")
    _log.info("Building delta package: %s <-> %s", first, second)
    package = DeltaWeights(cpu_base, state["gpu_tensors"])
    state.update(delta=package, delta_models=(first, second))
    state["cpu_backups"].clear()
    _log.info("Delta package ready: %s", json.dumps(package.stats))


def _restore(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Make ``command["model"]`` resident: a delta switch, or a full copy from its backup."""
    import torch

    state = _state(model)
    target = command["model"]
    if command["source"] == "delta":
        # Towards the first model of the pair the package applies B -> A.
        state["delta"].apply(reverse=target == state["delta_models"][0])
        return  # the identity is committed by the loader once every rank succeeded
    backup = state["cpu_backups"][target]
    tensors = state["gpu_tensors"]
    with torch.no_grad():
        for name, tensor in tensors.items():
            tensor.copy_(backup[name], non_blocking=state["pinned"])
    for device in {t.device for t in tensors.values() if t.is_cuda}:
        torch.cuda.synchronize(device)


_OPERATIONS: dict[str, Callable[[torch.nn.Module, dict[str, Any]], None]] = {"backup": _backup, "restore": _restore}


def _update_worker_weights(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Run one backup or restore command on this rank (weights.py:39-84)."""
    handler = _OPERATIONS.get(command["operation"])
    if handler is None:
        raise ValueError(f"Unknown operation: {command['operation']}")
    handler(model, command)


def _is_delta_restore(command: dict[str, Any] | None) -> bool:
    return bool(command) and command["source"] == "delta" and command["operation"] == "restore"


def _validate_delta_restore(model: torch.nn.Module, command: dict[str, Any]) -> None:
    """Refuse a delta restore that would read stale or moved weights (weights.py:87-103).

    Checked in order: a package exists, the command's source is the resident
    model, its target is the other model of the pair, the model still registers
    the very tensors the package was built on, and their storage is unchanged.
    """
    if not _is_delta_restore(command):
        return
    state = _state(model)
    if "delta" not in state:
        raise ValueError("Prepare the delta package before restoring")
    resident, target = state["current"], command["model"]
    if command.get("from_model") != resident:
        raise ValueError("Delta source model does not match resident weights")
    if target == resident or target not in state["delta_models"]:
        raise ValueError("Delta target must be the other model in the prepared pair")
    registered, bound = _collect_tensors(model), state["gpu_tensors"]
    if registered.keys() != bound.keys() or any(registered[n] is not bound[n] for n in bound):
        raise ValueError("Delta model tensors were replaced; prepare again")
    state["delta"].validate_bindings()


# --------------------------------------------------------------------------- the TP protocol
class _RankOutcome:
    """Context manager that records the first exception of one rank as the
    reference reports it ("rank r: Type: message") instead of raising it."""

    def __init__(self, rank: int, error: str | None = None) -> None:
        self.rank = rank
        self.error = error

    def __enter__(self) -> "_RankOutcome":
        return self

    def __exit__(self, kind, exc, traceback) -> bool:
        if isinstance(exc, Exception):
            self.fail(exc)
            return True
        return False

    def fail(self, exc: BaseException) -> None:
        if self.error is None:
            self.error = f"rank {self.rank}: {type(exc).__name__}: {exc}"


def _tp_groups() -> tuple[Any, Any]:
    """SGLang's TP CPU (gloo) group and device (NCCL) group of this worker."""
    from sglang.srt.distributed import get_tp_group

    tp = get_tp_group()
    return tp.cpu_group, getattr(tp, "device_group", None)


def _share(group: Any, size: int, mine: Any) -> list[Any]:
    """Every rank's ``mine``, in rank order (one all-gather on the CPU group)."""
    import torch.distributed as dist

    everyone: list[Any] = [None] * size
    dist.all_gather_object(everyone, mine, group=group)
    return everyone


def _confirm_switch(model: torch.nn.Module, command: dict[str, Any], device_group: Any, outcome: _RankOutcome) -> None:
    """Delta restores only; every rank calls it. One all-reduce of per-rank
    success flags over the device group; if the group did not switch as a
    whole, a rank whose own switch succeeded switches back to the source."""
    delta = _state(model).get("delta")
    if delta is None or device_group is None:
        return
    try:
        delta.confirm(device_group, failed=outcome.error is not None)
    except RuntimeError as exc:
        if outcome.error is None:
            outcome.fail(exc)
            undo = dict(command, model=command["from_model"])
            try:
                _restore(model, undo)
            except Exception as undo_exc:  # this rank's weights are then neither model: say so
                _log.error("Switching back to %s failed: %s", command["from_model"], undo_exc)
                outcome.error += (f"; switching back to {command['from_model']} failed "
                                  f"({type(undo_exc).__name__}: {undo_exc})")


def model_weight_loader(model: torch.nn.Module, named_tensors: Iterable[tuple[str, torch.Tensor]]) -> None:
    """SGLang custom weight loader: one command, agreed by every TP rank before any
    write and committed only after every rank succeeded (weights.py:106-137)."""
    import torch.distributed as dist

    cpu_group, device_group = _tp_groups()
    rank, size = dist.get_rank(cpu_group), dist.get_world_size(cpu_group)

    # 1. propose
    command = None
    proposal = _RankOutcome(rank)
    with proposal:
        ((payload, _),) = named_tensors
        command = json.loads(payload)
        _validate_delta_restore(model, command)
    proposals = _share(cpu_group, size, (command, proposal.error))
    refused = [error for _, error in proposals if error]
    if refused:
        raise RuntimeError("; ".join(refused))
    if any(other != command for other, _ in proposals):
        raise RuntimeError("TP ranks received different weight commands")

    # 2. execute, 3. confirm
    outcome = _RankOutcome(rank)
    with outcome:
        _update_worker_weights(model, command)
    if _is_delta_restore(command):
        _confirm_switch(model, command, device_group, outcome)

    # 4. acknowledge
    failures = [error for error in _share(cpu_group, size, outcome.error) if error]
    if failures:
        raise RuntimeError("; ".join(failures))
    if command["source"] == "delta":
        _state(model)["current"] = command["model"]
