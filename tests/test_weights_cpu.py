"""CPU contracts of the worker-side manager, after the reference's tests/test_weights.py.

Backups and restores on a tiny model, delta prepare with a CPU stand-in for the
codec, restore validation, and the tensor-parallel two-phase agreement with
``all_gather_object`` emulating 4 ranks (as the reference's tests do).
"""

from __future__ import annotations

import json
import sys
from types import ModuleType, SimpleNamespace
from typing import Any, Literal

import pytest
import torch

from warpshift_b200 import weights as backend


class TinyModel(torch.nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.weight = torch.nn.Parameter(torch.arange(8, dtype=torch.bfloat16).reshape(2, 4))
        self.tied = self.weight
        self.A_log = torch.nn.Parameter(torch.tensor([0.001], dtype=torch.float32))
        self.register_buffer("derived", torch.tensor([0.25, 0.5]), persistent=False)
        self.register_buffer("view", self.weight.detach()[:, :2])  # same start pointer, different shape


def command(operation: Literal["backup", "restore"], model: str, reset: bool = False, source: str | None = "pageable",
            from_model: str | None = None) -> dict[str, Any]:
    return {"operation": operation, "model": model, "reset": reset, "source": source, "from_model": from_model}


def test_collect_tensors_prefixes_dedups_aliases_and_keeps_views() -> None:
    model = TinyModel()
    names = list(backend._collect_tensors(model))
    assert names == ["parameter:weight", "parameter:A_log", "buffer:derived", "buffer:view"]
    model.register_buffer("empty", torch.zeros(0))
    assert "buffer:empty" not in backend._collect_tensors(model)


@pytest.mark.parametrize("source", ["pageable", "pinned"])
def test_round_trip_restores_bf16_fp32_buffers_and_preserves_pointers(monkeypatch, source: str) -> None:
    if source == "pinned":  # no CUDA here: record the request, allocate pageable
        original = torch.empty_like
        monkeypatch.setattr(torch, "empty_like", lambda t, **kw: original(t, **{**kw, "pin_memory": False}))
        monkeypatch.setattr(torch.cuda, "synchronize", lambda device=None: None)
    model = TinyModel()
    tensors = backend._collect_tensors(model)
    pointers = {name: t.data_ptr() for name, t in tensors.items()}
    expected = {"a": {n: t.detach().clone() for n, t in tensors.items()}}
    backend._update_worker_weights(model, command("backup", "a", reset=True, source=source))
    with torch.no_grad():
        model.weight.add_(10)
        model.A_log.add_(1)
        model.derived.add_(2)
    expected["b"] = {n: t.detach().clone() for n, t in tensors.items()}
    backend._update_worker_weights(model, command("backup", "b", source=source))
    for target in ("a", "b", "a", "b"):
        backend._update_worker_weights(model, command("restore", target, source=source))
        for name, t in tensors.items():
            assert torch.equal(t, expected[target][name])
            assert t.data_ptr() == pointers[name]
        assert model.tied is model.weight


def test_restore_uses_cached_tensors_and_reset_drops_old_cpu_backups(monkeypatch) -> None:
    model = TinyModel()
    backend._update_worker_weights(model, command("backup", "a", reset=True))
    backend._update_worker_weights(model, command("backup", "b"))
    collect = backend._collect_tensors
    monkeypatch.setattr(backend, "_collect_tensors", lambda _: pytest.fail("Hot path rescanned model"))
    backend._update_worker_weights(model, command("restore", "a"))
    monkeypatch.setattr(backend, "_collect_tensors", collect)
    backend._update_worker_weights(model, command("backup", "c", reset=True))
    assert list(getattr(model, backend._STATE)["cpu_backups"]) == ["c"]


def test_backup_rejects_changed_layout_before_storing_it() -> None:
    model = TinyModel()
    backend._update_worker_weights(model, command("backup", "a", reset=True))
    model.register_buffer("extra", torch.ones(1))
    with pytest.raises(ValueError, match="layout changed"):
        backend._update_worker_weights(model, command("backup", "b"))
    assert list(getattr(model, backend._STATE)["cpu_backups"]) == ["a"]


def test_pinned_backup_uses_pinned_allocator(monkeypatch) -> None:
    original, flags = torch.empty_like, []

    def allocate(tensor, **kwargs):
        flags.append(kwargs["pin_memory"])
        return original(tensor, **{**kwargs, "pin_memory": False})

    monkeypatch.setattr(torch, "empty_like", allocate)
    backend._update_worker_weights(TinyModel(), command("backup", "a", reset=True, source="pinned"))
    assert flags and all(flags)


def test_unknown_operation_is_rejected() -> None:
    model = TinyModel()
    backend._update_worker_weights(model, command("backup", "a", reset=True))
    with pytest.raises(ValueError, match="Unknown operation"):
        backend._update_worker_weights(model, {**command("backup", "a"), "operation": "erase"})


class FakeDelta:
    """CPU stand-in for the codec; the worker protocol owns model identity."""

    def __init__(self, cpu_base, gpu_tensors) -> None:
        self.base = {n: t.clone() for n, t in cpu_base.items()}
        self.target = {n: t.detach().clone() for n, t in gpu_tensors.items()}
        self.gpu_tensors = gpu_tensors
        self.pointers = {n: t.data_ptr() for n, t in gpu_tensors.items()}
        self.reverse_calls: list[bool] = []
        self.stats = {"payload_bytes": 1}
        self.last_apply = None

    def validate_bindings(self) -> None:
        if any(t.data_ptr() != self.pointers[n] for n, t in self.gpu_tensors.items()):
            raise ValueError("Delta tensor binding changed")

    def apply(self, *, reverse: bool) -> None:
        self.reverse_calls.append(reverse)
        src = self.base if reverse else self.target
        with torch.no_grad():
            for n, t in self.gpu_tensors.items():
                t.copy_(src[n])
        self.last_apply = {"ok": True, "checksum": 0, "expected": 0}


def install_fake_tp(monkeypatch, world: int = 1, gather=None, device_group=None) -> object:
    tp_group = object()
    dist_mod = ModuleType("sglang.srt.distributed")
    dist_mod.get_tp_group = lambda: SimpleNamespace(cpu_group=tp_group, device_group=device_group)
    monkeypatch.setitem(sys.modules, "sglang.srt.distributed", dist_mod)
    monkeypatch.setattr(torch.distributed, "get_rank", lambda group: 0)
    monkeypatch.setattr(torch.distributed, "get_world_size", lambda group: world)

    def all_gather_object(results, local, group):
        assert group is tp_group
        results[:] = [local] * len(results)
        if gather:
            gather(results, local)

    monkeypatch.setattr(torch.distributed, "all_gather_object", all_gather_object)
    return tp_group


@pytest.fixture
def delta_packages(monkeypatch) -> list[FakeDelta]:
    packages: list[FakeDelta] = []

    def build(cpu_base, gpu_tensors):
        packages.append(FakeDelta(cpu_base, gpu_tensors))
        return packages[-1]

    module = ModuleType("warpshift_b200.delta")
    module.DeltaWeights = build
    monkeypatch.setitem(sys.modules, "warpshift_b200.delta", module)
    install_fake_tp(monkeypatch)
    return packages


def prepare_delta_pair(model: TinyModel) -> None:
    backend.model_weight_loader(model, [(json.dumps(command("backup", "a", reset=True, source="delta")), torch.empty(0))])
    with torch.no_grad():
        model.weight.add_(10)
        model.A_log.add_(1)
        model.derived.add_(2)
    backend.model_weight_loader(model, [(json.dumps(command("backup", "b", source="delta")), torch.empty(0))])


def test_delta_prepare_builds_one_package_releases_backups_and_keeps_b(delta_packages) -> None:
    model = TinyModel()
    original = {n: t.detach().clone() for n, t in backend._collect_tensors(model).items()}
    prepare_delta_pair(model)
    state = getattr(model, backend._STATE)
    assert len(delta_packages) == 1 and state["delta"] is delta_packages[0]
    assert state["delta_models"] == ("a", "b") and state["current"] == "b"
    assert state["cpu_backups"] == {} and delta_packages[0].reverse_calls == []
    for name, t in state["gpu_tensors"].items():
        assert torch.equal(delta_packages[0].base[name], original[name])
        assert torch.equal(t, delta_packages[0].target[name])


def test_delta_prepare_rejects_the_same_model_twice(delta_packages) -> None:
    model = TinyModel()
    backend.model_weight_loader(model, [(json.dumps(command("backup", "a", reset=True, source="delta")), torch.empty(0))])
    with pytest.raises(RuntimeError, match="exactly two distinct models"):
        backend.model_weight_loader(model, [(json.dumps(command("backup", "a", source="delta")), torch.empty(0))])
    assert delta_packages == []


@pytest.mark.parametrize(("from_model", "target", "message"),
                         [(None, "a", "source model"), ("a", "a", "source model"), ("b", "b", "other model"), ("b", "c", "other model")])
def test_delta_restore_requires_current_source_and_other_target(delta_packages, from_model, target, message) -> None:
    model = TinyModel()
    prepare_delta_pair(model)
    with pytest.raises(ValueError, match=message):
        backend._validate_delta_restore(model, command("restore", target, source="delta", from_model=from_model))
    assert delta_packages[0].reverse_calls == []


@pytest.mark.parametrize("replacement", ["storage", "parameter"])
def test_delta_restore_rejects_changed_bindings(delta_packages, replacement: str) -> None:
    model = TinyModel()
    prepare_delta_pair(model)
    if replacement == "storage":
        model.weight.data = model.weight.detach().clone()
    else:
        model.weight = torch.nn.Parameter(model.weight.detach().clone())
    with pytest.raises(ValueError, match="(?i)(binding|storage|tensor)"):
        backend._validate_delta_restore(model, command("restore", "a", source="delta", from_model="b"))
    assert delta_packages[0].reverse_calls == []


def test_delta_restore_before_prepare_is_rejected() -> None:
    model = TinyModel()
    setattr(model, backend._STATE, {"cpu_backups": {}})
    with pytest.raises(ValueError, match="Prepare the delta"):
        backend._validate_delta_restore(model, command("restore", "a", source="delta", from_model="b"))


@pytest.mark.parametrize("outcome", ["preflight_error", "different_commands", "apply_error", "success"])
def test_tp4_agrees_before_writes_and_commits_only_after_all_ranks_succeed(monkeypatch, delta_packages, outcome) -> None:
    model = TinyModel()
    prepare_delta_pair(model)
    cmd = command("restore", "a", source="delta", from_model="b")
    gathers: list[Any] = []
    updates: list[dict[str, Any]] = []

    def gather(results, local):
        gathers.append(local)
        if len(gathers) == 1:
            if outcome == "preflight_error":
                results[3] = (cmd, "rank 3: ValueError: stale source")
            elif outcome == "different_commands":
                results[2] = ({**cmd, "model": "b"}, None)
        elif outcome == "apply_error":
            results[2] = "rank 2: RuntimeError: decode failed"

    install_fake_tp(monkeypatch, world=4, gather=gather)
    update = backend._update_worker_weights

    def update_weights(target_model, received):
        updates.append(received)
        update(target_model, received)
        assert getattr(target_model, backend._STATE)["current"] == "b"

    monkeypatch.setattr(backend, "_update_worker_weights", update_weights)
    payload = [(json.dumps(cmd), torch.empty(0, dtype=torch.uint8))]
    if outcome == "success":
        backend.model_weight_loader(model, payload)
    else:
        message = {"preflight_error": "rank 3", "different_commands": "different weight commands", "apply_error": "rank 2"}
        with pytest.raises(RuntimeError, match=message[outcome]):
            backend.model_weight_loader(model, payload)
    assert updates == ([] if outcome in {"preflight_error", "different_commands"} else [cmd])
    assert len(gathers) == (1 if not updates else 2)
    assert getattr(model, backend._STATE)["current"] == ("a" if outcome == "success" else "b")
    assert delta_packages[0].reverse_calls == ([] if not updates else [True])
