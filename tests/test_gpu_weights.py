"""The worker loader on a real GPU, as SGLang drives it on one tensor-parallel
rank: pinned backups of two models, the delta package built by the real
DeltaWeights (GPU encoder), restores both ways through the fused kernel, and the
checksum confirmation all-reduce (a one-rank gloo group stands in for the NCCL
device group). Byte-exact against the models' own bytes."""

from __future__ import annotations

import json
import socket
import sys
from types import ModuleType, SimpleNamespace

import pytest
import torch
import torch.distributed as dist

from warpshift_b200 import weights as backend

pytestmark = pytest.mark.gpu


class Model(torch.nn.Module):
    def __init__(self, device) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(5)
        self.proj = torch.nn.Parameter((torch.randn(1536, 1024, generator=g) * 0.02).to(torch.bfloat16).to(device))
        self.embed = torch.nn.Parameter((torch.randn(4099, 512, generator=g) * 0.02).to(torch.bfloat16).to(device))
        self.norm = torch.nn.Parameter(torch.ones(1024, dtype=torch.bfloat16, device=device))
        self.register_buffer("rope", torch.randn(257, 64, generator=g).to(device), persistent=False)


def command(operation, model, reset=False, source="delta", from_model=None):
    return {"operation": operation, "model": model, "reset": reset, "source": source, "from_model": from_model}


def call(model, cmd) -> None:
    backend.model_weight_loader(model, [(json.dumps(cmd), torch.empty(0, dtype=torch.uint8))])


@pytest.fixture
def one_rank_group(monkeypatch):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    group = dist.group.WORLD
    mod = ModuleType("sglang.srt.distributed")
    mod.get_tp_group = lambda: SimpleNamespace(cpu_group=group, device_group=group)
    monkeypatch.setitem(sys.modules, "sglang.srt.distributed", mod)
    yield group
    dist.destroy_process_group()


def snapshot(model) -> dict[str, torch.Tensor]:
    return {n: t.detach().clone() for n, t in backend._collect_tensors(model).items()}


def same(model, want) -> None:
    got = backend._collect_tensors(model)
    assert got.keys() == want.keys()
    for name, t in got.items():
        assert torch.equal(t.view(-1).view(torch.uint8), want[name].view(-1).view(torch.uint8)), name


def test_worker_loader_switches_both_ways_on_the_gpu(cuda_device, one_rank_group) -> None:
    model = Model(cuda_device)
    a = snapshot(model)
    call(model, command("backup", "a", reset=True))
    with torch.no_grad():
        model.proj.add_(model.proj * 0.01)  # Teacher2-like relative perturbation
        model.embed[7:11].add_(0.5)
        model.rope.mul_(1.5)
    b = snapshot(model)
    pointers = {n: t.data_ptr() for n, t in backend._collect_tensors(model).items()}
    call(model, command("backup", "b"))
    delta = getattr(model, backend._STATE)["delta"]
    assert delta.stats["encoder"] == "gpu" and delta.stats["runtime_bytes"] > 0
    same(model, b)  # building the package never changes the resident weights
    call(model, command("restore", "a", from_model="b"))
    same(model, a)
    assert delta.last_apply["ok"] and delta.last_apply["checksum"] == delta.last_apply["expected"]
    call(model, command("restore", "b", from_model="a"))
    same(model, b)
    call(model, command("restore", "a", from_model="b"))
    same(model, a)
    assert {n: t.data_ptr() for n, t in backend._collect_tensors(model).items()} == pointers
    with pytest.raises(RuntimeError):
        call(model, command("restore", "a", from_model="b"))  # stale source: the resident model is a
    same(model, a)
