"""Two real ranks (gloo, world size 2) running the worker loader protocol.

Each rank runs model_weight_loader with a real process group: the two-phase
agreement of weights.py:106-137 on the CPU group, plus the checksum
confirmation all-reduce (DeltaWeights.confirm) on the "device" group, which is
NCCL in production and gloo here. Failures are injected on the host: a rank
whose apply raises, a rank whose written bytes do not hash to the expected
checksum, a rank with a stale source model. When the switch is not confirmed
on every rank, the ranks whose own switch succeeded switch back, so every rank
ends on the source model.
"""

from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path
from types import ModuleType, SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, scenario: str, queue) -> None:
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        device_group = dist.new_group(backend="gloo")
        fake_tp = ModuleType("sglang.srt.distributed")
        fake_tp.get_tp_group = lambda: SimpleNamespace(cpu_group=dist.group.WORLD, device_group=device_group)
        sys.modules["sglang.srt.distributed"] = fake_tp

        from warpshift_b200 import weights as backend
        from warpshift_b200.delta import DeltaWeights

        class RankDelta:
            """Host stand-in for one rank's package; confirm() is the product's all-reduce."""

            def __init__(self, cpu_base, gpu_tensors):
                self.base = {n: t.clone() for n, t in cpu_base.items()}
                self.target = {n: t.detach().clone() for n, t in gpu_tensors.items()}
                self.tensors = gpu_tensors
                self.stats = {}
                self.device = torch.device("cpu")
                self.last_apply = None

            def validate_bindings(self):
                pass

            def apply(self, *, reverse):
                if scenario == "apply_error" and rank == 1:
                    raise RuntimeError("delta decode failed: device errors 0x1")
                if scenario == "undo_error" and rank == 0 and not reverse:
                    raise RuntimeError("copy engine error")  # rank 0's switch back fails
                src = self.base if reverse else self.target
                with torch.no_grad():
                    for n, t in self.tensors.items():
                        t.copy_(src[n])
                bad = scenario in ("checksum_mismatch", "undo_error") and rank == 1
                self.last_apply = {"ok": True, "checksum": 1000 + rank + (7 if bad else 0), "expected": 1000 + rank}

            confirm = DeltaWeights.confirm

        fake_delta = ModuleType("warpshift_b200.delta")
        fake_delta.DeltaWeights = RankDelta
        sys.modules["warpshift_b200.delta"] = fake_delta

        model = torch.nn.Linear(4, 4, bias=False)
        with torch.no_grad():
            model.weight.fill_(1.0)

        def send(cmd):
            backend.model_weight_loader(model, [(json.dumps(cmd), torch.empty(0, dtype=torch.uint8))])

        base = {"operation": "backup", "source": "delta", "from_model": None}
        send({**base, "model": "a", "reset": True})
        with torch.no_grad():
            model.weight.fill_(2.0 + rank)
        send({**base, "model": "b", "reset": False})
        from_model = "a" if (scenario == "stale_source" and rank == 1) else "b"
        outcome = "ok"
        try:
            send({"operation": "restore", "source": "delta", "model": "a", "from_model": from_model, "reset": False})
        except RuntimeError as exc:
            outcome = f"error: {exc}"
        state = getattr(model, backend._STATE)
        queue.put((rank, outcome, state["current"], float(model.weight[0, 0])))
        dist.destroy_process_group()
    except Exception:
        queue.put((rank, "crash: " + traceback.format_exc(), None, None))


def _run(scenario: str) -> dict[int, tuple]:
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, scenario, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, outcome, current, w = queue.get(timeout=180)
        results[rank] = (outcome, current, w)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("scenario", ["success", "apply_error", "checksum_mismatch", "stale_source", "undo_error"])
def test_two_ranks_agree_before_writing_and_confirm_after(scenario: str) -> None:
    results = _run(scenario)
    for rank, (outcome, current, weight) in results.items():
        assert not outcome.startswith("crash"), outcome
        if scenario == "success":
            assert outcome == "ok" and current == "a" and weight == 1.0
        elif scenario == "stale_source":
            assert "rank 1" in outcome and "source model" in outcome
            assert current == "b" and weight == 2.0 + rank  # no rank wrote
        elif scenario == "undo_error":
            # rank 1 missed its checksum; rank 0 switched but could not switch back,
            # and every rank's error names that.
            assert "rank 1" in outcome and "switching back to b failed" in outcome
            assert current == "b"
        else:
            assert outcome.startswith("error") and "rank 1" in outcome
            assert current == "b"  # identity not committed on any rank
            assert weight == 2.0 + rank  # every rank holds the source model again
    if scenario == "checksum_mismatch":
        assert "not confirmed" in results[0][0]
