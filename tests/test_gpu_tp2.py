"""Two tensor-parallel ranks on two GPUs, NCCL between them (skipped with fewer GPUs).

Each rank builds the package of its own TP=2 shard of the Llama-3-70B shape
(one layer), switches it with the fused kernel, and confirms the switch with
DeltaWeights.confirm: one NCCL all-reduce of per-rank success flags. In the
failure scenario rank 1's payload arena is corrupted on the host before the
switch: rank 1's apply fails and rolls itself back, both ranks learn through
the all-reduce that the switch was not confirmed, and rank 0 switches back, so
both GPUs end on the source model. Both ranks take every collective in the same
order; the process group has a short timeout; NVLS is off.
"""

from __future__ import annotations

import ctypes
import dataclasses
import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, scenario: str, queue) -> None:
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import numpy as np
        import torch.distributed as dist

        from oracle import stream as ostream
        from warpshift_b200 import synth
        from warpshift_b200.delta import DeltaWeights

        device = torch.device("cuda", rank)
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60), device_id=device)
        spec = synth.model_spec(dataclasses.replace(synth.LLAMA3_70B, layers=1), tp=2, rank=rank)
        cpu_base, gpu = {}, {}
        for i, t in enumerate(spec.tensors):
            x = synth.teacher1_tensor(t, i, device)
            cpu_base[t.name] = x.cpu()
            gpu[t.name] = synth.perturb_(x, t, i, 0.01)
        # One encoder batch for the whole ~3 GB shard keeps the host arena in a
        # single chunk, so the arena that plan_view exposes (and this test
        # corrupts) is the one staged to the GPU, not a contiguous copy.
        delta = DeltaWeights(cpu_base, gpu, policy="auto", encode_batch_bytes=4 << 30)
        teacher2 = {k: v.clone() for k, v in gpu.items()}
        spot = None
        if scenario == "corrupt" and rank == 1:
            view = delta.plan_view()
            blocks = np.ctypeslib.as_array((ctypes.c_uint8 * (32 * view.nblocks)).from_address(view.blocks))
            blocks = blocks.view(ostream.BLOCK_DTYPE)
            arena = np.ctypeslib.as_array((ctypes.c_uint8 * view.arena_bytes).from_address(view.arena))
            k = next(i for i, b in enumerate(blocks) if b["kind"] != 0 and b["clen"] > 1024)
            spot = int(blocks[k]["src"]) + 256 + (2 * int(blocks[k]["nwords"]) - 256) // 2
            arena[spot] ^= 0x77
        failed = False
        try:
            delta.apply(reverse=True)
        except RuntimeError:
            failed = True
        outcome = "confirmed"
        try:
            delta.confirm(dist.group.WORLD, failed=failed)
        except RuntimeError as exc:
            outcome = f"unconfirmed: {exc}"
            if not failed:
                delta.apply(reverse=False)  # this rank switched: switch back to the source
        teachers_equal = {}
        for i, t in enumerate(spec.tensors):
            ref = synth.teacher1_tensor(t, i, device)
            teachers_equal[t.name] = (torch.equal(gpu[t.name].view(-1).view(torch.uint8), ref.view(-1).view(torch.uint8)),
                                      torch.equal(gpu[t.name].view(-1).view(torch.uint8),
                                                  teacher2[t.name].view(-1).view(torch.uint8)))
        on_a = all(a for a, _ in teachers_equal.values())
        on_b = all(b for _, b in teachers_equal.values())
        rollback = (delta.last_apply or {}).get("rollback")
        delta.close()
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, outcome, failed, rollback, on_a, on_b))
    except Exception:
        queue.put((rank, "crash: " + traceback.format_exc(), None, None, None, None))


def _run(scenario: str) -> dict[int, tuple]:
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, scenario, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, *rest = queue.get(timeout=300)
            results[rank] = tuple(rest)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return results


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("scenario", ["success", "corrupt"])
def test_two_gpu_ranks_switch_their_shards_and_confirm_over_nccl(scenario: str) -> None:
    results = _run(scenario)
    assert set(results) == {0, 1}
    for rank, (outcome, failed, rollback, on_a, on_b) in results.items():
        assert not outcome.startswith("crash"), outcome
        if scenario == "success":
            assert outcome == "confirmed" and not failed and on_a, (rank, outcome)
        else:
            assert outcome.startswith("unconfirmed") and "1 of 2" in outcome, (rank, outcome)
            assert failed == (rank == 1)
            assert on_b, rank  # every rank holds the source model (Teacher2) again
            if rank == 1:
                assert rollback == "restored"
