"""A failed switch is rolled back: after a device error or a checksum mismatch
the weights hold, bit for bit, the bytes that were resident before the call.

Faults are injected on the host only: a flipped byte of the pinned payload
arena (the kernel then decodes garbage into one block, which its final-state
check reports), or one resident weight byte changed before the switch (the
written bytes then miss the checksum recorded at prepare). Neither faults the
GPU; every kernel access stays inside its block and staging ring.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import stream as ostream
from tests.helpers import as_bytes, edge_pair
from warpshift_b200.delta import DeltaWeights

pytestmark = pytest.mark.gpu


def blocks_and_arena(delta: DeltaWeights):
    view = delta.plan_view()
    blocks = np.ctypeslib.as_array((ctypes.c_uint8 * (32 * view.nblocks)).from_address(view.blocks))
    arena = np.ctypeslib.as_array((ctypes.c_uint8 * view.arena_bytes).from_address(view.arena))
    return blocks.view(ostream.BLOCK_DTYPE), arena


def snapshot(gpu: dict[str, torch.Tensor]) -> dict[str, np.ndarray]:
    return {k: as_bytes(v).copy() for k, v in gpu.items()}


def assert_same(gpu: dict[str, torch.Tensor], want: dict[str, np.ndarray]) -> None:
    for name, t in gpu.items():
        np.testing.assert_array_equal(as_bytes(t), want[name], err_msg=name)


@pytest.mark.parametrize("policy", ["xor", "u16"])
@pytest.mark.parametrize("reverse", [True, False])
def test_corrupt_stream_switch_is_rolled_back_exactly(cuda_device, policy: str, reverse: bool) -> None:
    a, b = edge_pair(seed=11, big=False)
    gpu = {k: v.to(cuda_device) for k, v in b.items()}
    delta = DeltaWeights(a, gpu, policy=policy)
    if not reverse:
        delta.apply(reverse=True)  # resident: Teacher1, so the failing switch runs A -> B
    before = snapshot(gpu)
    blocks, arena = blocks_and_arena(delta)
    coded = [i for i, bk in enumerate(blocks) if bk["kind"] != 0 and bk["clen"] > 1024]
    assert coded
    # Corrupt a renormalisation word in the middle of the stream of two coded
    # blocks (first and last): past the 256-byte state header, before any escape list.
    spots = [int(blocks[i]["src"]) + 256 + (2 * int(blocks[i]["nwords"]) - 256) // 2 for i in (coded[0], coded[-1])]
    for s in spots:
        arena[s] ^= 0x5A
    with pytest.raises(RuntimeError, match="rolled back"):
        delta.apply(reverse=reverse)
    assert not delta.last_apply["ok"]
    assert delta.last_apply["rollback"] == "restored"
    assert_same(gpu, before)
    for s in spots:
        arena[s] ^= 0x5A
    # The package is intact again and switches exactly.
    delta.apply(reverse=reverse)
    assert_same(gpu, {k: as_bytes(v) for k, v in (a if reverse else b).items()})


def test_checksum_mismatch_is_rolled_back_to_the_resident_bytes(cuda_device) -> None:
    a, b = edge_pair(seed=12, big=False)
    gpu = {k: v.to(cuda_device) for k, v in b.items()}
    delta = DeltaWeights(a, gpu, policy="auto")
    name = max(gpu, key=lambda k: gpu[k].numel())
    flat = gpu[name].view(-1).view(torch.uint8)
    flat[1001] ^= 0x40  # the resident model is no longer the package's source
    before = snapshot(gpu)
    with pytest.raises(RuntimeError, match="checksum mismatch"):
        delta.apply(reverse=True)
    assert delta.last_apply["rollback"] == "unverified"  # restored bytes are not the source model's
    assert_same(gpu, before)
    flat[1001] ^= 0x40
    delta.apply(reverse=True)
    assert_same(gpu, {k: as_bytes(v) for k, v in a.items()})
