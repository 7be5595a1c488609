"""GPU test of ws_apply_device_noalloc, the allocation-free apply entry point.

Callers such as a serving engine whose KV-cache pool already holds all free HBM
(or one that owns every device allocation through its own allocator) cannot let
the library call cudaMalloc when they switch models. For them the library
exposes one entry point that takes descriptors, tables and payload already in
the caller's device memory and keeps its only scratch in a fixed device array
inside the library. This file checks, through the C ABI, that two calls in a
row write exactly the bytes (and report exactly the checksum) of the plan-based
entry point ws_apply, that the second call changes no free device memory, that
oversized requests are rejected, that a corrupt block comes back as a device
error naming it, and that descriptors pointing outside the caller's arrays are
refused on the device without being followed. Bytes are compared bit-exactly, as in
every parity test of this repository. The file is named so pytest collects it
last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import as_bytes, edge_pair, plan_arrays
from warpshift_b200 import _lib
from warpshift_b200.delta import DeltaWeights

pytestmark = pytest.mark.gpu


def build_device_plan(a, targets, device, policy: str = "auto", split: int = 0):
    """Host-side plan for `targets` (device tensors), its arrays copied into caller-owned torch memory."""
    lib = _lib.load()
    descs = (_lib.TensorDesc * len(a))()
    for i, name in enumerate(targets):
        t = targets[name]
        descs[i] = _lib.TensorDesc(a[name].data_ptr(), t.data_ptr(), t.numel() * t.element_size(),
                                   int(t.dtype == torch.bfloat16), 0)
    opts = _lib.BuildOptions(policy=_lib.POLICIES[policy], threads=0, target_on_device=1, device=device.index,
                             batch_bytes=0, staging_slots=0, pin_arena=0, split=split)
    plan = ctypes.c_void_p()
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check(lib.ws_plan_build(descs, len(a), ctypes.byref(opts), stream, ctypes.byref(plan)))
    blocks, tiles, tables, arena, stats = plan_arrays(plan)
    dev = {
        "blocks": torch.from_numpy(blocks.view(np.uint8).copy()).to(device),
        "tiles": torch.from_numpy(tiles.view(np.uint8).copy()).to(device),
        "tables": torch.from_numpy(tables.copy() if tables.size else np.zeros(1, np.uint32)).view(torch.int32).to(device),
        "payload": torch.from_numpy(arena.copy() if arena.size else np.zeros(16, np.uint8)).to(device),
        "ntiles": int(tiles.size),
        "nblocks": int(blocks.size),
        "ntables": int(tables.size // 512),
        "host_blocks": blocks.copy(),
        "host_tiles": tiles.copy(),
        "expected": (int(stats.expected_checksum[0]), int(stats.expected_checksum[1])),
    }
    lib.ws_plan_destroy(plan)
    return dev


def call_noalloc(dev, reverse: bool, device, check: bool = True) -> tuple[int, _lib.ApplyResult]:
    result = _lib.ApplyResult()
    rc = _lib.load().ws_apply_device_noalloc(
        dev["tiles"].data_ptr(), dev["ntiles"], dev["blocks"].data_ptr(), dev["nblocks"], dev["tables"].data_ptr(),
        dev["ntables"], dev["payload"].data_ptr(), dev["payload"].numel(), int(reverse), device.index,
        torch.cuda.current_stream(device).cuda_stream, ctypes.byref(result),
    )
    if check:
        _lib.check(rc)
    return rc, result


def test_noalloc_matches_plan_apply_on_two_calls(cuda_device) -> None:
    a, b = edge_pair(seed=21, big=True)
    with_plan = {k: v.to(cuda_device) for k, v in b.items()}
    without_alloc = {k: v.to(cuda_device) for k, v in b.items()}
    delta = DeltaWeights(a, with_plan, policy="auto")
    dev = build_device_plan(a, without_alloc, cuda_device)
    assert dev["ntiles"] > 1
    for call, (reverse, teacher) in enumerate(((True, a), (False, b))):
        delta.apply(reverse=reverse)
        torch.cuda.synchronize(cuda_device)
        free_before = torch.cuda.mem_get_info(cuda_device)[0]
        _, result = call_noalloc(dev, reverse, cuda_device)
        free_after = torch.cuda.mem_get_info(cuda_device)[0]
        if call == 1:  # the first call may load the module's fixed array; later calls allocate nothing
            assert free_after == free_before
        assert result.device_errors == 0 and result.launches == 2
        assert result.checksum == delta.last_apply["checksum"] == dev["expected"][int(reverse)]
        for name in b:
            got = as_bytes(without_alloc[name])
            np.testing.assert_array_equal(got, as_bytes(with_plan[name]), err_msg=name)
            np.testing.assert_array_equal(got, as_bytes(teacher[name]), err_msg=name)


def test_noalloc_rejects_more_tiles_than_its_fixed_scratch(cuda_device) -> None:
    dummy = torch.zeros(64, dtype=torch.uint8, device=cuda_device)
    result = _lib.ApplyResult()
    rc = _lib.load().ws_apply_device_noalloc(
        dummy.data_ptr(), _lib.WS_NOALLOC_MAX_TILES + 1, dummy.data_ptr(), 1, dummy.data_ptr(), 1, dummy.data_ptr(), 64,
        0, cuda_device.index, torch.cuda.current_stream(cuda_device).cuda_stream, ctypes.byref(result),
    )
    assert rc == _lib.WS_ERR_INVALID
    assert "exceed the maximum" in _lib.last_error()


def test_noalloc_reports_a_corrupt_block_with_its_index(cuda_device) -> None:
    """A flipped payload byte of one coded block comes back as a device error
    naming that block, through the per-tile slots and their reduction."""
    a, b = edge_pair(seed=22, big=False)
    targets = {k: v.to(cuda_device) for k, v in b.items()}
    dev = build_device_plan(a, targets, cuda_device)
    coded = [i for i, bk in enumerate(dev["host_blocks"]) if bk["kind"] != 0 and bk["clen"] > 1024]
    assert coded
    victim = coded[len(coded) // 2]
    bk = dev["host_blocks"][victim]
    spot = int(bk["src"]) + 256 + (2 * int(bk["nwords"]) - 256) // 2
    dev["payload"][spot] ^= 0x3C
    rc, result = call_noalloc(dev, True, cuda_device, check=False)
    assert rc == _lib.WS_ERR_DEVICE
    assert result.device_errors & 3 and result.bad_block_plus1 == victim + 1
    assert "corrupt block" in _lib.last_error()


@pytest.mark.parametrize("field", ["tile_first_block", "block_src", "block_src_misaligned", "tile_table"])
def test_noalloc_refuses_descriptors_outside_the_arrays(cuda_device, field: str) -> None:
    """Caller-written descriptors that point outside the given arrays are
    reported as WS_DEVERR_BOUNDS and never followed: the weights stay as they were."""
    a, b = edge_pair(seed=23, big=False)
    targets = {k: v.to(cuda_device) for k, v in b.items()}
    dev = build_device_plan(a, targets, cuda_device)
    before = {k: as_bytes(v).copy() for k, v in targets.items()}
    tiles, blocks = dev["host_tiles"].copy(), dev["host_blocks"].copy()
    coded_tile = next(i for i, t in enumerate(tiles) if t["table"] != 0xFFFFFFFF)
    if field == "tile_first_block":
        tiles[0]["first_block"] = dev["nblocks"]
    elif field == "tile_table":
        tiles[coded_tile]["table"] = dev["ntables"]
    elif field == "block_src":
        blocks[0]["src"] = dev["payload"].numel() - 16
        blocks[0]["clen"] = max(32, int(blocks[0]["clen"]))
    else:
        blocks[0]["src"] = int(blocks[0]["src"]) + 8
    dev["tiles"] = torch.from_numpy(tiles.view(np.uint8).copy()).to(cuda_device)
    dev["blocks"] = torch.from_numpy(blocks.view(np.uint8).copy()).to(cuda_device)
    rc, result = call_noalloc(dev, True, cuda_device, check=False)
    assert rc == _lib.WS_ERR_DEVICE
    assert result.device_errors & _lib.WS_DEVERR_BOUNDS
    assert "outside the given arrays" in _lib.last_error()
    assert result.bad_block_plus1 >= 1
    # The refused tile's blocks (or the refused block) were not written.
    if field.startswith("tile"):
        orig = dev["host_tiles"][coded_tile if field == "tile_table" else 0]
        refused = range(int(orig["first_block"]), int(orig["first_block"]) + int(orig["nblocks"]))
    else:
        refused = [0]
    bases = {n: t.data_ptr() for n, t in targets.items()}
    for i in refused:
        dst = int(dev["host_blocks"][i]["dst"])
        owner = max((n for n in bases if bases[n] <= dst), key=lambda n: bases[n])
        off, n = dst - bases[owner], int(dev["host_blocks"][i]["nbytes"])
        np.testing.assert_array_equal(as_bytes(targets[owner])[off : off + n], before[owner][off : off + n])


@pytest.mark.parametrize("split", [2, 7])
def test_noalloc_refuses_a_tile_split_code_its_blocks_do_not_have(cuda_device, split: int) -> None:
    """A tile's split code names the raw-bit table its split-word blocks are
    expanded with: blocks of another code are reported as WS_DEVERR_KIND and a
    code that is not one of 0..3 refuses the tile (WS_DEVERR_BOUNDS); neither
    writes the weights."""
    from tests.helpers import bf16_pair, split_bits

    x, y = bf16_pair(3 << 20, 0.01, 24)  # XOR s = 0.01: split words, k = 1
    targets = {"w": y.to(cuda_device)}
    dev = build_device_plan({"w": x}, targets, cuda_device, policy="xor", split=1)
    tiles = dev["host_tiles"].copy()
    victim = next(i for i, t in enumerate(tiles) if t["split"] == 1)
    first, count = int(tiles[victim]["first_block"]), int(tiles[victim]["nblocks"])
    assert all(split_bits(dev["host_blocks"][i]["flags"]) == 1 for i in range(first, first + count))
    tiles[victim]["split"] = split
    dev["tiles"] = torch.from_numpy(tiles.view(np.uint8).copy()).to(cuda_device)
    before = as_bytes(targets["w"]).copy()
    rc, result = call_noalloc(dev, True, cuda_device, check=False)
    assert rc == _lib.WS_ERR_DEVICE
    assert result.device_errors & (_lib.WS_DEVERR_BOUNDS if split > 3 else 8)
    base = targets["w"].data_ptr()
    for i in range(first, first + count):
        off, n = int(dev["host_blocks"][i]["dst"]) - base, int(dev["host_blocks"][i]["nbytes"])
        np.testing.assert_array_equal(as_bytes(targets["w"])[off : off + n], before[off : off + n])
