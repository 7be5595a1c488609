"""GPU test of ws_apply_device_noalloc, the allocation-free apply entry point.

Callers such as a serving engine whose KV-cache pool already holds all free HBM
(or one that owns every device allocation through its own allocator) cannot let
the library call cudaMalloc when they switch models. For them the library
exposes one entry point that takes descriptors, tables and payload already in
the caller's device memory and keeps its only scratch in a fixed device array
inside the library. This file checks, through the C ABI, that two calls in a
row write exactly the bytes (and report exactly the checksum) of the plan-based
entry point ws_apply, that the second call changes no free device memory, and
that oversized requests are rejected. Bytes are compared bit-exactly, as in
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


def build_device_plan(a, targets, device):
    """Host-side plan for `targets` (device tensors), its arrays copied into caller-owned torch memory."""
    lib = _lib.load()
    descs = (_lib.TensorDesc * len(a))()
    for i, name in enumerate(targets):
        t = targets[name]
        descs[i] = _lib.TensorDesc(a[name].data_ptr(), t.data_ptr(), t.numel() * t.element_size(),
                                   int(t.dtype == torch.bfloat16), 0)
    opts = _lib.BuildOptions(policy=_lib.POLICIES["auto"], threads=0, target_on_device=1, device=device.index,
                             batch_bytes=0, staging_slots=0, pin_arena=0)
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
        "expected": (int(stats.expected_checksum[0]), int(stats.expected_checksum[1])),
    }
    lib.ws_plan_destroy(plan)
    return dev


def call_noalloc(dev, reverse: bool, device) -> _lib.ApplyResult:
    result = _lib.ApplyResult()
    rc = _lib.load().ws_apply_device_noalloc(
        dev["tiles"].data_ptr(), dev["ntiles"], dev["blocks"].data_ptr(), dev["tables"].data_ptr(),
        dev["payload"].data_ptr(), int(reverse), device.index, torch.cuda.current_stream(device).cuda_stream,
        ctypes.byref(result),
    )
    _lib.check(rc)
    return result


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
        result = call_noalloc(dev, reverse, cuda_device)
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
        dummy.data_ptr(), _lib.WS_NOALLOC_MAX_TILES + 1, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 0,
        cuda_device.index, torch.cuda.current_stream(cuda_device).cuda_stream, ctypes.byref(result),
    )
    assert rc == _lib.WS_ERR_INVALID
    assert "exceed the maximum" in _lib.last_error()
