"""Saved delta packages on the GPU: DeltaWeights.save / DeltaWeights.load.

A package saved after prepare and loaded onto fresh copies of the resident
weights (new addresses) switches both ways bit-exactly; loading it onto weights
that are not the expected source is caught by the apply checksum; a GPU-encoded
plan whose arena spans several host chunks saves and loads unchanged.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from tests.helpers import as_bytes, bf16_pair, edge_pair, plan_arrays
from warpshift_b200 import _lib
from warpshift_b200.delta import DeltaWeights

pytestmark = pytest.mark.gpu


def same(got: dict, want: dict) -> None:
    for name in want:
        np.testing.assert_array_equal(as_bytes(got[name]), as_bytes(want[name]), err_msg=name)


def test_saved_package_switches_fresh_weights(cuda_device, tmp_path) -> None:
    a, b = edge_pair(seed=19)
    gpu = {k: v.to(cuda_device) for k, v in b.items()}
    delta = DeltaWeights(a, gpu)
    path = tmp_path / "qwen_edge.wsd"
    delta.save(path)
    stats = dict(delta.stats)
    del delta
    fresh = {k: v.to(cuda_device).clone() for k, v in b.items()}
    del gpu
    loaded = DeltaWeights.load(path, fresh)
    assert loaded.stats["encoder"] == "loaded"
    for key in ("transferred_bytes", "mode_counts", "touched_bytes", "blocks", "skipped_bytes"):
        assert loaded.stats[key] == stats[key], key
    loaded.apply(reverse=True)
    same(fresh, a)
    loaded.apply(reverse=False)
    same(fresh, b)
    loaded.set_resident(True)
    loaded.apply(reverse=True)
    same(fresh, a)


def test_loading_onto_the_wrong_source_is_caught(cuda_device, tmp_path) -> None:
    x, y = bf16_pair(3 << 20, 0.01, 8)
    gpu = {"w": y.to(cuda_device)}
    path = tmp_path / "w.wsd"
    DeltaWeights({"w": x}, gpu).save(path)
    holding_a = {"w": x.to(cuda_device)}
    loaded = DeltaWeights.load(path, holding_a)
    with pytest.raises(RuntimeError, match="checksum"):
        loaded.apply(reverse=True)  # B -> A, but A is resident
    with pytest.raises(ValueError, match="differs from the saved plan"):
        DeltaWeights.load(path, {"w": torch.zeros(5, dtype=torch.bfloat16, device=cuda_device)})


def test_multi_chunk_gpu_plan_saves_and_loads_unchanged(cuda_device, tmp_path) -> None:
    x, y = bf16_pair((40 << 20) // 2 + 5, 0.01, 9)
    lib = _lib.load()
    target = y.to(cuda_device)
    descs = (_lib.TensorDesc * 1)(_lib.TensorDesc(x.data_ptr(), target.data_ptr(), target.numel() * 2, 1, 0))
    opts = _lib.BuildOptions(policy=0, threads=4, target_on_device=1, device=cuda_device.index or 0, batch_bytes=0,
                             staging_slots=0, pin_arena=1, dict_slack_pct=6, encode_on_device=1,
                             encode_batch_bytes=16 << 20)
    plan, loaded = ctypes.c_void_p(), ctypes.c_void_p()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.ws_plan_build(descs, 1, ctypes.byref(opts), stream, ctypes.byref(plan)))
    try:
        path = tmp_path / "chunks.wsd"
        _lib.check(lib.ws_plan_save(plan, os.fsencode(path)))
        _lib.check(lib.ws_plan_load(os.fsencode(path), descs, 1, ctypes.byref(opts), ctypes.byref(loaded)))
        for got, want in zip(plan_arrays(loaded)[:4], plan_arrays(plan)[:4]):
            np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))
    finally:
        lib.ws_plan_destroy(plan)
        lib.ws_plan_destroy(loaded)
