"""Per-tensor content hash: the oracle's vectorised form against a word-by-word
loop, and the C ABI's host-side handling (empty tensors, bad arguments)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import torch

from oracle import hashes
from warpshift_b200 import _lib
from warpshift_b200.verify import tensor_hashes


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 15, 16, 17, 255, 4096, 65535, 65536, 65537, 200_003])
def test_vectorised_hash_matches_the_loop(n: int) -> None:
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert hashes.tensor_hash(data) == hashes.tensor_hash_loop(data)


def test_hash_separates_length_position_and_content() -> None:
    base = bytes(range(256)) * 64
    seen = {hashes.tensor_hash(base)}
    for variant in (base[:-1], base + b"\0", base[8:] + base[:8], base[:100] + b"\x01" + base[101:]):
        h = hashes.tensor_hash(variant)
        assert h not in seen
        seen.add(h)
    assert hashes.tensor_hash(b"") != hashes.tensor_hash(b"\0" * 8)


def test_empty_tensors_need_no_device() -> None:
    lib = _lib.load()
    ptrs = (ctypes.c_void_p * 2)(None, None)
    sizes = (ctypes.c_uint64 * 2)(0, 0)
    out = (ctypes.c_uint64 * 2)()
    assert lib.ws_tensor_hashes(ptrs, sizes, 2, 0, None, out) == _lib.WS_OK
    assert list(out) == [hashes.tensor_hash(b"")] * 2
    assert lib.ws_tensor_hashes(None, None, 0, 0, None, None) == _lib.WS_OK


def test_null_pointer_is_rejected() -> None:
    lib = _lib.load()
    ptrs = (ctypes.c_void_p * 1)(None)
    sizes = (ctypes.c_uint64 * 1)(16)
    out = (ctypes.c_uint64 * 1)()
    assert lib.ws_tensor_hashes(ptrs, sizes, 1, 0, None, out) == _lib.WS_ERR_INVALID
    assert "null pointer" in _lib.last_error()


def test_cpu_tensors_are_rejected() -> None:
    with pytest.raises(ValueError, match="CUDA"):
        tensor_hashes({"w": torch.zeros(4)})
