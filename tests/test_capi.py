"""The C-ABI library loads without a GPU and exports every symbol include/warpshift_b200.h declares."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

from warpshift_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "warpshift_b200.h"


def declared() -> set[str]:
    return set(re.findall(r"^WS_API\s+(?:int|void)\s+(ws_\w+)\s*\(", HEADER.read_text(), flags=re.M))


def test_header_declares_the_api() -> None:
    names = declared()
    assert {"ws_plan_build", "ws_plan_upload", "ws_apply", "ws_last_error", "ws_plan_destroy"} <= names


def test_library_exports_every_declared_symbol() -> None:
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert declared() == set(_lib.SIGNATURES), "ctypes signatures must cover exactly the header"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIBRARY)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (ws_\w+)", out))
    assert exported == declared(), "the library must export exactly the declared ABI"


def test_version_and_error_buffer_without_a_gpu() -> None:
    lib = _lib.load()
    assert lib.ws_version() >= 100
    assert lib.ws_u16_residual(None, None, 3, None) == _lib.WS_ERR_INVALID
    assert "even" in _lib.last_error()


def test_self_test_rejects_bad_arguments_without_a_gpu() -> None:
    import ctypes

    lib = _lib.load()
    errors = ctypes.c_uint32(0)
    assert lib.ws_selftest_wait_timeout(0, 0, None, ctypes.byref(errors)) == _lib.WS_ERR_INVALID
    assert lib.ws_selftest_wait_timeout((1 << 20) + 1, 0, None, ctypes.byref(errors)) == _lib.WS_ERR_INVALID
    assert lib.ws_selftest_wait_timeout(10, 0, None, None) == _lib.WS_ERR_INVALID


def test_noalloc_rejects_bad_arguments_before_touching_a_gpu() -> None:
    """Host-side checks of the allocation-free apply: no CUDA call is made for
    these, so they run without a GPU."""
    import ctypes

    lib = _lib.load()
    res = _lib.ApplyResult()

    def call(tiles=16, ntiles=1, blocks=32, nblocks=1, tables=64, ntables=1, payload=48, nbytes=64, device=0, out=True):
        return lib.ws_apply_device_noalloc(tiles, ntiles, blocks, nblocks, tables, ntables, payload, nbytes, 0, device,
                                           None, ctypes.byref(res) if out else None)

    assert call(ntiles=0) == _lib.WS_OK  # nothing to do
    assert call(out=False) == _lib.WS_ERR_INVALID and "result pointer" in _lib.last_error()
    assert call(ntiles=_lib.WS_NOALLOC_MAX_TILES + 1) == _lib.WS_ERR_INVALID and "maximum" in _lib.last_error()
    for bad in ({"tiles": None}, {"blocks": None}, {"payload": None}, {"nblocks": 0}, {"nbytes": 0},
                {"tables": None}):
        assert call(**bad) == _lib.WS_ERR_INVALID, bad
    for misaligned in ({"tiles": 24}, {"blocks": 40}, {"payload": 56}, {"tables": 66}):
        assert call(**misaligned) == _lib.WS_ERR_INVALID, misaligned
        assert "aligned" in _lib.last_error()
    assert call(device=-1) == _lib.WS_ERR_INVALID and "device" in _lib.last_error()
    assert call(device=1 << 20) == _lib.WS_ERR_INVALID
