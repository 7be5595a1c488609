"""ctypes bindings for ``libwarpshift_b200.so`` (declarations: include/warpshift_b200.h).

The library is built in-tree by ``python -m warpshift_b200.build``. There is no
fallback: if it is missing, every caller gets a RuntimeError naming the build
command.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libwarpshift_b200.so"

WS_OK, WS_ERR_INVALID, WS_ERR_CUDA, WS_ERR_DEVICE, WS_ERR_CHECKSUM, WS_ERR_NOMEM, WS_ERR_STATE, WS_ERR_IO = range(8)
POLICIES = {"auto": 0, "xor": 1, "u16": 2}
MODE_NAMES = ("XOR_RAW", "XOR_GROUP2_ANS", "XOR_ANS", "U16_ANS", "SKIP")

u64, u32, i32, i64, P = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class TensorDesc(ctypes.Structure):
    _fields_ = [("base", P), ("target", P), ("nbytes", u64), ("is_bf16", i32), ("reserved", i32)]


class BuildOptions(ctypes.Structure):
    _fields_ = [
        ("policy", i32),
        ("threads", i32),
        ("target_on_device", i32),
        ("device", i32),
        ("batch_bytes", u64),
        ("staging_slots", i32),
        ("pin_arena", i32),
        ("dict_slack_pct", i32),
        ("encode_on_device", i32),
        ("encode_batch_bytes", u64),
        ("escapes", i32),
        ("host_fallback", i32),
        ("split", i32),
    ]


class PlanStats(ctypes.Structure):
    _fields_ = [
        ("runtime_bytes", u64),
        ("skipped_bytes", u64),
        ("zero_block_bytes", u64),
        ("touched_bytes", u64),
        ("payload_bytes", u64),
        ("arena_bytes", u64),
        ("table_bytes", u64),
        ("metadata_bytes", u64),
        ("scratch_bytes", u64),
        ("mode_counts", u64 * 5),
        ("blocks", u64),
        ("tiles", u64),
        ("batches", u64),
        ("packets", u64),
        ("expected_checksum", u64 * 2),
        ("encode_seconds", ctypes.c_double),
        ("encoder", u32),
        ("reserved", u32),
    ]


class ApplyResult(ctypes.Structure):
    _fields_ = [
        ("checksum", u64),
        ("expected", u64),
        ("device_errors", u32),
        ("bad_block_plus1", u32),
        ("h2d_bytes", u64),
        ("launches", u32),
        ("rollback", u32),
    ]


ROLLBACK = {0: "none", 1: "restored", 2: "unverified", 3: "failed"}


class PlanView(ctypes.Structure):
    _fields_ = [
        ("blocks", P),
        ("nblocks", u64),
        ("tiles", P),
        ("ntiles", u64),
        ("tables", P),
        ("ntables", u64),
        ("arena", P),
        ("arena_bytes", u64),
    ]


# Every symbol declared in include/warpshift_b200.h, with its ctypes signature.
SIGNATURES = {
    "ws_version": ([], ctypes.c_int),
    "ws_last_error": ([ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "ws_u16_residual": ([P, P, u64, P], ctypes.c_int),
    "ws_plan_build": ([ctypes.POINTER(TensorDesc), u64, ctypes.POINTER(BuildOptions), P, ctypes.POINTER(P)], ctypes.c_int),
    "ws_plan_upload": ([P, P], ctypes.c_int),
    "ws_plan_set_resident": ([P, ctypes.c_int, P], ctypes.c_int),
    "ws_apply": ([P, ctypes.c_int, P, P, ctypes.POINTER(ApplyResult)], ctypes.c_int),
    "ws_apply_async": ([P, ctypes.c_int, P, P], ctypes.c_int),
    "ws_apply_finish": ([P, P, ctypes.POINTER(ApplyResult)], ctypes.c_int),
    "ws_plan_get_stats": ([P, ctypes.POINTER(PlanStats)], ctypes.c_int),
    "ws_plan_get_view": ([P, ctypes.POINTER(PlanView)], ctypes.c_int),
    "ws_plan_destroy": ([P], None),
    "ws_apply_device_noalloc": ([P, u32, P, u32, P, u32, P, u64, ctypes.c_int, ctypes.c_int, P, ctypes.POINTER(ApplyResult)], ctypes.c_int),
    "ws_plan_save": ([P, ctypes.c_char_p], ctypes.c_int),
    "ws_plan_load": ([ctypes.c_char_p, ctypes.POINTER(TensorDesc), u64, ctypes.POINTER(BuildOptions), ctypes.POINTER(P)], ctypes.c_int),
    "ws_selftest_wait_timeout": ([u32, ctypes.c_int, P, ctypes.POINTER(u32)], ctypes.c_int),
    "ws_tensor_hashes": ([ctypes.POINTER(P), ctypes.POINTER(u64), u64, ctypes.c_int, P, ctypes.POINTER(u64)], ctypes.c_int),
}
WS_NOALLOC_MAX_TILES = 16384
WS_DEVERR_BOUNDS = 16
ENCODERS = {0: "host", 1: "gpu", 2: "loaded"}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the native library (raises RuntimeError if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise RuntimeError(
                    f"{LIBRARY.name} is missing: build it with `python -m warpshift_b200.build` "
                    "(warpshift_b200 has no CPU or Triton fallback)"
                )
            lib = ctypes.CDLL(str(LIBRARY))
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
        return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().ws_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    """Map a WS_* status to the reference's exception types (ValueError for layout, else RuntimeError)."""
    if rc == WS_OK:
        return
    message = last_error()
    if rc == WS_ERR_INVALID:
        raise ValueError(message)
    if rc == WS_ERR_IO:
        raise OSError(message)
    raise RuntimeError(message)
