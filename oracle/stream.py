"""ORACLE — test infrastructure only. ctypes loader (and gcc build) for stream_oracle.c."""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "stream_oracle.c"
LIBRARY = HERE / "_build" / "libws_oracle.so"

BLOCK_DTYPE = np.dtype(
    [
        ("dst", "<u8"),
        ("src", "<u8"),
        ("nbytes", "<u4"),
        ("clen", "<u4"),
        ("nwords", "<u4"),
        ("kind", "<u2"),
        ("tail", "u1"),
        ("flags", "u1"),
    ]
)
TILE_DTYPE = np.dtype([("first_block", "<u4"), ("nblocks", "<u4"), ("table", "<u4"), ("split", "<u4")])
assert BLOCK_DTYPE.itemsize == 32 and TILE_DTYPE.itemsize == 16


def build(force: bool = False) -> Path:
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        LIBRARY.parent.mkdir(exist_ok=True)
        tmp = LIBRARY.with_suffix(".tmp")
        subprocess.run(
            ["gcc", "-O2", "-std=c11", "-shared", "-fPIC", "-pthread", "-o", str(tmp), str(SOURCE)], check=True
        )
        os.replace(tmp, LIBRARY)
    return LIBRARY


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P, U32, U64, I32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        _lib.wso_decode_words.argtypes = [P, U32, U32, U32, P, P]
        _lib.wso_decode_words.restype = I32
        _lib.wso_decode_dict_words.argtypes = [P, U32, U32, U32, P, P]
        _lib.wso_decode_dict_words.restype = I32
        _lib.wso_block_hash.argtypes = [P, U32, U64]
        _lib.wso_block_hash.restype = U64
        _lib.wso_apply_plan.argtypes = [P, U64, P, U64, P, P, ctypes.c_int64, I32, I32, ctypes.POINTER(U64)]
        _lib.wso_apply_plan.restype = I32
    return _lib


def decode_words(payload: np.ndarray, block: np.void, table512: np.ndarray) -> tuple[np.ndarray, int]:
    """Decode an ANS block's coded words; returns (uint16 words, error bits)."""
    nbytes = int(block["nbytes"])
    words = np.zeros(max(1, nbytes // 2), dtype="<u2")
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    table512 = np.ascontiguousarray(table512, dtype=np.uint32)
    decode = lib().wso_decode_dict_words if int(block["kind"]) in (3, 4) else lib().wso_decode_words
    err = decode(
        payload.ctypes.data, int(block["clen"]), int(block["nwords"]), nbytes, table512.ctypes.data, words.ctypes.data
    )
    return words[: nbytes // 2], err


def block_hash(data: np.ndarray, block_index: int) -> int:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    return int(lib().wso_block_hash(data.ctypes.data, data.size, block_index))


def apply_plan(blocks: np.ndarray, tiles: np.ndarray, tables: np.ndarray, arena: np.ndarray | int,
               dst_delta: int, reverse: bool, threads: int) -> tuple[int, int]:
    """Apply a whole plan on the host; returns (error bits, plan checksum)."""
    checksum = ctypes.c_uint64(0)
    arena_ptr = arena if isinstance(arena, int) else arena.ctypes.data
    err = lib().wso_apply_plan(
        blocks.ctypes.data, blocks.size, tiles.ctypes.data, tiles.size,
        tables.ctypes.data if tables.size else None, arena_ptr, dst_delta, int(reverse), threads,
        ctypes.byref(checksum),
    )
    return err, checksum.value
