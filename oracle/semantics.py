"""ORACLE — test infrastructure only, never part of the product path.

NumPy restatement of the reference's delta semantics (DrRyanHuang/WarpShift,
``warpshift/delta.py``). Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import this module, and only as a checker.

Parity status: pinned. ``tests/golden/`` holds vectors produced by the reference
itself (``tests/golden/make_golden.py`` imports ``warpshift.delta`` from the
reference checkout and runs ``_u16_residual``, ``_batch_layout``,
``DeltaWeights._encode_chunk`` with a stub compressor, and the Triton kernel
``_restore_batch`` under ``TRITON_INTERPRET=1``); ``tests/test_oracle_golden.py``
checks every function below against them. The entropy stage of the reference is
nvCOMP's closed ANS codec; it has no golden vectors and is not restated here.
"""

from __future__ import annotations

from collections import Counter
from typing import Any, Callable

import numpy as np

CHUNK_BYTES = 16 * 1024**2  # delta.py:20
BATCH_BYTES = 64 * 1024**2  # delta.py:21
TILE_BYTES = 4096  # delta.py:22
MODES = {0: "XOR_RAW", 1: "XOR_GROUP2_ANS", 2: "XOR_ANS", 3: "U16_ANS"}  # delta.py:23
COMPRESS_MIN = 16384  # delta.py:185


def u16_residual(base: np.ndarray, target: np.ndarray) -> np.ndarray:
    """delta.py:26-34: low-byte plane then high-byte plane of zigzag((B - A) mod 2^16)."""
    b = base.view("<u2").astype(np.int64)
    t = target.view("<u2").astype(np.int64)
    d = ((t - b + 32768) & 65535) - 32768
    z = ((d << 1) ^ (d >> 15)) & 0xFFFF
    out = np.empty(z.size * 2, dtype=np.uint8)
    out[: z.size] = z & 0xFF
    out[z.size :] = z >> 8
    return out


def unzigzag_u16(residual: np.ndarray) -> np.ndarray:
    """delta.py:78-81: signed word deltas from grouped zigzag planes."""
    half = residual.size // 2
    z = residual[:half].astype(np.int64) | (residual[half : 2 * half].astype(np.int64) << 8)
    return (z >> 1) ^ -(z & 1)


def xor_residual(base: np.ndarray, target: np.ndarray) -> np.ndarray:
    """delta.py:180."""
    return np.bitwise_xor(base, target)


def group_planes(xor: np.ndarray) -> np.ndarray:
    """delta.py:186: even sizes are regrouped into low-byte and high-byte planes; odd sizes stay as is."""
    if xor.size % 2:
        return xor
    out = np.empty_like(xor)
    half = xor.size // 2
    out[:half] = xor[0::2]
    out[half:] = xor[1::2]
    return out


def encode_chunk(
    base: np.ndarray, target: np.ndarray, is_bf16: bool, compressed_size: Callable[[np.ndarray], int]
) -> tuple[int, np.ndarray, dict[int, np.ndarray]] | None:
    """delta.py:176-194 with the compressor replaced by ``compressed_size``.

    Returns (mode, residual handed to the compressor for that mode, all
    candidates tried), or None for an unchanged chunk.
    """
    xor = xor_residual(base, target)
    if not np.any(xor):
        return None
    mode, size, residual = 0, xor.size, xor
    candidates: dict[int, np.ndarray] = {}
    if xor.size >= COMPRESS_MIN:
        grouped = group_planes(xor)
        grouped_mode = 1 if xor.size % 2 == 0 else 2
        candidates[grouped_mode] = grouped
        c = compressed_size(grouped)
        if c < size:
            mode, size, residual = grouped_mode, c, grouped
        if is_bf16:
            u16 = u16_residual(base, target)
            candidates[3] = u16
            c = compressed_size(u16)
            if c < size:
                mode, size, residual = 3, c, u16
    return mode, residual, candidates


def encode_packets(
    cpu_base: dict[str, np.ndarray],
    target: dict[str, np.ndarray],
    bf16: dict[str, bool],
    compressed_size: Callable[[np.ndarray], int],
    chunk_bytes: int = CHUNK_BYTES,
) -> tuple[list[dict[str, Any]], Counter, int]:
    """delta.py:196-216 over uint8 views, in dict order; skipped chunks counted."""
    packets, counts, skipped = [], Counter(), 0
    for name, tgt in target.items():
        base = cpu_base[name]
        for offset in range(0, tgt.size, chunk_bytes):
            b = base[offset : offset + chunk_bytes]
            t = tgt[offset : offset + chunk_bytes]
            enc = encode_chunk(b, t, bf16[name], compressed_size)
            if enc is None:
                counts["SKIP"] += 1
                skipped += t.size
                continue
            mode, residual, _ = enc
            packets.append(dict(name=name, offset=offset, num_bytes=t.size, mode=mode, residual=residual))
            counts[MODES[mode]] += 1
    return packets, counts, skipped


def batch_layout(sizes: list[tuple[int, int]], limit: int = BATCH_BYTES) -> list[dict[str, Any]]:
    """delta.py:37-57: bounded batches of (encoded, decoded) frames, 256-byte aligned offsets."""
    batches: list[dict[str, Any]] = []
    packets: list[tuple[int, int, int]] = []
    used_in = used_out = payload = 0
    for index, (encoded, decoded) in enumerate(sizes):
        if min(encoded, decoded) < 0 or encoded == 0 or max(encoded, decoded) > limit:
            raise ValueError("Invalid delta frame size")
        in_off = -(-used_in // 256) * 256
        out_off = -(-used_out // 256) * 256
        if packets and max(in_off + encoded, out_off + decoded) > limit:
            batches.append(dict(payload_offset=payload, input_bytes=used_in, decoded_bytes=used_out, packets=packets))
            payload += used_in
            packets, in_off, out_off = [], 0, 0
        packets.append((index, in_off, out_off))
        used_in, used_out = in_off + encoded, out_off + decoded
    if packets:
        batches.append(dict(payload_offset=payload, input_bytes=used_in, decoded_bytes=used_out, packets=packets))
    return batches


def restore(dst: np.ndarray, mode: int, residual: np.ndarray, reverse: bool) -> None:
    """delta.py:74-92 for one packet, in place on a uint8 array of num_bytes."""
    n = dst.size
    if mode == 3:
        words = dst[: n - n % 2].view("<u2")
        d = unzigzag_u16(residual[: n - n % 2])
        w = words.astype(np.int64)
        w = (w - d) if reverse else (w + d)
        words[:] = (w % 65536).astype("<u2")
        return
    if mode == 1:
        i = np.arange(n)
        res = residual[i // 2 + (i % 2) * (n // 2)]
    else:
        res = residual[:n]
    np.bitwise_xor(dst, res, out=dst)


def apply_packets(tensors: dict[str, np.ndarray], packets: list[dict[str, Any]], reverse: bool) -> None:
    """delta.py:294-327 semantics on host arrays (uint8 views, modified in place)."""
    for p in packets:
        view = tensors[p["name"]][p["offset"] : p["offset"] + p["num_bytes"]]
        restore(view, p["mode"], p["residual"], reverse)
