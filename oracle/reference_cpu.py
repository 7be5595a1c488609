"""ORACLE — test infrastructure only, never part of the product path.

The reference's switch path restated for host cores: what ``bench.py`` times as
the reference arm and as ``cpu_baseline``, and what ``tests/`` checks against
the golden-pinned ``oracle.semantics``. Nothing here loads the product library.

The reference (``warpshift/delta.py``) switches by decoding each packet's
residual with nvCOMP into a scratch buffer (delta.py:313-316) and running the
Triton kernel ``_restore_batch`` over it (delta.py:60-92, launched at 317-324).
nvCOMP is a closed GPU codec with no CPU counterpart, so the host path starts
from the decoded residuals, exactly as ``_restore_batch`` receives them:

* mode 0 / 2: the raw XOR bytes (delta.py:180, 189);
* mode 1: the XOR regrouped into a low-byte plane then a high-byte plane
  (delta.py:186), de-interleaved by the restore (``i // 2 + (i % 2) * (n / 2)``,
  delta.py:88-90);
* mode 3: the zigzag planes of ``_u16_residual`` (delta.py:26-34), applied as a
  wrapping uint16 add (forward) or subtract (reverse) (delta.py:77-85).

``restore_packet`` computes the same bytes as ``oracle.semantics.restore`` (the
literal restatement the golden vectors pin) with uint16 views instead of index
arrays, in slices that stay in the host caches, so its time measures the
restore itself rather than NumPy temporaries. ``CpuSwitch`` runs one switch
over a whole set of packets on a thread pool (NumPy releases the GIL inside
its array loops).

Mode choice follows delta.py:176-194 (raw XOR below 16384 bytes; otherwise the
grouped/odd XOR candidate, then U16 for BF16, strictly-smaller wins). The
reference ranks candidates by nvCOMP's compressed size; here the stand-in size
is the order-0 byte entropy of the candidate (``order0_bytes``), which is what
an ANS coder approaches. The ``xor`` and ``u16`` policies restrict the
candidates as the product's policies do.
"""

from __future__ import annotations

import math
import os
import time
from concurrent.futures import ThreadPoolExecutor
from typing import Callable

import numpy as np

from . import semantics as sem

SLICE_WORDS = 1 << 17  # 256 KiB of weights per restore step: operands and temporaries stay in cache


def order0_bytes(residual: np.ndarray) -> int:
    """Order-0 byte entropy of ``residual`` in bytes: the compressed-size stand-in for nvCOMP ANS."""
    counts = np.bincount(residual, minlength=256).astype(np.float64)
    p = counts[counts > 0] / residual.size
    return int(math.ceil(-(p * np.log2(p)).sum() * residual.size / 8))


def choose_packet(base: np.ndarray, target: np.ndarray, is_bf16: bool, policy: str = "xor",
                  compressed_size: Callable[[np.ndarray], int] = order0_bytes) -> tuple[int, np.ndarray] | None:
    """(mode, residual handed to the restore) for one packet, or None when unchanged (delta.py:176-194)."""
    if policy == "auto":
        enc = sem.encode_chunk(base, target, is_bf16, compressed_size)
        return None if enc is None else (enc[0], enc[1])
    xor = sem.xor_residual(base, target)
    if not xor.any():
        return None
    if xor.size < sem.COMPRESS_MIN:
        return 0, xor
    if policy == "u16" and is_bf16 and xor.size % 2 == 0:
        return 3, sem.u16_residual(base, target)
    grouped = sem.group_planes(xor)
    return (1 if xor.size % 2 == 0 else 2), grouped


def restore_packet(dst: np.ndarray, mode: int, residual: np.ndarray, reverse: bool) -> None:
    """delta.py:74-92 on one packet of uint8 ``dst`` (in place); same bytes as ``semantics.restore``."""
    n = dst.size
    if mode == 3 and n % 2:
        raise ValueError("U16 packets have an even byte count (delta.py:190)")
    if mode in (0, 2) or (mode == 1 and n % 2):
        for s in range(0, n, 2 * SLICE_WORDS):
            np.bitwise_xor(dst[s : s + 2 * SLICE_WORDS], residual[s : s + 2 * SLICE_WORDS], out=dst[s : s + 2 * SLICE_WORDS])
        return
    half = n // 2
    words = dst[: 2 * half].view("<u2")
    lo, hi = residual[:half], residual[half : 2 * half]
    for s in range(0, half, SLICE_WORDS):
        e = min(half, s + SLICE_WORDS)
        z = hi[s:e].astype(np.uint16)
        z <<= 8
        z |= lo[s:e]
        w = words[s:e]
        if mode == 1:
            w ^= z
            continue
        # mode 3: d = unzigzag(z) = (z >> 1) ^ -(z & 1), added or subtracted modulo 2^16
        sign = np.bitwise_and(z, 1)
        np.negative(sign, out=sign)
        z >>= 1
        z ^= sign
        if reverse:
            w -= z
        else:
            w += z


def packets_of(base: dict[str, np.ndarray], target: dict[str, np.ndarray], bf16: dict[str, bool], policy: str,
               threads: int) -> list[tuple[str, int, int, np.ndarray]]:
    """Every changed 16 MiB packet of the pair as (name, offset, mode, residual), in dict order."""
    jobs = [(name, off) for name, t in target.items() for off in range(0, t.size, sem.CHUNK_BYTES)]

    def one(job):
        name, off = job
        b = base[name][off : off + sem.CHUNK_BYTES]
        t = target[name][off : off + sem.CHUNK_BYTES]
        got = choose_packet(b, t, bf16[name], policy)
        return None if got is None else (name, off, got[0], got[1])

    with ThreadPoolExecutor(max(1, threads)) as pool:
        return [p for p in pool.map(one, jobs) if p is not None]


class CpuSwitch:
    """The reference's restore over a set of resident host tensors, one switch per call."""

    def __init__(self, tensors: dict[str, np.ndarray], packets: list[tuple[str, int, int, np.ndarray]],
                 threads: int | None = None) -> None:
        self.tensors = tensors
        self.packets = packets
        self.cores = threads or len(os.sched_getaffinity(0))
        self.bytes = sum(t.size for t in tensors.values())
        self.reverse = True  # the tensors hold Teacher2

    def _run(self, threads: int) -> None:
        reverse = self.reverse

        def one(p):
            name, off, mode, residual = p
            restore_packet(self.tensors[name][off : off + residual.size], mode, residual, reverse)

        if threads == 1:
            for p in self.packets:
                one(p)
        else:
            with ThreadPoolExecutor(threads) as pool:
                list(pool.map(one, self.packets))

    def switch(self, threads: int | None = None) -> float:
        """One switch (Teacher2 -> Teacher1 or back, alternating); returns seconds."""
        t0 = time.perf_counter()
        self._run(threads or self.cores)
        dt = time.perf_counter() - t0
        self.reverse = not self.reverse
        return dt
