"""ORACLE — test infrastructure only, never part of the product path.

NumPy restatement of the per-tensor content hash that ``ws_tensor_hashes``
computes on the GPU (the device-side replacement for the sha256 of every tensor
in the reference's acceptance check, ``scripts/validate.py:50-56``). The hash is
this project's own definition, so there is no reference output to pin it to;
``tests/test_hash_cpu.py`` checks this vectorised form against a word-by-word
Python loop and the GPU tests check the kernel against it.

    w_j  = little-endian 64-bit words of the bytes, the last one zero-padded
    sum  = sum_j xmul(w_j ^ ((j + 1) * KPOS))         (mod 2^64)
    hash = mix64(sum + (nbytes + 1) * KLEN)           (mod 2^64)

xmul(x) = y ^ (y >> 32) with y = x * KMUL (mod 2^64): one multiply by an odd
constant and a fold of the high half into the low half, both bijections, per
word. mix64, applied once per tensor, is the splitmix64 finaliser (Steele, Lea
and Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014;
constants as published).
"""

from __future__ import annotations

import numpy as np

KPOS = 0xC2B2AE3D27D4EB4F
KLEN = 0x165667B19E3779F9
KMUL = 0x9E3779B97F4A7C15
MASK = (1 << 64) - 1


def mix64_int(x: int) -> int:
    x &= MASK
    x ^= x >> 30
    x = (x * 0xBF58476D1CE4E5B9) & MASK
    x ^= x >> 27
    x = (x * 0x94D049BB133111EB) & MASK
    return x ^ (x >> 31)


def xmul_int(x: int) -> int:
    y = ((x & MASK) * KMUL) & MASK
    return y ^ (y >> 32)


def _xmul(x: np.ndarray) -> np.ndarray:
    y = x * np.uint64(KMUL)
    return y ^ (y >> np.uint64(32))


def tensor_hash(data: bytes | np.ndarray) -> int:
    """Hash of a byte string (vectorised; uint64 arithmetic wraps mod 2^64)."""
    raw = np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else data.reshape(-1).view(np.uint8)
    n = raw.size
    total = 0
    if n:
        padded = np.zeros((n + 7) // 8 * 8, dtype=np.uint8)
        padded[:n] = raw
        words = padded.view("<u8")
        pos = np.arange(1, words.size + 1, dtype=np.uint64) * np.uint64(KPOS)
        with np.errstate(over="ignore"):
            terms = _xmul(words ^ pos)
        total = int(terms.sum(dtype=np.uint64))
    return mix64_int(total + (n + 1) * KLEN)


def tensor_hash_loop(data: bytes) -> int:
    """The same hash word by word in plain Python (small inputs only)."""
    n = len(data)
    total = 0
    for j in range(0, n, 8):
        w = int.from_bytes(data[j : j + 8].ljust(8, b"\0"), "little")
        total += xmul_int(w ^ (((j // 8 + 1) * KPOS) & MASK))
    return mix64_int(total + (n + 1) * KLEN)


def hex_hash(data: bytes | np.ndarray) -> str:
    return f"{tensor_hash(data):016x}"
