"""Test helpers: seeded tensor pairs covering the edge cases of the reference path."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import stream as ostream
from warpshift_b200 import _lib
from warpshift_b200.delta import _BLOCK_BYTES

BLOCK_WORDS = _BLOCK_BYTES // 2  # 16-bit words per rANS block


def bf16_pair(numel: int, scale: float, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(numel, generator=g) * 0.02).to(torch.bfloat16)
    f = a.float()
    b = (f + scale * f.abs() * torch.randn(numel, generator=g)).to(torch.bfloat16)
    return a, b


def edge_pair(seed: int = 0, scale: float = 0.01, big: bool = True) -> tuple[dict[str, torch.Tensor], dict[str, torch.Tensor]]:
    """CPU A/B dicts with every size class the reference path distinguishes.

    Tiny raw-XOR tensors (< 16384 B, delta.py:185), the 16383/16384 boundary,
    odd byte counts (mode 2, delta.py:186/189), fp32 and uint8 tensors (XOR only,
    delta.py:190), unchanged tensors (SKIP, delta.py:181), partial 512-byte groups
    and blocks, and (with ``big``) a tensor spanning two 16 MiB packets.
    """
    rng = np.random.default_rng(seed)
    a: dict[str, torch.Tensor] = {}
    b: dict[str, torch.Tensor] = {}

    def put(name: str, x: torch.Tensor, y: torch.Tensor) -> None:
        a[name], b[name] = x.contiguous(), y.contiguous()

    sizes = [1, 3, 8, 4097, 8191, 8192, 40000, 65536 // 2, 65536 // 2 + 7, 3 * 32768 + 256 * 3 + 5]
    if big:
        sizes.append((16 << 20) // 2 + 70001)
    for k, n in enumerate(sizes):
        put(f"parameter:bf16_{n}", *bf16_pair(n, scale, seed * 100 + k))
    x, y = bf16_pair(2048, 0.1, seed + 7)
    put("parameter:bf16_high_entropy", x, y)
    x, _ = bf16_pair(70000, scale, seed + 8)
    put("parameter:bf16_unchanged", x, x.clone())
    f = torch.from_numpy(rng.standard_normal(30001).astype(np.float32))
    put("buffer:fp32_cache", f, f * (1 + 1e-3 * torch.from_numpy(rng.standard_normal(30001).astype(np.float32))))
    u = torch.from_numpy(rng.integers(0, 256, 50001, dtype=np.uint8))
    v = u.clone()
    v[::5] ^= torch.from_numpy(rng.integers(1, 4, v[::5].numel(), dtype=np.uint8))  # small change alphabet
    put("buffer:u8_odd", u, v)
    u = torch.from_numpy(rng.integers(0, 256, 16383, dtype=np.uint8))
    put("buffer:u8_16383", u, u ^ 1)
    return a, b


def _lane_positions(lane: int, count: int) -> np.ndarray:
    """Word indexes of a block that decode lane ``lane`` owns: words
    8*lane .. 8*lane+7 of every 256-word (512-byte) group, in stream order."""
    groups = np.arange((count + 7) // 8)[:, None] * 256
    return (groups + 8 * lane + np.arange(8)[None, :]).reshape(-1)[:count]


def adversarial_pair(seed: int = 0) -> tuple[dict[str, torch.Tensor], dict[str, torch.Tensor]]:
    """CPU A/B dicts whose residuals sit on the coding boundaries.

    Every pattern is built twice: as an XOR residual (B = A ^ r) and as a U16
    residual (B = A + d mod 2^16), so that both transforms meet it exactly.
    Patterns: a single changed word among three blocks, two distinct
    words, exactly 255 and 256 distinct words (the dictionary limit), extreme
    skew (one word 99.9 %), rare words that fill one decode lane's escape list
    to its limit of 64 and past it, one residual word everywhere (a single
    symbol of probability 1 per table), and the largest U16 steps (d = 0x8000,
    0x7FFF, -1). Plus a packet of exactly 16 MiB and an odd-sized multi-block
    uint8 tensor with a three-word alphabet and a changed tail byte.
    """
    rng = np.random.default_rng(seed)
    a: dict[str, torch.Tensor] = {}
    b: dict[str, torch.Tensor] = {}

    def base_words(n: int) -> np.ndarray:
        x, _ = bf16_pair(n, 0.0, int(rng.integers(1 << 30)))
        return x.view(torch.int16).numpy().view(np.uint16).copy()

    def put_words(name: str, r: np.ndarray) -> None:
        w = base_words(r.size)
        for kind, t in (("x", w ^ r), ("u", (w.astype(np.uint32) + r) & 0xFFFF)):
            a[f"parameter:{name}_{kind}"] = torch.from_numpy(w.view(np.int16).copy()).view(torch.bfloat16)
            b[f"parameter:{name}_{kind}"] = torch.from_numpy(t.astype(np.uint16).view(np.int16)).view(torch.bfloat16)

    def alphabet(size: int, n: int) -> np.ndarray:
        values = rng.permutation(np.arange(1, 65536, dtype=np.uint32))[: size - 1]
        values = np.concatenate([[0], values]).astype(np.uint32)
        r = values[rng.integers(0, size, n)]
        r[:size] = values  # every value at least once
        return r[rng.permutation(n)]

    r = np.zeros(3 * BLOCK_WORDS, np.uint32)
    r[40000] = 0x0040
    put_words("one_word", r)
    put_words("two_words", rng.integers(0, 2, 2 * BLOCK_WORDS).astype(np.uint32))
    put_words("distinct_255", alphabet(255, 2 * BLOCK_WORDS + 100))
    put_words("distinct_256", alphabet(256, 2 * BLOCK_WORDS + 100))
    r = np.where(rng.random(2 * BLOCK_WORDS) < 0.999, 0, rng.integers(1, 4, 2 * BLOCK_WORDS)).astype(np.uint32)
    put_words("skew", r)
    for escapes in (64, 126):
        # 192 frequent words (the largest dictionary kept beside escapes) and
        # escapes / 2 rare words, each twice, all in lane 5 of the first block.
        frequent = rng.permutation(np.arange(1, 65536, dtype=np.uint32))[:192]
        r = frequent[rng.integers(0, 192, 2 * BLOCK_WORDS)]
        pool = np.setdiff1d(np.arange(1, 65536, dtype=np.uint32), frequent)
        r[_lane_positions(5, escapes)] = np.repeat(rng.choice(pool, escapes // 2, replace=False), 2)
        put_words(f"lane5_escapes_{escapes}", r)
    for word in (0x0101, 0x8000, 0xFFFF):  # one residual word everywhere: single-symbol tables
        put_words(f"constant_{word:04x}", np.full(2 * BLOCK_WORDS + 50, word, np.uint32))
    steps = np.array([0, 0x8000, 0x7FFF, 0xFFFF, 1], np.uint32)
    put_words("u16_extremes", steps[rng.integers(0, 5, BLOCK_WORDS + 4096)])
    put_words("packet_16mib", alphabet(40, (16 << 20) // 2))
    u = rng.integers(0, 256, 3 * _BLOCK_BYTES + 3, dtype=np.uint8)
    v = u ^ np.array([0, 1, 2], np.uint8)[rng.integers(0, 3, u.size)]
    v[-1] = u[-1] ^ 0x80
    a["buffer:u8_odd_blocks"], b["buffer:u8_odd_blocks"] = torch.from_numpy(u), torch.from_numpy(v)
    return a, b


def random_pair(size_class: tuple[int, int], kind: str, param: float, transform: str, odd: bool,
                seed: int) -> tuple[dict[str, torch.Tensor], dict[str, torch.Tensor]]:
    """A seeded random A/B pair for property tests: one bf16 tensor whose word
    count is drawn from ``size_class`` and whose residual is bf16 relative noise of
    strength ``param`` ("noise"), a skewed alphabet of 1 + 400 * param words
    ("alphabet") or a fraction param / 10 of changed words ("sparse"), applied as
    XOR or as a wrapping U16 add (``transform``); with ``odd``, also the same
    bytes as a uint8 tensor of odd length."""
    rng = np.random.default_rng(seed)
    n = int(rng.integers(size_class[0], size_class[1] + 1))
    if kind == "noise":
        a_t, b_t = bf16_pair(n, param, seed)
    else:
        if kind == "alphabet":
            size = 1 + int(param * 400)
            values = rng.integers(0, 65536, size).astype(np.uint32)
            r = values[rng.choice(size, n, p=rng.dirichlet(np.full(size, 0.3)))]
        else:
            r = np.zeros(n, np.uint32)
            hit = rng.random(n) < param / 10
            r[hit] = rng.integers(1, 65536, int(hit.sum()))
        a_t, _ = bf16_pair(n, 0.0, seed)
        w = a_t.view(torch.int16).numpy().view(np.uint16).astype(np.uint32)
        t = (w ^ r) if transform == "xor" else (w + r) & 0xFFFF
        b_t = torch.from_numpy(t.astype(np.uint16).view(np.int16)).view(torch.bfloat16)
    a, b = {"w": a_t}, {"w": b_t.clone()}
    if odd:
        a["u"] = a_t.view(torch.uint8)[: 2 * n - 1].clone()
        b["u"] = b_t.view(torch.uint8)[: 2 * n - 1].clone()
    return a, b


def _fuzz_strategies() -> dict:
    from hypothesis import strategies as st

    return dict(
        size_class=st.sampled_from([(1, 8191), (8191, 8193), (8192, 32768), (32769, 300_000)]),  # words
        kind=st.sampled_from(["noise", "alphabet", "sparse"]),
        param=st.sampled_from([0.0, 0.001, 0.01, 0.03, 0.1, 0.3]),
        transform=st.sampled_from(["xor", "u16"]),
        odd=st.booleans(),
        policy=st.sampled_from(["auto", "xor", "u16"]),
        # (dict_slack_pct, escapes, split)
        coding=st.sampled_from([(-1, -1, -1), (6, 0, 0), (100, -1, -1), (100, 1, -1), (100, -1, 1), (100, 0, 2),
                                (100, 1, 4)]),
        seed=st.integers(0, 2**31 - 1),
    )


# Hypothesis strategies of the property tests (random_pair's arguments, policy, coding).
FUZZ = _fuzz_strategies()


def host_plan(a: dict[str, torch.Tensor], b: dict[str, torch.Tensor], policy: str, dict_slack_pct: int = 6,
              escapes: int = 0, split: int = 0, threads: int = 4):
    """Build a plan on host targets (no GPU); b's tensors are the destinations."""
    lib = _lib.load()
    descs = (_lib.TensorDesc * len(a))()
    for i, name in enumerate(b):
        descs[i] = _lib.TensorDesc(
            a[name].data_ptr(), b[name].data_ptr(), b[name].numel() * b[name].element_size(),
            int(b[name].dtype == torch.bfloat16), 0,
        )
    opts = _lib.BuildOptions(policy=_lib.POLICIES[policy], threads=threads, target_on_device=0, device=0,
                             batch_bytes=0, staging_slots=0, pin_arena=0, dict_slack_pct=dict_slack_pct,
                             escapes=escapes, split=split)
    plan = ctypes.c_void_p()
    _lib.check(lib.ws_plan_build(descs, len(a), ctypes.byref(opts), None, ctypes.byref(plan)))
    return plan


def plan_arrays(plan) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, _lib.PlanStats]:
    lib = _lib.load()
    view, stats = _lib.PlanView(), _lib.PlanStats()
    _lib.check(lib.ws_plan_get_view(plan, ctypes.byref(view)))
    _lib.check(lib.ws_plan_get_stats(plan, ctypes.byref(stats)))

    def arr(ptr: int, nbytes: int, dtype) -> np.ndarray:
        if not nbytes:
            return np.zeros(0, dtype=dtype)
        return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(ptr)).view(dtype)

    blocks = arr(view.blocks, 32 * view.nblocks, ostream.BLOCK_DTYPE)
    tiles = arr(view.tiles, 16 * view.ntiles, ostream.TILE_DTYPE)
    tables = arr(view.tables, 4 * 512 * view.ntables, np.uint32)
    arena = arr(view.arena, view.arena_bytes, np.uint8)
    return blocks, tiles, tables, arena, stats


def split_bits(flags: int) -> int:
    """Raw low bits per word of a split-word block (flags bits 2-3: 0, 1, 2, 4)."""
    return (0, 1, 2, 4)[(int(flags) >> 2) & 3]


def split_raw_bytes(words: int, k: int) -> int:
    """Bytes of a split-word block's raw section: one uint32 per lane per 4 / k groups."""
    if not k:
        return 0
    groups = (words + 255) // 256
    per = 4 // k
    return 128 * ((groups + per - 1) // per)


def escape_list_offset(blk) -> int:
    """Arena offset of a dictionary block's escape list (after the stream and any raw section)."""
    return (int(blk["src"]) + ((2 * int(blk["nwords"]) + 15) & ~15)
            + split_raw_bytes(int(blk["nbytes"]) // 2, split_bits(blk["flags"])))


def as_bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy().reshape(-1)
