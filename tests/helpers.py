"""Test helpers: seeded tensor pairs covering the edge cases of the reference path."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from oracle import stream as ostream
from warpshift_b200 import _lib


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
    and 64 KiB blocks, and (with ``big``) a tensor spanning two 16 MiB packets.
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


def host_plan(a: dict[str, torch.Tensor], b: dict[str, torch.Tensor], policy: str, threads: int = 4, dict_slack_pct: int = 6,
              escapes: int = 0):
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
                             escapes=escapes)
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


def as_bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy().reshape(-1)
