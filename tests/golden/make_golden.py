"""Generate golden vectors from the reference implementation itself.

Run in a container that has a checkout of the reference (its repository root):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports the reference's ``warpshift.delta`` (no bytecode is written into the
read-only checkout) and records, on seeded inputs:
  * ``_u16_residual`` outputs (delta.py:26-34), including the reference test's
    exhaustive 65536-word sweep as SHA-256 digests;
  * ``_batch_layout`` results and rejections (delta.py:37-57);
  * ``DeltaWeights._encode_chunk`` mode decisions and the residuals it hands
    to its compressor (delta.py:176-194), with ``_compress`` replaced by a stub
    that returns buffers of chosen sizes (nvCOMP is not installable offline);
  * the Triton kernel ``_restore_batch`` (delta.py:60-92) for modes 0-3, forward
    and reverse, executed by Triton's CPU interpreter (TRITON_INTERPRET=1).
Outputs: tests/golden/reference_vectors.npz and tests/golden/reference_vectors.json.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="root of the reference checkout")
    args = parser.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import numpy as np
    import torch

    from warpshift import delta as ref  # the reference module

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"source": "reference warpshift/delta.py", "u16": [], "layout": [], "encode": [], "restore": []}
    rng = np.random.default_rng(20261201)

    # --- _u16_residual (delta.py:26-34)
    for k, words in enumerate([1, 5, 2048, 40000]):
        base = rng.integers(0, 65536, words, dtype=np.uint16)
        if k == 3:  # realistic small BF16 deltas
            base = (torch.randn(words, generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16)
            f = base.float()
            tgt = (f + 0.01 * f.abs() * torch.randn(words, generator=torch.Generator().manual_seed(2))).to(torch.bfloat16)
            base = base.view(torch.int16).numpy().view(np.uint16)
            tgt = tgt.view(torch.int16).numpy().view(np.uint16)
        else:
            tgt = rng.integers(0, 65536, words, dtype=np.uint16)
        out = ref._u16_residual(base.view(np.uint8), tgt.view(np.uint8))
        arrays[f"u16_{k}_base"], arrays[f"u16_{k}_target"], arrays[f"u16_{k}_out"] = base.view(np.uint8), tgt.view(np.uint8), out
        meta["u16"].append(k)
    sweep = {}
    for base_word in (0, 0x3F80, 0x8000, 0xFFFF, 0x7F80, 0x0001):
        target = np.arange(65536, dtype="<u2")
        base = np.full(target.shape, base_word, dtype="<u2")
        sweep[str(base_word)] = hashlib.sha256(ref._u16_residual(base.view(np.uint8), target.view(np.uint8)).tobytes()).hexdigest()
    meta["u16_sweep_sha256"] = sweep

    # --- _batch_layout (delta.py:37-57)
    cases = [([(300, 900), (300, 900), (700, 0), (400, 500), (1, 0)], 2048), ([], 2048), ([(2048, 2048)], 2048),
             ([(1, 1)] * 20, 300), ([(257, 0), (255, 255), (1, 2047)], 2048)]
    for n in (7, 30):
        sizes = [(int(rng.integers(1, 5000)), int(rng.integers(0, 5000)) * int(rng.integers(0, 2))) for _ in range(n)]
        cases.append((sizes, 6000))
    for sizes, limit in cases:
        meta["layout"].append({"sizes": sizes, "limit": limit, "batches": ref._batch_layout(sizes, limit=limit)})
    rejects = []
    for size in [(0, 1), (-1, 1), (1, -1), (2049, 1), (1, 2049)]:
        try:
            ref._batch_layout([size], limit=2048)
            rejects.append({"size": size, "error": None})
        except ValueError as exc:
            rejects.append({"size": size, "error": str(exc)})
    meta["layout_rejects"] = rejects

    # --- _encode_chunk (delta.py:176-194) with a stub compressor
    def encode_case(name, base, target, is_bf16, sizes):
        calls = []
        stub = ref.DeltaWeights.__new__(ref.DeltaWeights)

        def compress(data, configs):
            calls.append(np.array(data, copy=True))
            return torch.empty(sizes[len(calls) - 1], dtype=torch.uint8)

        stub._compress = compress
        result = ref.DeltaWeights._encode_chunk(stub, base, target, is_bf16, {})
        entry = {"name": name, "is_bf16": is_bf16, "stub_sizes": sizes, "calls": len(calls)}
        arrays[f"enc_{name}_base"], arrays[f"enc_{name}_target"] = base, target
        if result is None:
            entry["mode"] = None
        else:
            mode, payload = result
            entry["mode"] = int(mode)
            entry["payload_numel"] = int(payload.numel())
            if mode == 0:
                arrays[f"enc_{name}_payload"] = payload.numpy().copy()
        for i, c in enumerate(calls):
            arrays[f"enc_{name}_call{i}"] = c
        meta["encode"].append(entry)

    def bf16_bytes(n, s, seed):
        g = torch.Generator().manual_seed(seed)
        a = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
        f = a.float()
        b = (f + s * f.abs() * torch.randn(n, generator=g)).to(torch.bfloat16)
        return a.view(torch.uint8).numpy().copy(), b.view(torch.uint8).numpy().copy()

    a, b = bf16_bytes(12000, 0.01, 3)  # 24000 B >= 16384
    encode_case("bf16_u16_wins", a, b, True, [9000, 7000])
    encode_case("bf16_group_wins", a, b, True, [7000, 9000])
    encode_case("bf16_tie_keeps_group", a, b, True, [7000, 7000])
    encode_case("bf16_raw_wins", a, b, True, [24000, 24000])
    encode_case("bf16_unchanged", a, a.copy(), True, [])
    a, b = bf16_bytes(4000, 0.01, 4)  # 8000 B < 16384: raw only
    encode_case("bf16_small_raw", a, b, True, [])
    u = rng.integers(0, 256, 20001, dtype=np.uint8)
    v = u.copy()
    v[::3] ^= 0x5A
    encode_case("u8_odd_xor_ans", u, v, False, [5000])
    encode_case("u8_odd_raw", u, v, False, [20001])

    # --- _restore_batch (delta.py:60-92) under the Triton interpreter
    def run_restore(name, mode, dst, residual, reverse):
        n = dst.size
        dst_t = torch.from_numpy(dst.copy())
        res_t = torch.from_numpy(residual.copy() if residual.size else np.zeros(1, np.uint8))
        payload_t = res_t if mode == 0 else torch.zeros(16, dtype=torch.uint8)
        decoded_t = res_t if mode else torch.zeros(16, dtype=torch.uint8)
        desc = torch.tensor([[mode, dst_t.data_ptr(), n, 0, 0]], dtype=torch.int64)
        tiles = (n + ref._TILE_BYTES - 1) // ref._TILE_BYTES
        ref._restore_batch[(tiles,)](payload_t, decoded_t, desc, torch.zeros(tiles, dtype=torch.int32), reverse, ref._TILE_BYTES)
        arrays[f"res_{name}_dst"], arrays[f"res_{name}_residual"], arrays[f"res_{name}_out"] = dst, residual, dst_t.numpy().copy()
        meta["restore"].append({"name": name, "mode": mode, "reverse": bool(reverse)})

    a, b = bf16_bytes(5000, 0.01, 5)  # 10000 B: 3 tiles, last partial
    xor = np.bitwise_xor(a, b)
    grouped = xor.reshape(-1, 2).T.copy().reshape(-1)
    u16 = ref._u16_residual(a, b)
    run_restore("m0_fwd", 0, a, xor, False)
    run_restore("m1_fwd", 1, a, grouped, False)
    run_restore("m1_rev", 1, b, grouped, True)
    run_restore("m3_fwd", 3, a, u16, False)
    run_restore("m3_rev", 3, b, u16, True)
    extreme_a = np.array([0, 0, 0xFFFF, 0, 0x8000, 0x7FFF, 0x8000], dtype="<u2").view(np.uint8)
    extreme_b = np.array([0, 1, 0, 0xFFFF, 0, 0x8000, 0x7FFF], dtype="<u2").view(np.uint8)
    run_restore("m3_extreme_fwd", 3, extreme_a, ref._u16_residual(extreme_a, extreme_b), False)
    run_restore("m3_extreme_rev", 3, extreme_b, ref._u16_residual(extreme_a, extreme_b), True)
    u = rng.integers(0, 256, 9001, dtype=np.uint8)
    v = rng.integers(0, 256, 9001, dtype=np.uint8)
    run_restore("m2_odd_fwd", 2, u, np.bitwise_xor(u, v), False)

    np.savez_compressed(HERE / "reference_vectors.npz", **arrays)
    (HERE / "reference_vectors.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(arrays)} arrays, {len(meta['encode'])} encode cases, {len(meta['restore'])} restore cases")


if __name__ == "__main__":
    main()
