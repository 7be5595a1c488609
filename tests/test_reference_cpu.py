"""The host-core restatement of the reference's switch (oracle/reference_cpu.py),
which bench.py times as the reference arm, against the golden-pinned oracle and
the reference's own vectors."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import reference_cpu as ref
from oracle import semantics as sem

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_vectors.json").read_text())
ARR = np.load(GOLDEN / "reference_vectors.npz")


@pytest.mark.parametrize("entry", META["restore"], ids=lambda e: e["name"])
def test_restore_packet_matches_reference_vectors(entry) -> None:
    name = entry["name"]
    dst = ARR[f"res_{name}_dst"].copy()
    ref.restore_packet(dst, entry["mode"], ARR[f"res_{name}_residual"], entry["reverse"])
    np.testing.assert_array_equal(dst, ARR[f"res_{name}_out"])


@pytest.mark.parametrize("n", [2, 16384, 2 * ref.SLICE_WORDS * 2 + 6, 3 * ref.SLICE_WORDS + 1000])
@pytest.mark.parametrize("mode", [0, 1, 3])
@pytest.mark.parametrize("reverse", [False, True])
def test_restore_packet_matches_semantics(n: int, mode: int, reverse: bool) -> None:
    rng = np.random.default_rng(n + mode)
    dst = rng.integers(0, 256, n, dtype=np.uint8)
    residual = rng.integers(0, 256, n, dtype=np.uint8)
    want = dst.copy()
    sem.restore(want, mode, residual, reverse)
    got = dst.copy()
    ref.restore_packet(got, mode, residual, reverse)
    np.testing.assert_array_equal(got, want)


def test_odd_sizes_use_plain_xor() -> None:
    rng = np.random.default_rng(3)
    dst = rng.integers(0, 256, 40001, dtype=np.uint8)
    residual = rng.integers(0, 256, 40001, dtype=np.uint8)
    want = dst.copy()
    sem.restore(want, 2, residual, False)
    ref.restore_packet(dst, 2, residual, False)
    np.testing.assert_array_equal(dst, want)
    with pytest.raises(ValueError):
        ref.restore_packet(dst, 3, residual, False)


@pytest.mark.parametrize("policy", ["xor", "u16", "auto"])
def test_switch_round_trip_restores_both_teachers(policy: str) -> None:
    """A whole switch over a set of tensors (threads and one core) gives Teacher1, then Teacher2."""
    rng = np.random.default_rng(7)
    a, b, bf16 = {}, {}, {}
    for k, n in enumerate([7, 16383, 16384, 100_001 * 2, sem.CHUNK_BYTES + 4098]):
        x = (rng.standard_normal(n // 2 + 1, dtype=np.float32) * 0.02).view(np.uint8)[:n].copy()
        y = x.copy()
        y[:: 3] ^= rng.integers(0, 4, y[::3].size, dtype=np.uint8)
        a[f"t{k}"], b[f"t{k}"], bf16[f"t{k}"] = x, y, n % 2 == 0
    a["same"] = b["same"] = np.arange(1000, dtype=np.uint8)
    bf16["same"] = False
    packets = ref.packets_of(a, b, bf16, policy, threads=2)
    assert all(p[0] != "same" for p in packets)  # unchanged packets are skipped (delta.py:181)
    modes = {p[2] for p in packets}
    assert 0 in modes  # tensors below 16384 bytes stay raw XOR (delta.py:185)
    if policy == "u16":
        assert 3 in modes
    work = {k: v.copy() for k, v in b.items()}
    sw = ref.CpuSwitch(work, packets, threads=3)
    sw.switch()
    for k in a:
        np.testing.assert_array_equal(work[k], a[k], err_msg=k)
    sw.switch(threads=1)
    for k in b:
        np.testing.assert_array_equal(work[k], b[k], err_msg=k)


def test_order0_stand_in_prefers_smaller_candidates() -> None:
    flat = np.zeros(1 << 16, dtype=np.uint8)
    noisy = np.random.default_rng(0).integers(0, 256, 1 << 16, dtype=np.uint8)
    assert ref.order0_bytes(flat) == 0
    assert ref.order0_bytes(noisy) > 0.99 * noisy.size
