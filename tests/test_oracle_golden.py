"""Pin the oracle (and the product's reference helpers) to vectors produced by the reference itself.

tests/golden/make_golden.py recorded these from the reference's own
_u16_residual, _batch_layout, DeltaWeights._encode_chunk (stub compressor) and
its Triton _restore_batch kernel run by Triton's CPU interpreter.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import semantics as sem
from warpshift_b200.delta import _batch_layout, _u16_residual

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_vectors.json").read_text())
ARR = np.load(GOLDEN / "reference_vectors.npz")


@pytest.mark.parametrize("k", META["u16"])
@pytest.mark.parametrize("impl", [sem.u16_residual, _u16_residual], ids=["oracle", "product"])
def test_u16_residual_matches_reference(k: int, impl) -> None:
    np.testing.assert_array_equal(impl(ARR[f"u16_{k}_base"], ARR[f"u16_{k}_target"]), ARR[f"u16_{k}_out"])


@pytest.mark.parametrize("impl", [sem.u16_residual, _u16_residual], ids=["oracle", "product"])
def test_u16_residual_exhaustive_sweep_digests(impl) -> None:
    for base_word, digest in META["u16_sweep_sha256"].items():
        target = np.arange(65536, dtype="<u2")
        base = np.full(target.shape, int(base_word), dtype="<u2")
        out = impl(base.view(np.uint8), target.view(np.uint8))
        assert hashlib.sha256(out.tobytes()).hexdigest() == digest, base_word


def _as_json(batches):
    return json.loads(json.dumps(batches))


@pytest.mark.parametrize("case", range(len(META["layout"])))
@pytest.mark.parametrize("impl", [sem.batch_layout, _batch_layout], ids=["oracle", "product"])
def test_batch_layout_matches_reference(case: int, impl) -> None:
    c = META["layout"][case]
    sizes = [tuple(s) for s in c["sizes"]]
    assert _as_json(impl(sizes, limit=c["limit"])) == c["batches"]


@pytest.mark.parametrize("impl", [sem.batch_layout, _batch_layout], ids=["oracle", "product"])
def test_batch_layout_rejections_match_reference(impl) -> None:
    for r in META["layout_rejects"]:
        if r["error"] is None:
            impl([tuple(r["size"])], limit=2048)
        else:
            with pytest.raises(ValueError, match="frame size"):
                impl([tuple(r["size"])], limit=2048)


@pytest.mark.parametrize("entry", META["encode"], ids=lambda e: e["name"])
def test_encode_chunk_mode_choice_matches_reference(entry) -> None:
    name = entry["name"]
    base, target = ARR[f"enc_{name}_base"], ARR[f"enc_{name}_target"]
    sizes = list(entry["stub_sizes"])
    calls = []

    def size_of(residual):
        calls.append(residual.copy())
        return sizes[len(calls) - 1]

    result = sem.encode_chunk(base, target, entry["is_bf16"], size_of)
    assert len(calls) == entry["calls"]
    for i, c in enumerate(calls):
        np.testing.assert_array_equal(c, ARR[f"enc_{name}_call{i}"])
    if entry["mode"] is None:
        assert result is None
        return
    mode, residual, _ = result
    assert mode == entry["mode"]
    if mode == 0:
        np.testing.assert_array_equal(residual, ARR[f"enc_{name}_payload"])


@pytest.mark.parametrize("entry", META["restore"], ids=lambda e: e["name"])
def test_restore_matches_reference_triton_kernel(entry) -> None:
    name = entry["name"]
    dst = ARR[f"res_{name}_dst"].copy()
    sem.restore(dst, entry["mode"], ARR[f"res_{name}_residual"], entry["reverse"])
    np.testing.assert_array_equal(dst, ARR[f"res_{name}_out"])


def test_round_trip_semantics_restore_both_directions() -> None:
    """Oracle's restore of every mode is involutive/invertible on the golden inputs (delta.py:84, 92)."""
    for entry in META["restore"]:
        if entry["reverse"]:
            continue
        name = entry["name"]
        a = ARR[f"res_{name}_dst"]
        b = ARR[f"res_{name}_out"]
        back = b.copy()
        sem.restore(back, entry["mode"], ARR[f"res_{name}_residual"], True)
        np.testing.assert_array_equal(back, a)
