"""GPU parity: the fused sm_100a decode+apply against the oracle, bit-exact.

Every case compares the bytes the kernel wrote with (a) Teacher2/Teacher1
themselves (a forward-then-reverse round trip must restore Teacher1 exactly)
and (b) the oracle's restatement of the reference's restore semantics
(oracle.semantics, pinned by tests/golden). Integer/byte work: no tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import semantics as sem
from tests.helpers import adversarial_pair, as_bytes, edge_pair
from warpshift_b200 import synth
from warpshift_b200.delta import _BLOCK_BYTES, DeltaWeights

pytestmark = pytest.mark.gpu


def to_device(d: dict[str, torch.Tensor], device) -> dict[str, torch.Tensor]:
    return {k: v.to(device) for k, v in d.items()}


def assert_bytes_equal(gpu: dict[str, torch.Tensor], ref: dict[str, torch.Tensor]) -> None:
    for name, t in gpu.items():
        np.testing.assert_array_equal(as_bytes(t), as_bytes(ref[name]), err_msg=name)


CODINGS = {"planes": (-1, -1), "dictionary": (100, -1), "escapes": (100, 1)}  # (dict_slack_pct, escapes)


@pytest.mark.parametrize("coding", list(CODINGS))
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_edge_cases_round_trip_bit_exact(cuda_device, policy: str, coding: str) -> None:
    a, b = edge_pair(seed=1)
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy=policy, dict_slack_pct=CODINGS[coding][0], escapes=CODINGS[coding][1])
    assert set(delta.stats) >= {
        "codec", "reversible", "chunk_bytes", "batch_bytes", "runtime_bytes", "skipped_bytes", "payload_bytes",
        "transferred_bytes", "pinned_bytes", "mode_counts", "batches", "gpu_scratch_bytes", "gpu_metadata_bytes",
        "memory_scope", "prepare_seconds",
    }
    assert_bytes_equal(gpu, b)  # construction never changes GPU weights
    for reverse, expected in ((True, a), (False, b), (True, a), (False, b)):
        delta.apply(reverse=reverse)
        assert_bytes_equal(gpu, expected)
        assert delta.last_apply["ok"] and delta.last_apply["checksum"] == delta.last_apply["expected"]


@pytest.fixture(scope="module")
def adversarial():
    return adversarial_pair(seed=5)


@pytest.mark.parametrize("coding", list(CODINGS))
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_boundary_residuals_round_trip_bit_exact(cuda_device, adversarial, policy: str, coding: str) -> None:
    """Residuals on the coding limits (255/256 distinct words, 64 escapes in one
    lane and more, one changed word, extreme skew, largest U16 steps, an exact
    16 MiB packet), encoded on the GPU and applied by the fused kernel."""
    a, b = adversarial
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy=policy, dict_slack_pct=CODINGS[coding][0], escapes=CODINGS[coding][1])
    for reverse, expected in ((True, a), (False, b), (True, a)):
        delta.apply(reverse=reverse)
        assert_bytes_equal(gpu, expected)
        assert delta.last_apply["ok"]


@pytest.mark.parametrize("coding", list(CODINGS))
@pytest.mark.parametrize("policy", ["xor", "u16"])
def test_decoded_residual_matches_oracle(cuda_device, policy: str, coding: str) -> None:
    """Apply onto zeroed weights: the kernel then writes the residual itself.

    The asynchronous halves (apply_async + finish) are used because the
    written bytes cannot match the checksum recorded at prepare, and the
    synchronous apply would roll such a switch back."""
    a, b = edge_pair(seed=2, big=False)
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy=policy, dict_slack_pct=CODINGS[coding][0], escapes=CODINGS[coding][1])
    for t in gpu.values():
        t.zero_()
    delta.apply_async(reverse=False)
    with pytest.raises(RuntimeError, match="checksum"):
        delta.finish()
    for name, t in gpu.items():
        base, target = as_bytes(a[name]), as_bytes(b[name])
        xor = sem.xor_residual(base, target)
        got = as_bytes(t)
        if not xor.any():
            assert not got.any(), name
            continue
        if policy == "u16" and b[name].dtype == torch.bfloat16 and base.size >= sem.COMPRESS_MIN:
            # U16 packets write d = (B - A) mod 2^16 onto zero; raw-XOR fallbacks write the XOR.
            d = (sem.unzigzag_u16(sem.u16_residual(base, target)) % 65536).astype("<u2").view(np.uint8)
            mode = delta.stats["mode_counts"]
            assert "U16_ANS" in mode
            ok = np.array_equal(got, d) or np.array_equal(got, xor)
            if not ok:  # blocks may mix (per-block raw fallback): check block by block
                for off in range(0, got.size, _BLOCK_BYTES):
                    sl = slice(off, off + _BLOCK_BYTES)
                    assert np.array_equal(got[sl], d[sl]) or np.array_equal(got[sl], xor[sl]), (name, off)
        else:
            np.testing.assert_array_equal(got, xor, err_msg=name)


def test_config0_qwen2_shape_matches_reference_semantics(cuda_device) -> None:
    """Qwen2-0.5B-shaped pair (NumPy seeds 0/1): GPU apply == oracle restore == Teacher bits."""
    spec = synth.model_spec("qwen2-0.5b")
    t1, t2 = synth.generate_pair_numpy(spec, 0.01)
    gpu = to_device(t2, cuda_device)
    delta = DeltaWeights(t1, gpu, policy="auto")
    # Oracle: reference packets (delta.py:196-216, compressor stand-in = residual size / 4) applied to B.
    base_u8 = {k: as_bytes(v) for k, v in t1.items()}
    tgt_u8 = {k: as_bytes(v).copy() for k, v in t2.items()}
    bf16 = {k: v.dtype == torch.bfloat16 for k, v in t2.items()}
    packets, counts, skipped = sem.encode_packets(base_u8, tgt_u8, bf16, lambda r: r.size // 4)
    assert skipped == delta.stats["skipped_bytes"]
    sem.apply_packets(tgt_u8, packets, reverse=True)
    delta.apply(reverse=True)
    for name, t in gpu.items():
        got = as_bytes(t)
        np.testing.assert_array_equal(got, tgt_u8[name], err_msg=name)
        np.testing.assert_array_equal(got, base_u8[name], err_msg=name)
    delta.apply(reverse=False)
    assert_bytes_equal(gpu, t2)


def test_async_applies_run_in_stream_order_and_teardown_waits(cuda_device) -> None:
    """Back-to-back apply_async calls (the kernel-only bench loop) run in stream
    order and finish reports the last; freeing the resident copy or the whole
    plan with an apply in flight waits for it first."""
    a, b = edge_pair(seed=6, big=False)
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy="auto")
    for resident in (True, False):
        delta.set_resident(resident)
        for k in range(3):  # B->A, A->B, B->A
            delta.apply_async(reverse=k % 2 == 0)
        assert delta.finish()["ok"]
        assert_bytes_equal(gpu, a)
        delta.apply(reverse=False)
        assert_bytes_equal(gpu, b)
    delta.set_resident(True)
    delta.apply_async(reverse=True)
    delta.set_resident(False)
    assert delta.finish()["ok"]
    assert_bytes_equal(gpu, a)
    delta.apply_async(reverse=False)
    delta.close()
    torch.cuda.synchronize(cuda_device)
    assert_bytes_equal(gpu, b)


def test_checksum_rejects_wrong_resident_model(cuda_device) -> None:
    a, b = edge_pair(seed=3, big=False)
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy="auto")
    delta.apply(reverse=True)
    with pytest.raises(RuntimeError, match="checksum"):
        delta.apply(reverse=True)  # weights already hold A: the written bytes are not A
    assert not delta.last_apply["ok"]
    assert delta.last_apply["rollback"] == "unverified"  # rolled back onto what was resident: A
    assert_bytes_equal(gpu, a)


def test_misaligned_destinations(cuda_device) -> None:
    """Views at odd element offsets (not 16-byte aligned) take the byte-wise store path."""
    g = torch.Generator().manual_seed(11)
    storage = torch.zeros(3 * (2 * 65536 + 4000), dtype=torch.bfloat16, device=cuda_device)
    a, b, ref_b = {}, {}, {}
    start = 0
    for k, (off, n) in enumerate(((1, 2 * 65536 + 999), (3, 40001), (7, 65536 + 17))):
        x = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
        f = x.float()
        y = (f + 0.01 * f.abs() * torch.randn(n, generator=g)).to(torch.bfloat16)
        view = storage[start + off : start + off + n]
        view.copy_(y)
        a[f"parameter:v{k}"], b[f"parameter:v{k}"], ref_b[f"parameter:v{k}"] = x, view, y
        start += off + n
    assert all(v.data_ptr() % 16 for v in b.values())
    for policy, slack in (("xor", -1), ("u16", -1), ("xor", 100), ("u16", 100)):
        delta = DeltaWeights(a, b, policy=policy, dict_slack_pct=slack)
        delta.apply(reverse=True)
        assert_bytes_equal(b, a)
        delta.apply(reverse=False)
        assert_bytes_equal(b, ref_b)


def test_corrupt_frame_is_reported_and_the_context_stays_usable(cuda_device) -> None:
    """Host-side fault injection: one flipped payload byte in the pinned arena.

    The kernel's reads stay inside the staging ring and the block whatever the
    bytes are, so a corrupt frame can only produce wrong values; the final rANS
    state / stream length check reports it as a device error (no trap, no fault).
    """
    import ctypes

    from oracle import stream as ostream

    a, b = edge_pair(seed=5, big=False)
    gpu = to_device(b, cuda_device)
    delta = DeltaWeights(a, gpu, policy="xor")
    view = delta.plan_view()
    blocks = np.ctypeslib.as_array((ctypes.c_uint8 * (32 * view.nblocks)).from_address(view.blocks)).view(ostream.BLOCK_DTYPE)
    arena = np.ctypeslib.as_array((ctypes.c_uint8 * view.arena_bytes).from_address(view.arena))
    ans = [i for i, bk in enumerate(blocks) if bk["kind"] != 0]
    assert ans
    target = blocks[ans[0]]
    arena[int(target["src"]) + 260] ^= 0x21  # a renormalisation word of the first ANS block
    with pytest.raises(RuntimeError, match="decode failed"):
        delta.apply(reverse=True)
    assert delta.last_apply["device_errors"] & 3
    arena[int(target["src"]) + 260] ^= 0x21
    # Same context, fresh package: still exact.
    gpu2 = to_device(b, cuda_device)
    fresh = DeltaWeights(a, gpu2, policy="xor")
    fresh.apply(reverse=True)
    assert_bytes_equal(gpu2, a)


def test_malformed_escape_list_is_reported(cuda_device) -> None:
    """Host-side fault injection in an escape list: a lane's count raised by one
    makes it read the next lane's first entry, which the kernel's ownership check
    reports as a device error; no access leaves the block or the payload."""
    import ctypes

    from oracle import stream as ostream
    from tests.helpers import bf16_pair, escape_list_offset

    x, y = bf16_pair(1 << 20, 0.01, 12)
    gpu = {"w": y.to(cuda_device)}
    delta = DeltaWeights({"w": x}, gpu, policy="xor")
    view = delta.plan_view()
    blocks = np.ctypeslib.as_array((ctypes.c_uint8 * (32 * view.nblocks)).from_address(view.blocks)).view(ostream.BLOCK_DTYPE)
    arena = np.ctypeslib.as_array((ctypes.c_uint8 * view.arena_bytes).from_address(view.arena))
    blk = next(bk for bk in blocks if bk["flags"] & 2)
    side = escape_list_offset(blk)
    counts = arena[side: side + 64].view(np.uint16)
    lane = next(l for l in range(31) if counts[l + 1] > 0)
    counts[lane] += 1  # lane now reads the next lane's first entry
    with pytest.raises(RuntimeError, match="decode failed"):
        delta.apply(reverse=True)
    assert delta.last_apply["device_errors"] & 2
