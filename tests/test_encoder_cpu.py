"""Host encoder (product) checked by the oracle's independent C decoder, on CPU.

Plans are built on host targets, so every byte the encoder emits is decoded by
oracle/stream_oracle.c and applied to host copies; results must equal Teacher1 /
Teacher2 bit-exactly and the oracle's checksum must equal the one recorded at
prepare. The U16 representation is pinned to the reference residual
(delta.py:26-34): coded word = rotr16(zigzag(d), 1).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import semantics as sem
from oracle import stream as ostream
from tests.helpers import (adversarial_pair, as_bytes, bf16_pair, edge_pair, escape_list_offset, host_plan,
                           plan_arrays, split_bits, split_raw_bytes)
from warpshift_b200 import _lib

KIND_RAW, KIND_XOR, KIND_U16, KIND_DICT_XOR, KIND_DICT_U16 = 0, 1, 2, 3, 4


def clone(d):
    return {k: v.clone() for k, v in d.items()}


# (dict_slack_pct, escapes, split): byte planes only, the default choice, a
# dictionary wherever possible, dictionaries with escape lists wherever
# eligible, and split-word dictionaries of k = 1, 2, 4 raw bits wherever
# eligible (k = 4 with escapes).
CODINGS = {"planes": (-1, -1, -1), "default": (6, 0, 0), "dictionary": (100, -1, -1), "escapes": (100, 1, -1),
           "split1": (100, -1, 1), "split2": (100, 0, 2), "split4": (100, 1, 4)}


@pytest.mark.parametrize("coding", list(CODINGS))
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_host_plan_round_trips_through_the_oracle_decoder(policy: str, coding: str) -> None:
    a, b = edge_pair(seed=7)
    work = clone(b)
    plan = host_plan(a, work, policy, *CODINGS[coding])
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        assert stats.runtime_bytes == sum(t.numel() * t.element_size() for t in b.values())
        for reverse, teacher in ((True, a), (False, b), (True, a)):
            err, checksum = ostream.apply_plan(blocks, tiles, tables, arena, 0, reverse, 4)
            assert err == 0
            assert checksum == stats.expected_checksum[1 if reverse else 0]
            for name in b:
                np.testing.assert_array_equal(as_bytes(work[name]), as_bytes(teacher[name]), err_msg=name)
    finally:
        _lib.load().ws_plan_destroy(plan)


@pytest.fixture(scope="module")
def adversarial():
    return adversarial_pair(seed=5)


def blocks_by_tensor(blocks, work) -> dict[str, list]:
    """The plan's blocks grouped by destination tensor, in stream order."""
    spans = [(t.data_ptr(), t.data_ptr() + t.numel() * t.element_size(), n.split(":")[1]) for n, t in work.items()]
    out: dict[str, list] = {}
    for bk in blocks:
        dst = int(bk["dst"])
        out.setdefault(next(n for lo, hi, n in spans if lo <= dst < hi), []).append(bk)
    return out


@pytest.mark.parametrize("coding", list(CODINGS))
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_boundary_residuals_round_trip_through_the_oracle_decoder(adversarial, policy: str, coding: str) -> None:
    a, b = adversarial
    work = clone(b)
    plan = host_plan(a, work, policy, *CODINGS[coding])
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        for reverse, teacher in ((True, a), (False, b), (True, a)):
            err, checksum = ostream.apply_plan(blocks, tiles, tables, arena, 0, reverse, 4)
            assert err == 0
            assert checksum == stats.expected_checksum[1 if reverse else 0]
            for name in b:
                np.testing.assert_array_equal(as_bytes(work[name]), as_bytes(teacher[name]), err_msg=name)
    finally:
        _lib.load().ws_plan_destroy(plan)


@pytest.mark.parametrize("policy, suffix, dict_kind", [("xor", "x", KIND_DICT_XOR), ("u16", "u", KIND_DICT_U16)])
def test_dictionary_and_escape_limits_are_exact(adversarial, policy: str, suffix: str, dict_kind: int) -> None:
    """255 distinct words fit a dictionary, 256 do not; a lane holds at most 64
    escapes, and a block that needs more is carried raw."""
    a, b = adversarial
    work = clone(b)
    plan = host_plan(a, work, policy, dict_slack_pct=100, escapes=1, split=-1)
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        by = blocks_by_tensor(blocks, work)
        kinds = {n: {int(bk["kind"]) for bk in bks} for n, bks in by.items()}
        assert dict_kind in kinds[f"distinct_255_{suffix}"]
        assert dict_kind not in kinds[f"distinct_256_{suffix}"]
        first, second = by[f"lane5_escapes_64_{suffix}"]
        assert first["kind"] == dict_kind and first["flags"] & 2
        side = escape_list_offset(first)
        counts = arena[side : side + 64].view(np.uint16)
        assert counts[5] == 64 and counts.sum() == 64
        first, second = by[f"lane5_escapes_126_{suffix}"]
        assert first["kind"] == KIND_RAW and second["kind"] == dict_kind and not second["flags"] & 2
        err, _ = ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 4)
        assert err == 0
        for name in a:
            np.testing.assert_array_equal(as_bytes(work[name]), as_bytes(a[name]), err_msg=name)
    finally:
        _lib.load().ws_plan_destroy(plan)


def test_plans_do_not_depend_on_the_thread_count() -> None:
    """The host encoder's plan is a function of the bytes alone: 1 and 7 threads
    give identical descriptors, tables, arena and checksums (the GPU encoder is
    checked against this plan byte for byte)."""
    a, b = edge_pair(seed=14)
    plans = [host_plan(a, clone(b), "auto", threads=t, escapes=0) for t in (1, 7)]
    try:
        (b1, t1, tab1, ar1, s1), (b7, t7, tab7, ar7, s7) = (plan_arrays(p) for p in plans)
        for field in ("src", "nbytes", "clen", "nwords", "kind", "tail", "flags"):
            np.testing.assert_array_equal(b1[field], b7[field], err_msg=field)
        np.testing.assert_array_equal(t1.view(np.uint8), t7.view(np.uint8))
        np.testing.assert_array_equal(tab1, tab7)
        np.testing.assert_array_equal(ar1, ar7)
        assert list(s1.expected_checksum) == list(s7.expected_checksum)
        assert list(s1.mode_counts) == list(s7.mode_counts)
    finally:
        for p in plans:
            _lib.load().ws_plan_destroy(p)


def test_mode_rule_follows_the_reference() -> None:
    """delta.py:176-194: <16384 B raw, unchanged SKIP, odd sizes XOR_ANS, XOR-only policy never U16."""
    a, b = edge_pair(seed=8)
    expected_skipped = sum(x.numel() * x.element_size() for n, x in a.items() if torch.equal(x, b[n]))
    for policy in ("auto", "xor", "u16"):
        plan = host_plan(a, clone(b), policy)
        *_, stats = plan_arrays(plan)
        counts = dict(zip(_lib.MODE_NAMES, list(stats.mode_counts)))
        assert counts["SKIP"] == 1 and stats.skipped_bytes == expected_skipped
        small = sum(1 for n, x in b.items() if 0 < x.numel() * x.element_size() < sem.COMPRESS_MIN and not torch.equal(x, a[n]))
        assert counts["XOR_RAW"] >= small
        if policy == "xor":
            assert counts["U16_ANS"] == 0 and counts["XOR_GROUP2_ANS"] > 0
        else:
            assert counts["U16_ANS"] > 0
        assert counts["XOR_ANS"] >= 1  # the odd-sized compressible uint8 tensor
        _lib.load().ws_plan_destroy(plan)


@pytest.mark.parametrize("coding", ["planes", "dictionary"])
@pytest.mark.parametrize("policy", ["xor", "u16"])
def test_coded_words_are_the_reference_residual(policy: str, coding: str) -> None:
    a_t, b_t = bf16_pair(3 * 32768 + 1000, 0.01, 9)
    a, b = {"w": a_t}, {"w": b_t.clone()}
    plan = host_plan(a, b, policy, *CODINGS[coding])
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        base, target = as_bytes(a_t), as_bytes(b_t)
        xor_words = sem.xor_residual(base, target).view("<u2")
        z = sem.u16_residual(base, target)
        half = z.size // 2
        zig = z[:half].astype(np.uint32) | (z[half:].astype(np.uint32) << 8)
        rot = ((zig >> 1) | ((zig & 1) << 15)).astype("<u2")
        t = tiles[0]
        table = tables[512 * t["table"] : 512 * t["table"] + 512]
        for i, blk in enumerate(blocks):
            if blk["kind"] == KIND_RAW:
                continue
            payload = arena[blk["src"] : blk["src"] + blk["clen"]]
            words, err = ostream.decode_words(payload, blk, table)
            assert err == 0
            w0 = (int(blk["dst"]) - b["w"].data_ptr()) // 2
            ref = (rot if blk["kind"] in (KIND_U16, KIND_DICT_U16) else xor_words)[w0 : w0 + words.size]
            np.testing.assert_array_equal(words, ref, err_msg=f"block {i}")
            expected = {("u16", "planes"): KIND_U16, ("xor", "planes"): KIND_XOR,
                        ("u16", "dictionary"): KIND_DICT_U16, ("xor", "dictionary"): KIND_DICT_XOR}
            assert blk["kind"] == expected[(policy, coding)]
    finally:
        _lib.load().ws_plan_destroy(plan)


def test_corrupt_payload_is_detected_by_the_final_state_check() -> None:
    a_t, b_t = bf16_pair(40000, 0.01, 10)
    work = {"w": b_t.clone()}
    plan = host_plan({"w": a_t}, work, "xor")
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        blk = next(bk for bk in blocks if bk["kind"] != KIND_RAW)
        arena[blk["src"] + 300] ^= 0x40  # a renormalisation word
        err, _ = ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 1)
        assert err & 3
    finally:
        _lib.load().ws_plan_destroy(plan)


def escape_block(blocks):
    return next(bk for bk in blocks if bk["flags"] & 2)


def test_escape_lists_shrink_the_stream_and_malformed_lists_are_reported() -> None:
    """Escape lists on the 8B-like distribution, decoded by the oracle; a lane
    count raised by one hands that lane an entry of the next lane, which is reported."""
    a_t, b_t = bf16_pair(1 << 20, 0.01, 12)
    sizes = {}
    for esc in (-1, 0):
        work = {"w": b_t.clone()}
        plan = host_plan({"w": a_t}, work, "xor", escapes=esc, split=-1)
        try:
            blocks, tiles, tables, arena, stats = plan_arrays(plan)
            sizes[esc] = int(stats.arena_bytes)
            err, ck = ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 2)
            assert err == 0 and ck == stats.expected_checksum[1]
            np.testing.assert_array_equal(as_bytes(work["w"]), as_bytes(a_t))
            if esc == 0:
                blk = escape_block(blocks)
                side = escape_list_offset(blk)
                counts = arena[side: side + 64].view(np.uint16)
                lane = next(l for l in range(31) if counts[l + 1] > 0)
                counts[lane] += 1  # lane now reads the next lane's first entry
                err, _ = ostream.apply_plan(blocks, tiles, tables, arena, 0, False, 2)
                assert err & 2
        finally:
            _lib.load().ws_plan_destroy(plan)
    assert sizes[0] < sizes[-1] * 0.97


def test_overlapping_targets_and_bad_options_are_rejected() -> None:
    lib = _lib.load()
    buf = torch.zeros(1000, dtype=torch.uint8)
    base = torch.zeros(1000, dtype=torch.uint8)
    descs = (_lib.TensorDesc * 2)()
    descs[0] = _lib.TensorDesc(base.data_ptr(), buf.data_ptr(), 600, 0, 0)
    descs[1] = _lib.TensorDesc(base.data_ptr(), buf.data_ptr() + 500, 500, 0, 0)
    opts = _lib.BuildOptions(policy=0, threads=1, target_on_device=0, device=0, batch_bytes=0, staging_slots=0, pin_arena=0)
    plan = ctypes.c_void_p()
    assert lib.ws_plan_build(descs, 2, ctypes.byref(opts), None, ctypes.byref(plan)) == _lib.WS_ERR_INVALID
    assert "overlapping" in _lib.last_error()
    opts.batch_bytes = 1 << 20
    assert lib.ws_plan_build(descs, 1, ctypes.byref(opts), None, ctypes.byref(plan)) == _lib.WS_ERR_INVALID
    opts.batch_bytes, opts.policy = 0, 9
    assert lib.ws_plan_build(descs, 1, ctypes.byref(opts), None, ctypes.byref(plan)) == _lib.WS_ERR_INVALID
    assert lib.ws_plan_upload(None, None) == _lib.WS_ERR_INVALID


def test_host_plan_cannot_be_uploaded_or_applied() -> None:
    a, b = {"w": torch.ones(10)}, {"w": torch.zeros(10)}
    plan = host_plan(a, b, "auto")
    lib = _lib.load()
    try:
        assert lib.ws_plan_upload(plan, None) == _lib.WS_ERR_STATE
        res = _lib.ApplyResult()
        assert lib.ws_apply(plan, 0, None, None, ctypes.byref(res)) == _lib.WS_ERR_STATE
    finally:
        lib.ws_plan_destroy(plan)


def test_empty_and_fully_unchanged_models_have_nothing_to_apply() -> None:
    x = torch.randn(50000)
    plan = host_plan({"x": x, "e": torch.zeros(0)}, {"x": x.clone(), "e": torch.zeros(0)}, "auto")
    blocks, tiles, tables, arena, stats = plan_arrays(plan)
    assert stats.blocks == 0 and stats.arena_bytes == 0 and stats.skipped_bytes == x.numel() * 4
    assert ostream.apply_plan(blocks, tiles, tables, np.zeros(1, np.uint8), 0, True, 1) == (0, 0)
    _lib.load().ws_plan_destroy(plan)


def test_high_entropy_blocks_fall_back_to_raw_and_stay_exact() -> None:
    rng = np.random.default_rng(3)
    u = torch.from_numpy(rng.integers(0, 256, 3 * 65536, dtype=np.uint8))
    v = torch.from_numpy(rng.integers(0, 256, 3 * 65536, dtype=np.uint8))
    work = {"u": v.clone()}
    plan = host_plan({"u": u}, work, "auto")
    blocks, tiles, tables, arena, stats = plan_arrays(plan)
    assert all(bk["kind"] == KIND_RAW for bk in blocks)
    assert ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 2)[0] == 0
    assert torch.equal(work["u"], u)
    _lib.load().ws_plan_destroy(plan)


def test_dictionary_needs_few_distinct_words_and_planes_cover_the_rest() -> None:
    """Word dictionary only for 2..255 distinct residual words; otherwise byte planes."""
    a_t, b_t = bf16_pair(40000, 0.01, 12)  # ~100 distinct XOR words
    rng = np.random.default_rng(4)
    u = torch.from_numpy(rng.integers(0, 65536, 40000, dtype=np.uint16).astype(np.int16)).view(torch.bfloat16)
    v = u.view(torch.int16).clone()
    v[::3] ^= torch.from_numpy(rng.integers(1, 65536, v[::3].numel(), dtype=np.uint16).astype(np.int16))  # thousands of words
    cases = {"few": ({"w": a_t}, {"w": b_t.clone()}), "many": ({"w": u}, {"w": v.view(torch.bfloat16)})}
    for name, (a, b) in cases.items():
        plan = host_plan(a, b, "xor", dict_slack_pct=100)
        blocks, *_ = plan_arrays(plan)
        kinds = set(int(k) for k in blocks["kind"])
        if name == "few":
            assert kinds == {KIND_DICT_XOR}
        else:
            assert KIND_DICT_XOR not in kinds
        _lib.load().ws_plan_destroy(plan)


def test_split_words_shrink_the_stream_where_low_bits_are_noise() -> None:
    """Split-word dictionaries (the low k bits of each word stored raw, the rest
    coded): XOR s = 0.1 moves from byte planes to a k = 4 dictionary by default
    (13 % smaller); XOR s = 0.01 with k = 1 and U16 s = 0.1 with k = 4 are
    smaller too, but by less than the 3 % a split must save over the whole-word
    dictionary, so the default keeps whole words there. Every plan decodes
    exactly through the oracle."""
    # (policy, scale, k, its size bound against split = -1, the k the default picks)
    cases = [("xor", 0.01, 1, 0.99, 0), ("xor", 0.1, 4, 0.90, 4), ("u16", 0.1, 4, 0.985, 0)]
    for policy, scale, k, bound, default_k in cases:
        a_t, b_t = bf16_pair(1 << 20, scale, 21)
        sizes = {}
        for split in (-1, 0, k):
            work = {"w": b_t.clone()}
            plan = host_plan({"w": a_t}, work, policy, split=split)
            try:
                blocks, tiles, tables, arena, stats = plan_arrays(plan)
                sizes[split] = int(stats.arena_bytes)
                coded = blocks[blocks["kind"] != KIND_RAW]
                want = {0: default_k, -1: 0}.get(split, k)
                assert {split_bits(f) for f in coded["flags"]} == {want}, (policy, scale, split)
                assert set(tiles["split"][tiles["table"] != 0xFFFFFFFF]) == {(0, 1, 2, 3, 3)[want]}
                if want:
                    assert set(coded["kind"]) <= {KIND_DICT_XOR, KIND_DICT_U16}
                err, ck = ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 2)
                assert err == 0 and ck == stats.expected_checksum[1]
                np.testing.assert_array_equal(as_bytes(work["w"]), as_bytes(a_t))
            finally:
                _lib.load().ws_plan_destroy(plan)
        assert sizes[k] < sizes[-1] * bound, (policy, scale, sizes)


def residual_words(a_t: torch.Tensor, b_t: torch.Tensor, policy: str) -> np.ndarray:
    a = a_t.view(torch.int16).numpy().view(np.uint16).astype(np.int64)
    b = b_t.view(torch.int16).numpy().view(np.uint16).astype(np.int64)
    if policy == "xor":
        return (a ^ b).astype(np.uint16)
    d = ((b - a + 32768) & 0xFFFF) - 32768  # delta.py:26-34, then the coded rotation
    z = ((d << 1) ^ (d >> 15)) & 0xFFFF
    return (((z >> 1) | ((z & 1) << 15)) & 0xFFFF).astype(np.uint16)


@pytest.mark.parametrize("k", [1, 2, 4])
@pytest.mark.parametrize("policy", ["xor", "u16"])
def test_split_raw_section_holds_each_words_low_bits(policy: str, k: int) -> None:
    """The raw section of every split block, read back by the layout's own rule
    (raw word (g / G) * 32 + lane, G = 4 / k, bit (g % G) * 8k + j * k), equals
    the low k bits of the reference residual words; a flipped raw bit changes
    exactly that word of the applied result."""
    a_t, b_t = bf16_pair(70001, 0.01, 22)  # a partial last group and block
    work = {"w": b_t.clone()}
    plan = host_plan({"w": a_t}, work, policy, dict_slack_pct=100, split=k)
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        r = residual_words(a_t, b_t, policy)
        per, mask = 4 // k, (1 << k) - 1
        checked = 0
        for blk in blocks:
            if blk["kind"] == KIND_RAW:
                continue
            assert split_bits(blk["flags"]) == k
            W = int(blk["nbytes"]) // 2
            first = (int(blk["dst"]) - work["w"].data_ptr()) // 2  # host targets: dst is a host address
            off = int(blk["src"]) + ((2 * int(blk["nwords"]) + 15) & ~15)
            raw = arena[off: off + split_raw_bytes(W, k)].view(np.uint32)
            w = np.arange(W)
            g, lane, j = w // 256, (w % 256) // 8, w % 8
            bit = (g % per) * 8 * k + j * k
            got = (raw[(g // per) * 32 + lane] >> bit.astype(np.uint32)) & mask
            np.testing.assert_array_equal(got, r[first: first + W] & mask)
            checked += 1
        assert checked >= 1
        blk = next(bk for bk in blocks if bk["kind"] != KIND_RAW)
        off = int(blk["src"]) + ((2 * int(blk["nwords"]) + 15) & ~15)
        word = 256 * 3 + 8 * 7 + 5  # group 3, lane 7, lane word 5
        g, lane, j = 3, 7, 5
        bit = (g % per) * 8 * k + j * k
        raw = arena[off: off + split_raw_bytes(int(blk["nbytes"]) // 2, k)].view(np.uint32)
        raw[(g // per) * 32 + lane] ^= np.uint32(1 << bit)
        err, ck = ostream.apply_plan(blocks, tiles, tables, arena, 0, True, 2)
        assert err == 0 and ck != stats.expected_checksum[1]
        first = (int(blk["dst"]) - work["w"].data_ptr()) // 2
        got = work["w"].view(torch.int16).numpy().view(np.uint16)
        want = a_t.view(torch.int16).numpy().view(np.uint16)
        bad = np.nonzero(got != want)[0]
        assert list(bad) == [first + word]
    finally:
        _lib.load().ws_plan_destroy(plan)
