"""Saved delta plans (ws_plan_save / ws_plan_load) on host targets, checked by the
oracle's C decoder: a loaded plan rebased onto new buffers restores both teachers
bit-exactly and carries the same descriptors, tables, arena and checksums; files
that do not match the tensors, are corrupt or truncated are rejected."""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import stream as ostream
from tests.helpers import as_bytes, edge_pair, host_plan, plan_arrays
from warpshift_b200 import _lib


def clone(d):
    return {k: v.clone() for k, v in d.items()}


def descs_for(targets: dict[str, torch.Tensor]):
    descs = (_lib.TensorDesc * len(targets))()
    for i, t in enumerate(targets.values()):
        descs[i] = _lib.TensorDesc(None, t.data_ptr(), t.numel() * t.element_size(), int(t.dtype == torch.bfloat16), 0)
    return descs


def load(path, targets, threads=4):
    lib = _lib.load()
    opts = _lib.BuildOptions(policy=0, threads=threads, target_on_device=0, device=0, batch_bytes=0, staging_slots=0,
                             pin_arena=0, dict_slack_pct=6, encode_on_device=0, encode_batch_bytes=0)
    plan = ctypes.c_void_p()
    _lib.check(lib.ws_plan_load(os.fsencode(path), descs_for(targets), len(targets), ctypes.byref(opts), ctypes.byref(plan)))
    return plan


@pytest.fixture()
def saved(tmp_path):
    a, b = edge_pair(seed=11)
    work = clone(b)
    lib = _lib.load()
    plan = host_plan(a, work, "auto")
    path = tmp_path / "delta.wsd"
    _lib.check(lib.ws_plan_save(plan, os.fsencode(path)))
    yield a, b, work, plan, path
    lib.ws_plan_destroy(plan)


def test_loaded_plan_is_the_saved_plan_rebased(saved) -> None:
    a, b, work, plan, path = saved
    fresh = clone(b)  # new buffers: the loaded plan must point into these
    loaded = load(path, fresh)
    try:
        b0, t0, tab0, ar0, s0 = plan_arrays(plan)
        b1, t1, tab1, ar1, s1 = plan_arrays(loaded)
        base0 = {name: work[name].data_ptr() for name in work}
        base1 = {name: fresh[name].data_ptr() for name in fresh}
        ends0 = sorted((base0[n], base0[n] + work[n].numel() * work[n].element_size(), n) for n in work)

        def rel(dst, bases, spans):
            for lo, hi, n in spans:
                if lo <= dst < hi:
                    return n, dst - lo
            raise AssertionError(dst)

        ends1 = sorted((base1[n], base1[n] + fresh[n].numel() * fresh[n].element_size(), n) for n in fresh)
        assert [rel(int(d), base0, ends0) for d in b0["dst"]] == [rel(int(d), base1, ends1) for d in b1["dst"]]
        for field in ("src", "nbytes", "clen", "nwords", "kind", "tail", "flags"):
            np.testing.assert_array_equal(b0[field], b1[field], err_msg=field)
        np.testing.assert_array_equal(t0.view(np.uint8), t1.view(np.uint8))
        np.testing.assert_array_equal(tab0, tab1)
        np.testing.assert_array_equal(ar0, ar1)
        assert list(s0.expected_checksum) == list(s1.expected_checksum)
        assert list(s0.mode_counts) == list(s1.mode_counts)
        assert (s0.arena_bytes, s0.touched_bytes, s0.blocks, s0.tiles, s0.batches) == (
            s1.arena_bytes, s1.touched_bytes, s1.blocks, s1.tiles, s1.batches)
        for reverse, teacher in ((True, a), (False, b), (True, a)):
            err, checksum = ostream.apply_plan(b1, t1, tab1, ar1, 0, reverse, 4)
            assert err == 0 and checksum == s1.expected_checksum[1 if reverse else 0]
            for name in b:
                np.testing.assert_array_equal(as_bytes(fresh[name]), as_bytes(teacher[name]), err_msg=name)
    finally:
        _lib.load().ws_plan_destroy(loaded)


def test_files_that_do_not_match_are_rejected(saved, tmp_path) -> None:
    a, b, work, plan, path = saved
    names = list(b)
    with pytest.raises(ValueError, match="tensors"):
        load(path, {n: b[n].clone() for n in names[:-1]})
    resized = clone(b)
    resized[names[0]] = torch.zeros(resized[names[0]].numel() + 1, dtype=resized[names[0]].dtype)
    with pytest.raises(ValueError, match="differs from the saved plan"):
        load(path, resized)
    # Two targets over one buffer: rejected before anything is read into the arena.
    fresh = clone(b)
    sized = [n for n in names if fresh[n].numel() * fresh[n].element_size() > 0]
    n0, n1 = sized[0], sized[1]
    bytes0 = fresh[n0].numel() * fresh[n0].element_size()
    bytes1 = fresh[n1].numel() * fresh[n1].element_size()
    shared = torch.zeros(max(bytes0, bytes1), dtype=torch.uint8)
    descs = descs_for(fresh)
    descs[names.index(n0)].target = shared.data_ptr()
    descs[names.index(n1)].target = shared.data_ptr()
    opts = _lib.BuildOptions(policy=0, threads=2, target_on_device=0, device=0, batch_bytes=0, staging_slots=0,
                             pin_arena=0, dict_slack_pct=6, encode_on_device=0, encode_batch_bytes=0)
    out = ctypes.c_void_p()
    with pytest.raises(ValueError, match="overlapping"):
        _lib.check(_lib.load().ws_plan_load(os.fsencode(path), descs, len(names), ctypes.byref(opts), ctypes.byref(out)))


def test_corrupt_truncated_and_foreign_files_are_rejected(saved, tmp_path) -> None:
    a, b, work, plan, path = saved
    raw = path.read_bytes()
    bad = tmp_path / "bad.wsd"
    flipped = bytearray(raw)
    flipped[200] ^= 0x40  # inside the metadata
    bad.write_bytes(bytes(flipped))
    with pytest.raises(ValueError, match="corrupt"):
        load(bad, clone(b))
    bad.write_bytes(raw[:-100])
    with pytest.raises(OSError, match="truncated"):
        load(bad, clone(b))
    bad.write_bytes(b"not a delta plan at all" * 10)
    with pytest.raises(ValueError, match="not a saved delta plan"):
        load(bad, clone(b))
    with pytest.raises(OSError, match="cannot open"):
        load(tmp_path / "missing.wsd", clone(b))
    lib = _lib.load()
    with pytest.raises(OSError, match="cannot create"):
        _lib.check(lib.ws_plan_save(plan, os.fsencode(tmp_path / "no_such_dir" / "x.wsd")))
    assert not (tmp_path / "delta.wsd.tmp").exists()


def rehashed(raw: bytes, edit) -> bytes:
    """The saved file with its block/tile descriptors changed by ``edit`` and the
    metadata hash recomputed, so that only the descriptor checks can reject it.
    Header: magic, u32 version/header/stats/block-desc sizes, then u64 counts,
    arena offset and size, metadata hash (ws_persist.cpp)."""
    from oracle.hashes import mix64_int

    head = np.frombuffer(raw[:80], dtype=np.uint8)
    stats_bytes = int(head[16:20].view("<u4")[0])
    ntensors, nblocks, ntiles, _, arena_offset, _, _ = (int(x) for x in head[24:80].view("<u8"))
    meta = bytearray(raw[80:arena_offset])
    at = stats_bytes + 16 * ntensors
    blocks = np.frombuffer(meta, dtype=ostream.BLOCK_DTYPE, count=nblocks, offset=at).copy()
    tiles = np.frombuffer(meta, dtype=ostream.TILE_DTYPE, count=ntiles, offset=at + 36 * nblocks).copy()
    edit(blocks, tiles)
    meta[at : at + 32 * nblocks] = blocks.tobytes()
    meta[at + 36 * nblocks : at + 36 * nblocks + 16 * ntiles] = tiles.tobytes()
    h = 0x6A09E667F3BCC908 ^ len(meta)
    words = np.frombuffer(bytes(meta), dtype="<u8")
    for i, w in enumerate(words.tolist()):
        h = mix64_int(h ^ ((w + (i + 1) * 0x9E3779B97F4A7C15) & ((1 << 64) - 1)))
    out = bytearray(raw)
    out[72:80] = np.array([h], dtype="<u8").tobytes()
    out[80:arena_offset] = meta
    return bytes(out)


def test_descriptors_that_could_reach_outside_the_buffers_are_rejected(saved, tmp_path) -> None:
    """Metadata with a valid hash but descriptors that would make a kernel write
    outside a tensor, stage a payload with a size the bulk copies cannot take,
    or look up a missing table is rejected before any arena is read."""
    a, b, work, plan, path = saved
    raw = path.read_bytes()
    bad = tmp_path / "bad.wsd"
    bad.write_bytes(rehashed(raw, lambda bl, ti: None))
    lib = _lib.load()
    lib.ws_plan_destroy(load(bad, clone(b)))  # the rewriting itself keeps the file valid

    def first_coded(bl):
        return int(np.flatnonzero(bl["kind"] != 0)[0])

    def outside(bl, ti):
        bl["dst"][0] += 1 << 40

    def shift16(bl, ti):  # two payloads of lengths -8 / +8: still contiguous, no longer 16-byte multiples
        k = first_coded(bl)
        bl["clen"][k] -= 8
        bl["src"][k + 1] -= 8
        bl["clen"][k + 1] += 8

    def kind(bl, ti):
        bl["kind"][0] = 9

    def table(bl, ti):
        ti["table"][int(np.flatnonzero(ti["table"] != 0xFFFFFFFF)[0])] = 1 << 20

    def stream_length(bl, ti):
        k = first_coded(bl)
        bl["nwords"][k] = bl["clen"][k]  # 2 * nwords bytes no longer fit the payload

    def tile_split(bl, ti):  # a split code the kernel has no expansion table for
        ti["split"][0] = 5

    def block_split(bl, ti):  # a block whose split code is not its tile's
        bl["flags"][int(ti["first_block"][0])] ^= 3 << 2

    cases = {outside: "writes outside its tensor", shift16: "not a multiple of 16", kind: "unknown kind",
             table: "bad table", stream_length: "bad stream length", tile_split: "another split code",
             block_split: "another split code|not a word-dictionary block|raw section outside"}
    for edit, message in cases.items():
        bad.write_bytes(rehashed(raw, edit))
        with pytest.raises(ValueError, match=message):
            load(bad, clone(b))


def test_empty_model_round_trips(tmp_path) -> None:
    a = {"w": torch.zeros(1000, dtype=torch.bfloat16)}
    b = clone(a)
    lib = _lib.load()
    plan = host_plan(a, b, "auto")
    path = tmp_path / "empty.wsd"
    try:
        _lib.check(lib.ws_plan_save(plan, os.fsencode(path)))
    finally:
        lib.ws_plan_destroy(plan)
    loaded = load(path, clone(b))
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(loaded)
        assert stats.blocks == 0 and stats.arena_bytes == 0 and stats.batches == 0 and arena.size == 0
    finally:
        lib.ws_plan_destroy(loaded)
