"""GPU encoder (prepare on the device) against the host encoder: identical plans.

Both encoders read the same A (host) and B (device) bytes; the GPU path copies
only A to the device and computes statistics, tables' inputs and the rANS
streams there. Their plans must match byte for byte: arena, block and tile
descriptors, tables, expected checksums and mode counts.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import adversarial_pair, bf16_pair, edge_pair, plan_arrays
from warpshift_b200 import _lib

pytestmark = pytest.mark.gpu


def build(a, b_dev, policy, slack, on_device, encode_batch_bytes=0, pin_arena=0, batch_bytes=0, escapes=0,
          host_fallback=0, split=0):
    lib = _lib.load()
    descs = (_lib.TensorDesc * len(a))()
    for i, name in enumerate(b_dev):
        t = b_dev[name]
        descs[i] = _lib.TensorDesc(a[name].data_ptr(), t.data_ptr(), t.numel() * t.element_size(),
                                   int(t.dtype == torch.bfloat16), 0)
    opts = _lib.BuildOptions(policy=_lib.POLICIES[policy], threads=4, target_on_device=1, device=0,
                             batch_bytes=batch_bytes, staging_slots=0, pin_arena=pin_arena, dict_slack_pct=slack,
                             encode_on_device=int(on_device), encode_batch_bytes=encode_batch_bytes,
                             escapes=escapes, host_fallback=host_fallback, split=split)
    plan = ctypes.c_void_p()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.ws_plan_build(descs, len(a), ctypes.byref(opts), stream, ctypes.byref(plan)))
    return plan


def assert_same_plan(p_gpu, p_host) -> None:
    bg, tg, tabg, ag, sg = plan_arrays(p_gpu)
    bh, th, tabh, ah, sh = plan_arrays(p_host)
    assert list(sg.mode_counts) == list(sh.mode_counts)
    assert (sg.blocks, sg.tiles, sg.arena_bytes, sg.payload_bytes, sg.skipped_bytes, sg.zero_block_bytes) == (
        sh.blocks, sh.tiles, sh.arena_bytes, sh.payload_bytes, sh.skipped_bytes, sh.zero_block_bytes)
    assert list(sg.expected_checksum) == list(sh.expected_checksum)
    np.testing.assert_array_equal(bg.view(np.uint8), bh.view(np.uint8))
    np.testing.assert_array_equal(tg.view(np.uint8), th.view(np.uint8))
    np.testing.assert_array_equal(tabg, tabh)
    np.testing.assert_array_equal(ag, ah)


# (dict_slack_pct, escapes, split): planes only, the defaults, plain and escaped
# dictionaries, and split-word dictionaries of k = 1, 2, 4 raw bits.
CODINGS = [(-1, -1, -1), (6, 0, 0), (100, -1, -1), (100, 1, -1), (100, -1, 1), (100, 0, 2), (100, 1, 4)]


@pytest.mark.parametrize("slack, escapes, split", CODINGS)
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_gpu_encoder_matches_host_encoder(cuda_device, policy: str, slack: int, escapes: int, split: int) -> None:
    a, b = edge_pair(seed=13)
    b_dev = {k: v.to(cuda_device) for k, v in b.items()}
    lib = _lib.load()
    p_gpu = build(a, b_dev, policy, slack, True, escapes=escapes, split=split)
    p_host = build(a, b_dev, policy, slack, False, escapes=escapes, split=split)
    try:
        assert_same_plan(p_gpu, p_host)
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)


@pytest.fixture(scope="module")
def adversarial():
    return adversarial_pair(seed=5)


@pytest.mark.parametrize("slack, escapes, split", [(-1, -1, -1), (6, 0, 0), (100, 1, -1), (100, 1, 1), (100, 0, 4)])
@pytest.mark.parametrize("policy", ["auto", "xor", "u16"])
def test_gpu_encoder_matches_host_encoder_on_coding_limits(cuda_device, adversarial, policy: str, slack: int,
                                                          escapes: int, split: int) -> None:
    """255/256 distinct words (the device word table's limit), a lane's escape
    list at 64 entries and past it, extreme skew, an exact 16 MiB packet."""
    a, b = adversarial
    b_dev = {k: v.to(cuda_device) for k, v in b.items()}
    lib = _lib.load()
    p_gpu = build(a, b_dev, policy, slack, True, escapes=escapes, split=split)
    p_host = build(a, b_dev, policy, slack, False, escapes=escapes, split=split)
    try:
        assert_same_plan(p_gpu, p_host)
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)


def test_gpu_encoder_matches_on_unaligned_views_and_many_packets(cuda_device) -> None:
    x, y = bf16_pair((40 << 20) // 2 + 333, 0.01, 21)  # three packets, odd tail group
    storage = torch.zeros(x.numel() + 8, dtype=torch.bfloat16, device=cuda_device)
    view = storage[3 : 3 + x.numel()]
    view.copy_(y)
    lib = _lib.load()
    for policy in ("auto", "xor"):
        p_gpu = build({"w": x}, {"w": view}, policy, 6, True)
        p_host = build({"w": x}, {"w": view}, policy, 6, False)
        try:
            assert_same_plan(p_gpu, p_host)
        finally:
            lib.ws_plan_destroy(p_gpu)
            lib.ws_plan_destroy(p_host)


def test_gpu_encoder_matches_with_pinned_base(cuda_device) -> None:
    """Page-locked A goes to the device by DMA alone, without the staging threads."""
    a, b = edge_pair(seed=17)
    a_pinned = {k: v.pin_memory() for k, v in a.items()}
    b_dev = {k: v.to(cuda_device) for k, v in b.items()}
    lib = _lib.load()
    p_gpu = build(a_pinned, b_dev, "auto", 6, True)
    p_host = build(a, b_dev, "auto", 6, False)
    try:
        assert_same_plan(p_gpu, p_host)
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)


def test_gpu_encoder_arena_in_several_chunks(cuda_device) -> None:
    """16 MiB encoder batches over ~72 MiB of weights: five arena chunks. The plan,
    its contiguous view and a staged forward/reverse apply over the chunks match."""
    x, y = bf16_pair((72 << 20) // 2 + 77, 0.01, 5)
    x2, y2 = bf16_pair((3 << 20) // 2, 0.01, 6)
    a = {"w": x, "v": x2}
    b_dev = {"w": y.to(cuda_device), "v": y2.to(cuda_device)}
    lib = _lib.load()
    p_gpu = build(a, b_dev, "auto", 6, True, encode_batch_bytes=16 << 20, pin_arena=1, batch_bytes=3 << 20)
    p_host = build(a, b_dev, "auto", 6, False, pin_arena=1, batch_bytes=3 << 20)
    try:
        assert_same_plan(p_gpu, p_host)
        stats = _lib.PlanStats()
        _lib.check(lib.ws_plan_get_stats(p_gpu, ctypes.byref(stats)))
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.ws_plan_upload(p_gpu, stream))
        res = _lib.ApplyResult()
        _lib.check(lib.ws_apply(p_gpu, 1, stream, None, ctypes.byref(res)))  # B -> A
        assert res.launches == stats.batches > 1
        for k in a:
            assert torch.equal(b_dev[k].cpu().view(torch.int16), a[k].view(torch.int16)), k
        _lib.check(lib.ws_apply(p_gpu, 0, stream, None, ctypes.byref(res)))  # A -> B
        assert torch.equal(b_dev["w"].cpu().view(torch.int16), y.view(torch.int16))
        assert torch.equal(b_dev["v"].cpu().view(torch.int16), y2.view(torch.int16))
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)


def fill_device(cuda_device, leave: int) -> list:
    """Hold all but about `leave` bytes of free device memory in torch tensors."""
    torch.cuda.empty_cache()
    held = []
    free, _ = torch.cuda.mem_get_info(cuda_device)
    chunk = 1 << 30
    while free > leave + (2 << 20):
        size = min(chunk, free - leave)
        try:
            held.append(torch.empty(size, dtype=torch.uint8, device=cuda_device))
        except torch.OutOfMemoryError:
            if chunk <= (2 << 20):
                break
            chunk //= 2
        free, _ = torch.cuda.mem_get_info(cuda_device)
    return held


@pytest.mark.parametrize("leave_mb, encoder", [(190, "gpu"), (60, "host")])
def test_gpu_encoder_under_memory_pressure(cuda_device, leave_mb: int, encoder: str) -> None:
    """With little free HBM the GPU encoder retries with smaller batches (512 ->
    128 -> 32 MiB); below that the build fails with WS_ERR_NOMEM unless the host
    encoder was allowed to take over. Either encoder gives the same plan."""
    x, y = bf16_pair((96 << 20) // 2, 0.01, 31)
    b_dev = {"w": y.to(cuda_device)}
    lib = _lib.load()
    p_host = build({"w": x}, b_dev, "auto", 6, False)
    held = fill_device(cuda_device, leave_mb << 20)
    try:
        if encoder == "host":
            with pytest.raises(RuntimeError, match="host_fallback"):
                build({"w": x}, b_dev, "auto", 6, True)
        p_gpu = build({"w": x}, b_dev, "auto", 6, True, host_fallback=int(encoder == "host"))
    finally:
        del held
        torch.cuda.empty_cache()
    try:
        stats = _lib.PlanStats()
        _lib.check(lib.ws_plan_get_stats(p_gpu, ctypes.byref(stats)))
        assert _lib.ENCODERS[stats.encoder] == encoder
        assert_same_plan(p_gpu, p_host)
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)


@pytest.mark.parametrize("policy, scale, split, ks", [("xor", 0.01, 1, {1}), ("xor", 0.1, 0, {4}), ("u16", 0.1, 2, {2}),
                                                     ("u16", 0.1, 4, {4})])
def test_split_words_on_teacher_like_residuals(cuda_device, policy: str, scale: float, split: int, ks: set) -> None:
    """Split words on relative-noise BF16 pairs (the default picks k = 4 at XOR
    s = 0.1; the others are forced): both encoders give the same plan, and the
    kernel switches B -> A -> B exactly."""
    from tests.helpers import split_bits

    x, y = bf16_pair((24 << 20) // 2 + 4097, scale, 41)  # two packets, partial last block and group
    b_dev = {"w": y.to(cuda_device)}
    lib = _lib.load()
    p_gpu = build({"w": x}, b_dev, policy, 6, True, pin_arena=1, split=split)
    p_host = build({"w": x}, b_dev, policy, 6, False, split=split)
    try:
        assert_same_plan(p_gpu, p_host)
        blocks = plan_arrays(p_gpu)[0]
        coded = blocks[blocks["kind"] != 0]
        assert {split_bits(f) for f in coded["flags"]} == ks
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.ws_plan_upload(p_gpu, stream))
        res = _lib.ApplyResult()
        _lib.check(lib.ws_apply(p_gpu, 1, stream, None, ctypes.byref(res)))  # B -> A
        assert res.checksum == res.expected and res.device_errors == 0
        assert torch.equal(b_dev["w"].cpu().view(torch.int16), x.view(torch.int16))
        _lib.check(lib.ws_apply(p_gpu, 0, stream, None, ctypes.byref(res)))  # A -> B
        assert res.checksum == res.expected
        assert torch.equal(b_dev["w"].cpu().view(torch.int16), y.view(torch.int16))
    finally:
        lib.ws_plan_destroy(p_gpu)
        lib.ws_plan_destroy(p_host)
