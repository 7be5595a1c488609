"""GPU parity on the shapes of every benchmark configuration, truncated in depth.

Each case generates the Teacher pair on the device with the synth conventions,
prepares the delta with the GPU encoder, switches B -> A -> B -> A with the fused
kernel and compares every tensor, byte for byte, with the regenerated Teacher
(the reference's restore is exact, so the Teachers are the expected output):

* U16 mode at s in {0.001, 0.01, 0.1} on the Llama-3-8B shape (wrapping uint16
  add/subtract, delta.py:77-85);
* every one of the eight TP=8 shards of the Llama-3-70B shape (SGLang split:
  column-parallel QKV and gate/up, row-parallel o/down, vocabulary-parallel
  embedding and lm_head);
* the sparse Mixtral-8x7B TP=8 shard, whose skipped packets (delta.py:181-182,
  209-212) and all-zero blocks must match the oracle's count.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from oracle import semantics as sem
from warpshift_b200 import synth
from warpshift_b200.delta import _BLOCK_BYTES, DeltaWeights

pytestmark = pytest.mark.gpu


def generate(spec: synth.ModelSpec, device, scale: float):
    """Teacher1 in host memory (cpu_base), Teacher2 resident on the device."""
    cpu_base, gpu = {}, {}
    for i, t in enumerate(spec.tensors):
        x = synth.teacher1_tensor(t, i, device)
        cpu_base[t.name] = x.cpu()
        gpu[t.name] = synth.perturb_(x, t, i, scale)
    torch.cuda.synchronize(device)
    return cpu_base, gpu


def assert_teacher(spec: synth.ModelSpec, gpu, device, scale: float, teacher2: bool) -> None:
    for i, t in enumerate(spec.tensors):
        ref = synth.teacher1_tensor(t, i, device)
        if teacher2:
            synth.perturb_(ref, t, i, scale)
        got = gpu[t.name].reshape(-1).view(torch.uint8)
        if not torch.equal(ref.reshape(-1).view(torch.uint8), got):
            bad = int((ref.reshape(-1).view(torch.uint8) != got).nonzero()[0])
            raise AssertionError(f"{t.name}: byte {bad} differs from Teacher{2 if teacher2 else 1}")


def round_trip(spec, device, scale: float, policy: str) -> DeltaWeights:
    cpu_base, gpu = generate(spec, device, scale)
    delta = DeltaWeights(cpu_base, gpu, policy=policy)
    assert delta.stats["encoder"] == "gpu"
    assert_teacher(spec, gpu, device, scale, teacher2=True)  # prepare never changes GPU weights
    for reverse in (True, False, True):
        delta.apply(reverse=reverse)
        assert delta.last_apply["ok"] and delta.last_apply["checksum"] == delta.last_apply["expected"]
        assert_teacher(spec, gpu, device, scale, teacher2=not reverse)
    delta.close()
    return delta


@pytest.mark.parametrize("scale", [0.001, 0.01, 0.1])
def test_config2_llama8b_u16_sweep_every_tensor(cuda_device, scale: float) -> None:
    spec = synth.model_spec(dataclasses.replace(synth.LLAMA3_8B, layers=1))
    delta = round_trip(spec, cuda_device, scale, "u16")
    counts = delta.stats["mode_counts"]
    assert counts.get("U16_ANS", 0) > 0 and set(counts) <= {"U16_ANS", "XOR_RAW", "XOR_GROUP2_ANS", "SKIP"}


@pytest.mark.parametrize("rank", range(8))
def test_config3_llama70b_tp8_every_shard(cuda_device, rank: int) -> None:
    spec = synth.model_spec(dataclasses.replace(synth.LLAMA3_70B, layers=1), tp=8, rank=rank)
    names = {t.name: t.shape for t in spec.tensors}
    assert names["parameter:model.layers.0.self_attn.qkv_proj.weight"] == (1280, 8192)
    assert names["parameter:model.layers.0.mlp.down_proj.weight"] == (8192, 3584)
    assert names["parameter:lm_head.weight"] == (16032, 8192)
    round_trip(spec, cuda_device, 0.01, "auto")


def test_config4_mixtral_tp8_sparse_skips_like_the_oracle(cuda_device) -> None:
    spec = synth.model_spec(dataclasses.replace(synth.MIXTRAL_8X7B, layers=2), tp=8, rank=3)
    cpu_base, gpu = generate(spec, cuda_device, 0.01)
    # Oracle count: packets of 16 MiB whose XOR is all zero are skipped
    # (delta.py:181-182, 209-212); inside written packets, blocks whose XOR is
    # all zero are omitted from the stream.
    skipped = zero_blocks = 0
    for name, target in gpu.items():
        a = cpu_base[name].reshape(-1).view(torch.uint8).numpy()
        b = target.reshape(-1).view(torch.uint8).cpu().numpy()
        for off in range(0, b.size, sem.CHUNK_BYTES):
            xor = sem.xor_residual(a[off : off + sem.CHUNK_BYTES], b[off : off + sem.CHUNK_BYTES])
            if not xor.any():
                skipped += xor.size
                continue
            for k in range(0, xor.size, _BLOCK_BYTES):
                if not xor[k : k + _BLOCK_BYTES].any():
                    zero_blocks += xor[k : k + _BLOCK_BYTES].size
    assert skipped > 0.5 * spec.nbytes  # most of the shard is unchanged
    delta = DeltaWeights(cpu_base, gpu, policy="auto")
    assert delta.stats["skipped_bytes"] == skipped
    assert delta.stats["zero_block_bytes"] == zero_blocks
    assert delta.stats["touched_bytes"] == spec.nbytes - skipped - zero_blocks
    for reverse in (True, False):
        delta.apply(reverse=reverse)
        assert delta.last_apply["ok"]
        assert_teacher(spec, gpu, cuda_device, 0.01, teacher2=not reverse)
    delta.close()


def test_config0_numpy_pair_matches_oracle_restore(cuda_device) -> None:
    """Config 0's CPU pair (Qwen2-0.5B shape, NumPy streams), restored by the kernel
    and by the oracle's restatement of the reference restore: identical bytes."""
    spec = synth.model_spec(dataclasses.replace(synth.QWEN2_0_5B, layers=2))
    t1, t2 = synth.generate_pair_numpy(spec, 0.01)
    gpu = {k: v.to(cuda_device) for k, v in t2.items()}
    delta = DeltaWeights(t1, gpu, policy="auto")
    work = {k: v.reshape(-1).view(torch.uint8).numpy().copy() for k, v in t2.items()}
    base = {k: v.reshape(-1).view(torch.uint8).numpy() for k, v in t1.items()}
    bf16 = {k: v.dtype == torch.bfloat16 for k, v in t2.items()}
    packets, _, _ = sem.encode_packets(base, work, bf16, lambda r: r.size // 4)
    sem.apply_packets(work, packets, reverse=True)
    delta.apply(reverse=True)
    for name, t in gpu.items():
        np.testing.assert_array_equal(t.reshape(-1).view(torch.uint8).cpu().numpy(), work[name], err_msg=name)
    delta.close()
