"""Synthetic BF16 model pairs for the benchmark and parity workloads.

No checkpoints are available offline, so Teacher1/Teacher2 are generated with
fixed conventions:
  * Teacher1: BF16 of N(0, 0.02) for weights and biases, norm weights = 1.0,
    derived fp32 buffers (the rotary cos/sin cache) computed from positions;
  * Teacher2: bf16(fp32(T1) + s * |fp32(T1)| * N(0, 1)) with s = 0.01 by default,
    applied to every weight, norm and bias except where a sparse mask says
    otherwise (MoE: attention tensors and experts 0 and 1 only);
  * random streams: tensor k (in parameter-walk order) draws T1 from a generator
    seeded 1_000_003 * seed_t1 + k and the noise from 1_000_003 * seed_noise + k
    (seed_t1 = 0, seed_noise = 1), on the device the tensor lives on. The small
    CPU workload (Qwen2-0.5B shape) instead draws every tensor in order from one
    NumPy ``default_rng(0)`` / ``default_rng(1)`` stream.
Tensor names, shapes and the tensor-parallel split follow SGLang's layouts for
these architectures: merged ``qkv_proj`` and ``gate_up_proj`` split by output
rows (column parallel), ``o_proj`` and ``down_proj`` split by input columns (row
parallel), vocabulary-parallel ``embed_tokens``/``lm_head``, replicated norms
and router, MoE expert weights ``w13`` [E, 2F/tp, H] and ``w2`` [E, H, F/tp].
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

SEED_STRIDE = 1_000_003


@dataclass(frozen=True)
class ModelShape:
    name: str
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    tied: bool = False
    qkv_bias: bool = False
    experts: int = 0
    rope_positions: int = 0  # rows of the fp32 cos/sin cache buffer (0 = none)


QWEN2_0_5B = ModelShape("qwen2-0.5b", 24, 896, 4864, 14, 2, 64, 151936, tied=True, qkv_bias=True)
LLAMA3_8B = ModelShape("llama3-8b", 32, 4096, 14336, 32, 8, 128, 128256, rope_positions=8192)
LLAMA3_70B = ModelShape("llama3-70b", 80, 8192, 28672, 64, 8, 128, 128256, rope_positions=8192)
MIXTRAL_8X7B = ModelShape("mixtral-8x7b", 32, 4096, 14336, 32, 8, 128, 32000, experts=8, rope_positions=8192)
SHAPES = {s.name: s for s in (QWEN2_0_5B, LLAMA3_8B, LLAMA3_70B, MIXTRAL_8X7B)}


@dataclass
class TensorSpec:
    name: str
    shape: tuple[int, ...]
    dtype: torch.dtype = torch.bfloat16
    kind: str = "weight"  # weight | norm | bias | rope
    perturb: bool = True
    perturb_experts: tuple[int, ...] | None = None  # MoE: only these leading-dim slices change

    @property
    def nbytes(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * torch.empty((), dtype=self.dtype).element_size()


@dataclass
class ModelSpec:
    shape: ModelShape
    tp: int = 1
    rank: int = 0
    tensors: list[TensorSpec] = field(default_factory=list)

    @property
    def nbytes(self) -> int:
        return sum(t.nbytes for t in self.tensors)


def _split(n: int, tp: int, what: str) -> int:
    if n % tp:
        raise ValueError(f"{what}={n} is not divisible by tp={tp}")
    return n // tp


def model_spec(shape: ModelShape | str, tp: int = 1, rank: int = 0, moe_perturbed_experts: tuple[int, ...] = (0, 1)) -> ModelSpec:
    """Parameter list of one tensor-parallel rank, in SGLang's parameter-walk order."""
    s = SHAPES[shape] if isinstance(shape, str) else shape
    if not 0 <= rank < tp:
        raise ValueError("rank out of range")
    h, d = s.hidden, s.head_dim
    q_rows = _split(s.heads, tp, "heads") * d
    kv_heads = max(1, s.kv_heads // tp)  # KV heads are replicated when tp > kv_heads
    qkv_rows = q_rows + 2 * kv_heads * d
    vocab = _split(s.vocab, tp, "vocab")
    ffn = _split(s.ffn, tp, "ffn")
    moe = s.experts > 0
    attn_only = moe  # sparse delta: attention and selected experts change, the rest is identical
    out = [TensorSpec("parameter:model.embed_tokens.weight", (vocab, h), perturb=not attn_only)]
    for i in range(s.layers):
        p = f"parameter:model.layers.{i}."
        out.append(TensorSpec(p + "self_attn.qkv_proj.weight", (qkv_rows, h)))
        if s.qkv_bias:
            out.append(TensorSpec(p + "self_attn.qkv_proj.bias", (qkv_rows,), kind="bias"))
        out.append(TensorSpec(p + "self_attn.o_proj.weight", (h, _split(h, tp, "hidden"))))
        if moe:
            out.append(TensorSpec(p + "block_sparse_moe.gate.weight", (s.experts, h), perturb=False))
            out.append(
                TensorSpec(p + "block_sparse_moe.experts.w13_weight", (s.experts, 2 * ffn, h), perturb_experts=moe_perturbed_experts)
            )
            out.append(
                TensorSpec(p + "block_sparse_moe.experts.w2_weight", (s.experts, h, ffn), perturb_experts=moe_perturbed_experts)
            )
        else:
            out.append(TensorSpec(p + "mlp.gate_up_proj.weight", (2 * ffn, h)))
            out.append(TensorSpec(p + "mlp.down_proj.weight", (h, ffn)))
        out.append(TensorSpec(p + "input_layernorm.weight", (h,), kind="norm", perturb=not attn_only))
        out.append(TensorSpec(p + "post_attention_layernorm.weight", (h,), kind="norm", perturb=not attn_only))
    out.append(TensorSpec("parameter:model.norm.weight", (h,), kind="norm", perturb=not attn_only))
    if not s.tied:
        out.append(TensorSpec("parameter:lm_head.weight", (vocab, h), perturb=not attn_only))
    if s.rope_positions:
        out.append(TensorSpec("buffer:model.layers.0.self_attn.rotary_emb.cos_sin_cache", (s.rope_positions, d), torch.float32, kind="rope", perturb=False))
    return ModelSpec(s, tp, rank, out)


def _rope_cache(positions: int, dim: int, device: torch.device | str) -> torch.Tensor:
    inv = 1.0 / (500000.0 ** (torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim))
    freqs = torch.arange(positions, dtype=torch.float32, device=device)[:, None] * inv[None, :]
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1)


def _generator(device: torch.device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def teacher1_tensor(spec: TensorSpec, index: int, device: torch.device | str, seed: int = 0) -> torch.Tensor:
    device = torch.device(device)
    if spec.kind == "norm":
        return torch.ones(spec.shape, dtype=spec.dtype, device=device)
    if spec.kind == "rope":
        return _rope_cache(spec.shape[0], spec.shape[1], device).to(spec.dtype)
    g = _generator(device, SEED_STRIDE * seed + index)
    return (torch.randn(spec.shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(spec.dtype)


@torch.no_grad()
def perturb_(tensor: torch.Tensor, spec: TensorSpec, index: int, scale: float, seed: int = 1) -> torch.Tensor:
    """In place: T2 = bf16(fp32(T1) + scale * |fp32(T1)| * N(0, 1)) on the perturbed part."""
    if not spec.perturb or scale == 0:
        return tensor
    g = _generator(tensor.device, SEED_STRIDE * seed + index)
    if spec.perturb_experts is None:
        parts = [tensor]
    else:
        parts = [tensor[e] for e in spec.perturb_experts]
    for part in parts:
        f = part.float()
        noise = torch.randn(part.shape, generator=g, device=tensor.device, dtype=torch.float32)
        part.copy_((f + scale * f.abs() * noise).to(tensor.dtype))
    return tensor


def generate_teacher1(spec: ModelSpec, device: torch.device | str, seed: int = 0) -> dict[str, torch.Tensor]:
    return {t.name: teacher1_tensor(t, i, device, seed) for i, t in enumerate(spec.tensors)}


def generate_pair_numpy(spec: ModelSpec, scale: float = 0.01) -> tuple[dict[str, torch.Tensor], dict[str, torch.Tensor]]:
    """CPU pair from np.random.default_rng(0) (Teacher1) and default_rng(1) (noise), tensors in order."""
    rng1, rng2 = np.random.default_rng(0), np.random.default_rng(1)
    t1, t2 = {}, {}
    for i, t in enumerate(spec.tensors):
        if t.kind == "norm":
            a = torch.ones(t.shape, dtype=t.dtype)
        elif t.kind == "rope":
            a = _rope_cache(t.shape[0], t.shape[1], "cpu").to(t.dtype)
        else:
            a = torch.from_numpy((rng1.standard_normal(t.shape, dtype=np.float32) * 0.02)).to(t.dtype)
        b = a.clone()
        if t.perturb and scale:
            parts = [(a, b)] if t.perturb_experts is None else [(a[e], b[e]) for e in t.perturb_experts]
            for pa, pb in parts:
                f = pa.float()
                noise = torch.from_numpy(rng2.standard_normal(pa.shape, dtype=np.float32))
                pb.copy_((f + scale * f.abs() * noise).to(t.dtype))
        t1[t.name], t2[t.name] = a, b
    return t1, t2
