"""Device-side per-tensor hashes (ws_tensor_hashes) against the oracle's NumPy form."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import hashes
from warpshift_b200.verify import tensor_hashes

pytestmark = pytest.mark.gpu


def host_bytes(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().reshape(-1).view(torch.uint8).cpu().numpy().tobytes()


def test_hashes_match_the_oracle_on_every_size_class(cuda_device) -> None:
    g = torch.Generator().manual_seed(3)
    storage = torch.randint(0, 256, ((40 << 20) + 123,), dtype=torch.uint8, generator=g).to(cuda_device)
    tensors = {
        "empty": torch.empty(0, dtype=torch.bfloat16, device=cuda_device),
        "one_byte": storage[5:6],
        "odd_unaligned": storage[3 : 3 + 65_537],               # base not 8-byte aligned
        "aligned8_only": storage[8 : 8 + 1_000_001],            # 8- but not 16-byte aligned
        "bf16": torch.randn(4099, 1024, generator=g).to(torch.bfloat16).to(cuda_device),
        "fp32_buffer": torch.randn(777, generator=g).to(cuda_device),
        "large": storage[256 : 256 + (32 << 20) + 9],           # many 64 KiB segments, ragged tail
        "strided": torch.randn(300, 400, generator=g).to(cuda_device).t(),  # non-contiguous
    }
    got = tensor_hashes(tensors)
    assert list(got) == list(tensors)
    for name, t in tensors.items():
        assert got[name] == hashes.hex_hash(np.frombuffer(host_bytes(t), dtype=np.uint8)), name


def test_one_flipped_bit_changes_only_its_tensor(cuda_device) -> None:
    g = torch.Generator().manual_seed(4)
    a = torch.randn(1 << 20, generator=g).to(torch.bfloat16).to(cuda_device)
    b = a.clone()
    before = tensor_hashes({"a": a, "b": b})
    assert before["a"] == before["b"]
    b.view(torch.int16)[123_457] ^= 1
    after = tensor_hashes({"a": a, "b": b})
    assert after["a"] == before["a"] and after["b"] != before["b"]
    assert after["b"] == hashes.hex_hash(np.frombuffer(host_bytes(b), dtype=np.uint8))
