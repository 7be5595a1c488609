"""Per-tensor content hashes computed on the GPU.

The reference's acceptance check (``scripts/validate.py:32-83``, the
``check_weights`` test loader) proves that a switched model equals a native load
by hashing every tensor with sha256 after copying it to the host in 64 MiB
pieces (``validate.py:50-56``). ``tensor_hashes`` gives the same per-tensor
verdict from one HBM-bound pass over the resident bytes: a 64-bit hash per
tensor (definition in ``include/warpshift_b200.h``), returned as 16 hex digits.
Equal bytes give equal hashes; any change of a tensor's bytes changes its hash
except with probability about 2^-64. It is a checksum against accidental
corruption, not a cryptographic digest.
"""

from __future__ import annotations

import ctypes
from collections.abc import Mapping

import torch

from warpshift_b200 import _lib


def tensor_hashes(tensors: Mapping[str, torch.Tensor]) -> dict[str, str]:
    """Hash each CUDA tensor's bytes (row-major, as ``validate.py:51`` flattens them).

    Non-contiguous tensors are hashed through a contiguous copy. Raises
    ``ValueError`` for tensors that are not on a CUDA device.
    """
    lib = _lib.load()
    names = list(tensors)
    out: dict[str, str] = {}
    by_device: dict[int, list[str]] = {}
    for name in names:
        t = tensors[name]
        if t.device.type != "cuda":
            raise ValueError(f"tensor_hashes needs CUDA tensors; {name} is on {t.device}")
        by_device.setdefault(t.device.index, []).append(name)
    for device, group in by_device.items():
        keep = []
        ptrs = (ctypes.c_void_p * len(group))()
        sizes = (ctypes.c_uint64 * len(group))()
        for i, name in enumerate(group):
            t = tensors[name].detach()
            if not t.is_contiguous():
                t = t.contiguous()
            keep.append(t)
            ptrs[i] = t.data_ptr()
            sizes[i] = t.numel() * t.element_size()
        result = (ctypes.c_uint64 * len(group))()
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device).cuda_stream
            _lib.check(lib.ws_tensor_hashes(ptrs, sizes, len(group), device, stream, result))
        for i, name in enumerate(group):
            out[name] = f"{result[i]:016x}"
    return {name: out[name] for name in names}
