"""Drop-in replacement for the reference's ``warpshift/delta.py`` (DeltaWeights).

Same Python surface as warpshift/delta.py:95-327: ``DeltaWeights(cpu_base,
gpu_target)``, ``.apply(reverse)``, ``.validate_bindings()``, ``.bindings``,
``.device``, ``.stats`` and the module helpers ``_u16_residual`` and
``_batch_layout``. Underneath, nvCOMP and the Triton ``_restore_batch`` kernel
are replaced by ``libwarpshift_b200.so``: a GPU encoder for prepare (statistics,
rANS encode and packing kernels; host encoder threads only on request) and one fused
sm_100a decode+apply kernel per staging batch for apply.

Per-packet mode choice keeps the reference rule (delta.py:176-194: raw XOR, then
grouped/odd XOR-ANS, then U16-ANS, strictly-smaller wins). The keyword-only
``policy`` argument ("auto" = that rule, "xor", "u16") restricts the candidate
set, which the XOR-only and U16-only benchmark configurations need.
"""

from __future__ import annotations

import ctypes
import os
import time
from typing import Any

import numpy as np
import torch

from . import _lib

_CHUNK_BYTES = 16 * 1024**2  # delta.py:20, packet size
_BATCH_BYTES = 64 * 1024**2  # delta.py:21, default bound of _batch_layout
_BLOCK_BYTES = 131072  # rANS block: one warp decodes one block (WS_BLOCK_BYTES)
_STAGING_BATCH_BYTES = 64 * 1024**2  # H2D staging batch bound, as the reference's BATCH_BYTES (delta.py:21)
# A packet whose 16-bit residual words take <= 255 values may be coded one
# symbol per word (half the decode work of the two byte planes); it is chosen
# when its estimated size is at most this many percent above the planes'.
_DICT_SLACK_PCT = 6
_MODES = {0: "XOR_RAW", 1: "XOR_GROUP2_ANS", 2: "XOR_ANS", 3: "U16_ANS"}  # delta.py:23


def _u16_residual(base: np.ndarray, target: np.ndarray) -> np.ndarray:
    """Grouped low/high bytes of zigzag((B - A) mod 65536), without float math (delta.py:26-34)."""
    base = np.ascontiguousarray(base, dtype=np.uint8).reshape(-1)
    target = np.ascontiguousarray(target, dtype=np.uint8).reshape(-1)
    if base.size != target.size:
        raise ValueError("Residual inputs differ in size")
    out = np.empty(base.size, dtype=np.uint8)
    _lib.check(_lib.load().ws_u16_residual(base.ctypes.data, target.ctypes.data, base.size, out.ctypes.data))
    return out


def _batch_layout(sizes: list[tuple[int, int]], limit: int = _BATCH_BYTES) -> list[dict[str, Any]]:
    """Bound both encoded and decoded arenas; 256-byte aligned frames (delta.py:37-57).

    Kept with the reference's semantics for callers of the helper; the native
    plan bounds its own staging batches (only encoded bytes are staged, since the
    fused kernel decodes straight into the weights).
    """
    batches: list[dict[str, Any]] = []
    current: list[tuple[int, int, int]] = []
    input_end = output_end = offset = 0
    for index, (encoded, decoded) in enumerate(sizes):
        if encoded <= 0 or decoded < 0 or encoded > limit or decoded > limit:
            raise ValueError("Invalid delta frame size")
        start_in = (input_end + 255) & ~255
        start_out = (output_end + 255) & ~255
        if current and (start_in + encoded > limit or start_out + decoded > limit):
            batches.append(dict(payload_offset=offset, input_bytes=input_end, decoded_bytes=output_end, packets=current))
            offset += input_end
            current, start_in, start_out = [], 0, 0
        current.append((index, start_in, start_out))
        input_end, output_end = start_in + encoded, start_out + decoded
    if current:
        batches.append(dict(payload_offset=offset, input_bytes=input_end, decoded_bytes=output_end, packets=current))
    return batches


class DeltaWeights:
    """One rank's A<->B package; the caller owns model identity and update serialization.

    ``cpu_base`` contains A and ``gpu_target`` currently contains B. Construction
    never changes GPU weights and keeps no full CPU copy of A: only the encoded
    stream, in pinned host memory.

    Keyword-only options beyond the reference: ``policy`` ("auto" = the
    reference's mode rule, "xor", "u16"), ``threads`` (host threads; 0 = all),
    ``batch_bytes`` (bound on one H2D staging batch), ``staging_slots``,
    ``dict_slack_pct`` (word-dictionary coding when within this many percent of
    the byte planes' size; negative = never), ``encode_on_device`` (prepare on
    the GPU), ``encode_batch_bytes`` (GPU encoder batch; 0 = 512 MiB),
    ``escapes`` (dictionaries with escape lists: 0 when smaller, -1 never, 1
    whenever eligible), ``split`` (split-word dictionaries, whose words' low k
    bits are stored raw: 0 the k estimated smallest, a split one only when 3 %
    smaller than whole words, -1 never, 1 / 2 / 4 that k whenever eligible)
    and ``host_fallback`` (when the GPU encoder cannot get
    its device buffers, encode on host threads instead of raising
    RuntimeError; off by default). ``save`` / ``load`` persist a package
    across restarts.
    """

    def __init__(
        self,
        cpu_base: dict[str, torch.Tensor],
        gpu_target: dict[str, torch.Tensor],
        *,
        policy: str = "auto",
        threads: int = 0,
        batch_bytes: int = _STAGING_BATCH_BYTES,
        staging_slots: int = 3,
        dict_slack_pct: int = _DICT_SLACK_PCT,
        encode_on_device: bool = True,
        encode_batch_bytes: int = 0,
        escapes: int = 0,
        split: int = 0,
        host_fallback: bool = False,
    ) -> None:
        started = time.perf_counter()
        if policy not in _lib.POLICIES:
            raise ValueError(f"Unknown delta policy: {policy}")
        self._plan = None
        self._bind_tensors(cpu_base, gpu_target)
        self._native = _lib.load()
        self.policy = policy
        self.compute_stream = torch.cuda.current_stream(self.device)
        self.copy_stream = torch.cuda.Stream(device=self.device)
        descs = (_lib.TensorDesc * len(gpu_target))()
        for index, (name, target) in enumerate(gpu_target.items()):
            base = cpu_base[name]
            descs[index] = _lib.TensorDesc(
                base.data_ptr(),
                target.data_ptr(),
                target.numel() * target.element_size(),
                int(target.dtype == torch.bfloat16),
                0,
            )
        options = _lib.BuildOptions(
            policy=_lib.POLICIES[policy],
            threads=threads,
            target_on_device=1,
            device=self.device.index,
            batch_bytes=batch_bytes,
            staging_slots=staging_slots,
            pin_arena=1,
            dict_slack_pct=dict_slack_pct,
            encode_on_device=int(bool(encode_on_device)),
            encode_batch_bytes=encode_batch_bytes,
            escapes=escapes,
            host_fallback=int(bool(host_fallback)),
            split=split,
        )
        plan = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            stream = self.compute_stream.cuda_stream
            _lib.check(self._native.ws_plan_build(descs, len(gpu_target), ctypes.byref(options), stream, ctypes.byref(plan)))
            self._plan = plan
        self._finish(started, batch_bytes, dict_slack_pct)

    @classmethod
    def load(
        cls,
        path: str | os.PathLike,
        gpu_target: dict[str, torch.Tensor],
        *,
        threads: int = 0,
        batch_bytes: int = _STAGING_BATCH_BYTES,
        staging_slots: int = 3,
    ) -> "DeltaWeights":
        """Re-create a package written by ``save`` for ``gpu_target`` (no prepare, no A).

        ``gpu_target`` must hold the same tensors (names in the same order, same
        shapes and dtypes) as when the package was built; its storage may live at
        new addresses. The first ``apply`` checks, through the checksum recorded at
        prepare, that the resident weights are the expected source model. Raises
        ``ValueError`` if the file does not match the tensors and ``OSError`` if it
        cannot be read.
        """
        started = time.perf_counter()
        self = cls.__new__(cls)
        self._plan = None
        self._bind_targets(gpu_target)
        self._native = _lib.load()
        self.policy = "saved"
        self.compute_stream = torch.cuda.current_stream(self.device)
        self.copy_stream = torch.cuda.Stream(device=self.device)
        descs = (_lib.TensorDesc * len(gpu_target))()
        for index, target in enumerate(gpu_target.values()):
            descs[index] = _lib.TensorDesc(
                None, target.data_ptr(), target.numel() * target.element_size(), int(target.dtype == torch.bfloat16), 0
            )
        options = _lib.BuildOptions(
            policy=0, threads=threads, target_on_device=1, device=self.device.index, batch_bytes=batch_bytes,
            staging_slots=staging_slots, pin_arena=1, dict_slack_pct=_DICT_SLACK_PCT, encode_on_device=0,
        )
        plan = ctypes.c_void_p()
        _lib.check(self._native.ws_plan_load(os.fsencode(path), descs, len(gpu_target), ctypes.byref(options), ctypes.byref(plan)))
        self._plan = plan
        self._finish(started, batch_bytes, None)
        self.stats["loaded_from"] = os.fspath(path)
        return self

    def save(self, path: str | os.PathLike) -> None:
        """Write the package (descriptors, tables, checksums, encoded stream) to ``path``."""
        _lib.check(self._native.ws_plan_save(self._plan, os.fsencode(path)))

    def _finish(self, started: float, batch_bytes: int, dict_slack_pct: int | None) -> None:
        with torch.cuda.device(self.device):
            _lib.check(self._native.ws_plan_upload(self._plan, self.compute_stream.cuda_stream))
        self.last_apply: dict[str, Any] | None = None
        native = self.native_stats()
        counts = {name: int(native.mode_counts[i]) for i, name in enumerate(_lib.MODE_NAMES) if native.mode_counts[i]}
        self.stats = {
            "codec": "U16_XOR_RANS_SM100",
            "reversible": True,
            "chunk_bytes": _CHUNK_BYTES,
            "batch_bytes": batch_bytes,
            "runtime_bytes": int(native.runtime_bytes),
            "skipped_bytes": int(native.skipped_bytes),
            "payload_bytes": int(native.payload_bytes),
            "transferred_bytes": int(native.arena_bytes),
            "pinned_bytes": int(native.arena_bytes),
            "mode_counts": counts,
            "batches": int(native.batches),
            "gpu_scratch_bytes": int(native.scratch_bytes),
            "gpu_metadata_bytes": int(native.metadata_bytes),
            "memory_scope": "Staging slots, descriptors and decode tables; excludes the CUDA context and allocator caching",
            "prepare_seconds": time.perf_counter() - started,
            # Additions of this implementation.
            "policy": self.policy,
            "dict_slack_pct": dict_slack_pct,
            "encoder": _lib.ENCODERS.get(int(native.encoder), "unknown"),
            "block_bytes": _BLOCK_BYTES,
            "touched_bytes": int(native.touched_bytes),
            "zero_block_bytes": int(native.zero_block_bytes),
            "compression_ratio": (int(native.touched_bytes) / int(native.arena_bytes)) if native.arena_bytes else None,
            "blocks": int(native.blocks),
            "encode_seconds": float(native.encode_seconds),
        }

    def _bind_tensors(self, cpu_base: dict[str, torch.Tensor], gpu_target: dict[str, torch.Tensor]) -> None:
        """Validate the A/B layout and retain GPU storage bindings (delta.py:137-162)."""
        if not cpu_base or cpu_base.keys() != gpu_target.keys():
            raise ValueError("Delta tensor coverage differs")
        self._bind_targets(gpu_target, cpu_base)

    def _bind_targets(self, gpu_target: dict[str, torch.Tensor], cpu_base: dict[str, torch.Tensor] | None = None) -> None:
        """The checks of delta.py:141-162 in their order; without ``cpu_base`` (a loaded
        package) only the GPU side is checked."""
        if not gpu_target:
            raise ValueError("Delta tensor coverage differs")
        devices = {tensor.device for tensor in gpu_target.values()}
        if len(devices) != 1 or next(iter(devices)).type != "cuda":
            raise ValueError("Delta tensors must reside on one CUDA device")
        self.device = next(iter(devices))
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.bindings = []
        spans = []
        for name, target in gpu_target.items():
            base = cpu_base[name] if cpu_base is not None else None
            if base is not None and (base.device.type != "cpu" or base.shape != target.shape or base.dtype != target.dtype):
                raise ValueError(f"Delta layout differs: {name}")
            if (base is not None and not base.is_contiguous()) or not target.is_contiguous():
                raise ValueError(f"Delta requires contiguous tensors: {name}")
            size = target.numel() * target.element_size()
            if size:
                spans.append((target.data_ptr(), target.data_ptr() + size, name))
            self.bindings.append((target, target.data_ptr(), tuple(target.shape), tuple(target.stride()), target.dtype))
        spans.sort()
        for previous, current in zip(spans, spans[1:]):
            if current[0] < previous[1]:
                raise ValueError(f"Delta cannot update overlapping tensors: {previous[2]}, {current[2]}")

    def validate_bindings(self) -> None:
        """Reject changed GPU storage before dereferencing prepared kernel pointers (delta.py:282-292)."""
        for tensor, pointer, shape, stride, dtype in self.bindings:
            if (
                tensor.data_ptr() != pointer
                or tuple(tensor.shape) != shape
                or tuple(tensor.stride()) != stride
                or tensor.dtype != dtype
                or tensor.device != self.device
            ):
                raise ValueError("Delta GPU tensor storage changed; prepare again")

    def native_stats(self) -> _lib.PlanStats:
        stats = _lib.PlanStats()
        _lib.check(self._native.ws_plan_get_stats(self._plan, ctypes.byref(stats)))
        return stats

    @torch.no_grad()
    def apply(self, reverse: bool) -> None:
        """A->B when false, B->A when true; return only after GPU completion (delta.py:294-327).

        Raises RuntimeError if the device reports a corrupt frame or if the
        written bytes do not hash to the checksum recorded at prepare (for
        example when the resident weights were not the expected source model).
        Before raising, the library rolls the switch back by applying the other
        direction over the same stream; ``last_apply["rollback"]`` is
        "restored" when the restored bytes hash to the source model's checksum
        (see ``include/warpshift_b200.h``, ``WS_ROLLBACK_*``).
        """
        self.validate_bindings()
        caller_stream = torch.cuda.current_stream(self.device)
        self.compute_stream.wait_stream(caller_stream)
        result = _lib.ApplyResult()
        with torch.cuda.device(self.device):
            rc = self._native.ws_apply(
                self._plan,
                int(bool(reverse)),
                self.compute_stream.cuda_stream,
                self.copy_stream.cuda_stream,
                ctypes.byref(result),
            )
        self.last_apply = {
            "reverse": bool(reverse),
            "ok": rc == _lib.WS_OK,
            "checksum": int(result.checksum),
            "expected": int(result.expected),
            "device_errors": int(result.device_errors),
            "h2d_bytes": int(result.h2d_bytes),
            "launches": int(result.launches),
            "rollback": _lib.ROLLBACK.get(int(result.rollback), "unknown"),
        }
        _lib.check(rc)

    def confirm(self, group: Any = None, failed: bool = False) -> dict[str, int]:
        """All-reduce one success flag per rank over ``group`` (NCCL in production).

        This rank's flag is up when its last apply succeeded, the bytes it wrote
        hash to the checksum recorded at prepare, and ``failed`` is false.
        Counting flags (rather than summing checksums, whose errors on two ranks
        could cancel) tells every rank whether the whole switch happened. Raises
        RuntimeError naming how many ranks failed.
        """
        import torch.distributed as dist

        last = self.last_apply or {}
        ok = not failed and bool(last.get("ok")) and last.get("checksum") == last.get("expected")
        on_device = dist.get_backend(group) == "nccl"
        flags = torch.tensor([0 if ok else 1, 1], dtype=torch.int64, device=self.device if on_device else "cpu")
        dist.all_reduce(flags, group=group)
        failed_ranks, ranks = (int(v) for v in flags.tolist())
        if failed_ranks:
            raise RuntimeError(f"Delta switch not confirmed: {failed_ranks} of {ranks} rank(s) failed")
        return {"failed_ranks": 0, "ranks": ranks}

    def set_resident(self, resident: bool) -> None:
        """Keep the whole encoded stream in HBM (applies then skip the H2D staging)."""
        with torch.cuda.device(self.device):
            _lib.check(self._native.ws_plan_set_resident(self._plan, int(resident), self.compute_stream.cuda_stream))

    def apply_async(self, reverse: bool, stream: torch.cuda.Stream | None = None) -> None:
        """Enqueue an apply on ``stream`` (default: the compute stream) without waiting."""
        stream = stream or self.compute_stream
        with torch.cuda.device(self.device):
            _lib.check(self._native.ws_apply_async(self._plan, int(bool(reverse)), stream.cuda_stream, self.copy_stream.cuda_stream))

    def finish(self, stream: torch.cuda.Stream | None = None) -> dict[str, int]:
        """Wait for an ``apply_async`` and check its result like ``apply`` does."""
        stream = stream or self.compute_stream
        result = _lib.ApplyResult()
        rc = self._native.ws_apply_finish(self._plan, stream.cuda_stream, ctypes.byref(result))
        self.last_apply = {
            "reverse": None,
            "ok": rc == _lib.WS_OK,
            "checksum": int(result.checksum),
            "expected": int(result.expected),
            "device_errors": int(result.device_errors),
            "h2d_bytes": int(result.h2d_bytes),
            "launches": int(result.launches),
        }
        _lib.check(rc)
        return self.last_apply

    def plan_view(self) -> _lib.PlanView:
        view = _lib.PlanView()
        _lib.check(self._native.ws_plan_get_view(self._plan, ctypes.byref(view)))
        return view

    def close(self) -> None:
        plan, self._plan = getattr(self, "_plan", None), None
        if plan:
            self._native.ws_plan_destroy(plan)

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

