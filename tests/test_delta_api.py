"""CPU invariants of the DeltaWeights drop-in, after the reference's tests/test_delta.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from warpshift_b200.delta import DeltaWeights, _batch_layout, _u16_residual


@pytest.mark.parametrize("base_word", [0, 0x3F80, 0x8000, 0xFFFF])
def test_u16_residual_round_trip_covers_every_bit_pattern(base_word: int) -> None:
    # Signed zero, infinities and every NaN payload, without float conversion (reference test_delta.py:12-24).
    target = np.arange(65536, dtype="<u2")
    base = np.full(target.shape, base_word, dtype="<u2")
    grouped = _u16_residual(base.view(np.uint8), target.view(np.uint8))
    words = grouped.reshape(2, -1).T.copy().reshape(-1).view("<u2").astype(np.int32)
    signed = np.where(words % 2, -(words // 2) - 1, words // 2)
    np.testing.assert_array_equal(((base.astype(np.int32) + signed) % 65536).astype("<u2"), target)
    np.testing.assert_array_equal(((target.astype(np.int32) - signed) % 65536).astype("<u2"), base)
    assert grouped.size == base.nbytes


def test_u16_residual_known_values_and_byte_grouping() -> None:
    base = np.array([0, 0, 0xFFFF, 0, 0x8000], dtype="<u2")
    target = np.array([0, 1, 0, 0xFFFF, 0], dtype="<u2")
    expected = np.array([0, 2, 2, 1, 255, 0, 0, 0, 0, 255], dtype=np.uint8)  # reference test_delta.py:27-32
    np.testing.assert_array_equal(_u16_residual(base.view(np.uint8), target.view(np.uint8)), expected)


def test_u16_residual_rejects_odd_sizes() -> None:
    with pytest.raises(ValueError, match="even"):
        _u16_residual(np.zeros(3, np.uint8), np.zeros(3, np.uint8))


def test_batch_layout_bounds_both_arenas_and_preserves_packet_order() -> None:
    sizes = [(300, 900), (300, 900), (700, 0), (400, 500), (1, 0)]
    batches = _batch_layout(sizes, limit=2048)
    indices, expected_offset = [], 0
    for batch in batches:
        assert batch["payload_offset"] == expected_offset
        expected_offset += batch["input_bytes"]
        assert 0 < batch["input_bytes"] <= 2048 and 0 <= batch["decoded_bytes"] <= 2048
        input_end = output_end = 0
        for index, input_offset, output_offset in batch["packets"]:
            encoded, decoded = sizes[index]
            assert input_offset % 256 == output_offset % 256 == 0
            assert input_offset >= input_end and output_offset >= output_end
            input_end, output_end = input_offset + encoded, output_offset + decoded
            assert input_end <= batch["input_bytes"] and output_end <= batch["decoded_bytes"]
            indices.append(index)
    assert indices == list(range(len(sizes))) and len(batches) > 1
    assert _batch_layout([]) == []


@pytest.mark.parametrize("size", [(0, 1), (-1, 1), (1, -1), (2049, 1), (1, 2049)])
def test_batch_layout_rejects_frames_that_cannot_fit(size: tuple[int, int]) -> None:
    with pytest.raises(ValueError, match="frame size"):
        _batch_layout([size], limit=2048)


def test_bindings_reject_changed_storage_without_requiring_cuda() -> None:
    # The drop-in keeps the reference's attribute contract: only .device and .bindings are used.
    tensor = torch.arange(8, dtype=torch.float32)
    delta = DeltaWeights.__new__(DeltaWeights)
    delta.device = tensor.device
    delta.bindings = [(tensor, tensor.data_ptr(), tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype)]
    delta.validate_bindings()
    tensor.data = tensor.clone()
    with pytest.raises(ValueError, match="storage changed"):
        delta.validate_bindings()


@pytest.mark.parametrize("change", ["shape", "stride", "dtype"])
def test_bindings_reject_shape_stride_and_dtype_changes(change: str) -> None:
    tensor = torch.zeros(4, 4)
    delta = DeltaWeights.__new__(DeltaWeights)
    delta.device = tensor.device
    delta.bindings = [(tensor, tensor.data_ptr(), tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype)]
    if change == "shape":
        tensor.resize_(2, 8)
    elif change == "stride":
        tensor.set_(tensor.untyped_storage(), 0, (4, 4), (1, 4))
    else:
        delta.bindings = [(tensor, tensor.data_ptr(), tuple(tensor.shape), tuple(tensor.stride()), torch.float16)]
    with pytest.raises(ValueError, match="storage changed"):
        delta.validate_bindings()


def _bind(cpu, gpu):
    delta = DeltaWeights.__new__(DeltaWeights)
    delta._plan = None
    return delta._bind_tensors(cpu, gpu)


def test_bind_rejects_coverage_device_layout_and_overlap() -> None:
    a = {"x": torch.zeros(4)}
    with pytest.raises(ValueError, match="coverage"):
        _bind(a, {"y": torch.zeros(4)})
    with pytest.raises(ValueError, match="coverage"):
        _bind({}, {})
    with pytest.raises(ValueError, match="one CUDA device"):
        _bind(a, {"x": torch.zeros(4)})  # CPU targets are rejected (delta.py:143-145)


def test_drop_in_constants_and_unknown_policy() -> None:
    from warpshift_b200 import delta

    assert delta._CHUNK_BYTES == 16 * 1024**2 and delta._BATCH_BYTES == 64 * 1024**2
    assert delta._MODES == {0: "XOR_RAW", 1: "XOR_GROUP2_ANS", 2: "XOR_ANS", 3: "U16_ANS"}
    with pytest.raises(ValueError, match="policy"):
        DeltaWeights({"x": torch.zeros(1)}, {"x": torch.zeros(1)}, policy="bogus")
