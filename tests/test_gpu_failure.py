"""Failure detection on the GPU without a fault: a bounded staging-barrier wait
that can never complete gives up, reports WS_DEVERR_TIMEOUT through the result
word, and the context stays usable for a normal switch afterwards."""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from tests.helpers import as_bytes, bf16_pair
from warpshift_b200 import _lib
from warpshift_b200.delta import DeltaWeights

pytestmark = pytest.mark.gpu

WS_DEVERR_TIMEOUT = 4


@pytest.mark.parametrize("polls", [1, 1000, 20000])
def test_bounded_wait_gives_up_and_reports(cuda_device, polls: int) -> None:
    lib = _lib.load()
    errors = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    t0 = time.perf_counter()
    _lib.check(lib.ws_selftest_wait_timeout(polls, cuda_device.index or 0, stream, ctypes.byref(errors)))
    assert errors.value == WS_DEVERR_TIMEOUT
    assert time.perf_counter() - t0 < 30
    # The context is still healthy: a real switch round trip works.
    x, y = bf16_pair(1 << 20, 0.01, 3)
    gpu = {"w": y.to(cuda_device)}
    delta = DeltaWeights({"w": x}, gpu)
    delta.apply(reverse=True)
    np.testing.assert_array_equal(as_bytes(gpu["w"]), as_bytes(x))
    delta.apply(reverse=False)
    np.testing.assert_array_equal(as_bytes(gpu["w"]), as_bytes(y))
