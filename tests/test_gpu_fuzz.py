"""Property test of the GPU encoder and the fused kernel on random residuals.

The same derandomized cases generator as the CPU property test (random sizes,
noise strengths, alphabets, sparse changes, odd tails; every policy and coding):
a package prepared on the GPU and applied by the fused kernel must restore
Teacher1 and Teacher2 bit-exactly, with matching checksums.
"""

from __future__ import annotations

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings

from tests.helpers import FUZZ, as_bytes, random_pair
from warpshift_b200.delta import DeltaWeights

pytestmark = pytest.mark.gpu


@settings(max_examples=150, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(**FUZZ)
def test_random_residuals_round_trip_on_the_gpu(cuda_device, size_class, kind, param, transform, odd, policy, coding,
                                                seed):
    a, b = random_pair(size_class, kind, param, transform, odd, seed)
    gpu = {k: v.to(cuda_device) for k, v in b.items()}
    delta = DeltaWeights(a, gpu, policy=policy, dict_slack_pct=coding[0], escapes=coding[1], split=coding[2])
    try:
        for reverse, expected in ((True, a), (False, b)):
            delta.apply(reverse=reverse)
            assert delta.last_apply["ok"]
            for name, t in gpu.items():
                np.testing.assert_array_equal(as_bytes(t), as_bytes(expected[name]), err_msg=name)
    finally:
        delta.close()
