"""Property test of the host encoder against the oracle's C decoder, on CPU.

Seeded random tensors of random sizes and residual statistics (relative noise of
any strength, small skewed alphabets, sparse changes, odd byte counts) under
every policy and coding: decoding the plan with oracle/stream_oracle.c must
restore Teacher1 and Teacher2 bit-exactly, with the checksums the encoder
recorded. Hypothesis runs derandomized, so the cases are fixed.
"""

from __future__ import annotations

import numpy as np
from hypothesis import HealthCheck, given, settings

from oracle import stream as ostream
from tests.helpers import FUZZ, as_bytes, host_plan, plan_arrays, random_pair
from warpshift_b200 import _lib


@settings(max_examples=150, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(**FUZZ)
def test_random_residuals_round_trip_through_the_oracle_decoder(size_class, kind, param, transform, odd, policy, coding, seed):
    a, b = random_pair(size_class, kind, param, transform, odd, seed)
    work = {k: v.clone() for k, v in b.items()}
    plan = host_plan(a, work, policy, *coding)
    try:
        blocks, tiles, tables, arena, stats = plan_arrays(plan)
        for reverse, teacher in ((True, a), (False, b)):
            err, checksum = ostream.apply_plan(blocks, tiles, tables, arena, 0, reverse, 2)
            assert err == 0
            assert checksum == stats.expected_checksum[1 if reverse else 0]
            for name in b:
                np.testing.assert_array_equal(as_bytes(work[name]), as_bytes(teacher[name]), err_msg=name)
    finally:
        _lib.load().ws_plan_destroy(plan)
