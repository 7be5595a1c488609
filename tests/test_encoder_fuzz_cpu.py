"""Property test of the host encoder against the oracle's C decoder, on CPU.

Seeded random tensors of random sizes and residual statistics (relative noise of
any strength, small skewed alphabets, sparse changes, odd byte counts) under
every policy and coding: decoding the plan with oracle/stream_oracle.c must
restore Teacher1 and Teacher2 bit-exactly, with the checksums the encoder
recorded. Hypothesis runs derandomized, so the cases are fixed.
"""

from __future__ import annotations

import numpy as np
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import stream as ostream
from tests.helpers import as_bytes, bf16_pair, host_plan, plan_arrays
from warpshift_b200 import _lib

CODINGS = [(-1, -1), (6, 0), (100, -1), (100, 1)]  # (dict_slack_pct, escapes)


def residual_words(kind: str, n: int, param: float, rng: np.random.Generator) -> np.ndarray | None:
    """None: use a bf16 relative-noise pair with strength ``param``."""
    if kind == "noise":
        return None
    if kind == "alphabet":
        size = 1 + int(param * 400)
        values = rng.integers(0, 65536, size).astype(np.uint32)
        p = rng.dirichlet(np.full(size, 0.3))
        return values[rng.choice(size, n, p=p)]
    r = np.zeros(n, np.uint32)  # sparse: a fraction param / 10 of the words change
    hit = rng.random(n) < param / 10
    r[hit] = rng.integers(1, 65536, int(hit.sum()))
    return r


@settings(max_examples=150, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
@given(
    size_class=st.sampled_from([(1, 8191), (8191, 8193), (8192, 32768), (32769, 300_000)]),  # words
    kind=st.sampled_from(["noise", "alphabet", "sparse"]),
    param=st.sampled_from([0.0, 0.001, 0.01, 0.03, 0.1, 0.3]),
    transform=st.sampled_from(["xor", "u16"]),
    odd=st.booleans(),
    policy=st.sampled_from(["auto", "xor", "u16"]),
    coding=st.sampled_from(CODINGS),
    seed=st.integers(0, 2**31 - 1),
)
def test_random_residuals_round_trip_through_the_oracle_decoder(size_class, kind, param, transform, odd, policy, coding, seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(size_class[0], size_class[1] + 1))
    r = residual_words(kind, n, param, rng)
    if r is None:
        a_t, b_t = bf16_pair(n, param, seed)
    else:
        a_t, _ = bf16_pair(n, 0.0, seed)
        w = a_t.view(torch.int16).numpy().view(np.uint16).astype(np.uint32)
        t = (w ^ r) if transform == "xor" else (w + r) & 0xFFFF
        b_t = torch.from_numpy(t.astype(np.uint16).view(np.int16)).view(torch.bfloat16)
    a = {"w": a_t}
    b = {"w": b_t.clone()}
    if odd:  # the same bytes as a uint8 tensor of odd length: XOR only
        nb = 2 * n - 1
        a["u"] = a_t.view(torch.uint8)[:nb].clone()
        b["u"] = b_t.view(torch.uint8)[:nb].clone()
    work = {k: v.clone() for k, v in b.items()}
    plan = host_plan(a, work, policy, dict_slack_pct=coding[0], escapes=coding[1])
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
