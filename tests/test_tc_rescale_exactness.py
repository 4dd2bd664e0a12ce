"""The tcgen05 GEMM's rescale (gemm_tc.cu) folds the accumulator bias into the activation scale:
u = fma(v, dx, -1.5 * 2^23 * dx) with v = 1.5 * 2^23 + S read from TMEM.  That equals (v - 1.5 * 2^23) * dx =
S * dx rounded once only if -1.5 * 2^23 * dx is exact in fp32.  dx is always an fp16 value widened to fp32 (the
Q8_0 scale), so the claim is checked here for every finite fp16 value, and for the largest block sums the
int8 codes allow.  CPU only."""
from __future__ import annotations

import numpy as np

BIAS = 12582912.0  # 1.5 * 2^23, the word 0x4B400000 as a float


def test_minus_bias_times_every_fp16_scale_is_exact_in_fp32():
    d = np.arange(1 << 16, dtype=np.uint16).view(np.float16).astype(np.float64)
    d = d[np.isfinite(d)]
    exact = -BIAS * d  # float64 holds the exact product (13 + 24 significant bits at most)
    assert np.array_equal(exact.astype(np.float32).astype(np.float64), exact)


def test_folded_bias_gives_the_single_rounding_of_sum_times_scale():
    # v = BIAS + S is exact for |S| <= 32 * 128 * 128; fma(v, dx, nb) rounds v*dx + nb = S*dx once, so it must
    # equal fp32(S * dx) computed exactly -- checked for extreme and random sums and scales
    rng = np.random.default_rng(7)
    s = np.concatenate([np.array([0, 1, -1, 524288, -524288, 524287, -524287]), rng.integers(-524288, 524289, 4000)])
    d16 = np.concatenate([np.array([65504, -65504, 6.1e-5, 6e-8, 1.0, -2.5], np.float16),
                          rng.standard_normal(4000).astype(np.float16)])
    n = min(len(s), len(d16))
    s, dx = s[:n].astype(np.float64), d16[:n].astype(np.float64)
    v = (BIAS + s).astype(np.float32).astype(np.float64)
    assert np.array_equal(v - BIAS, s)  # the bias word holds every block sum exactly
    nb = (-BIAS * dx).astype(np.float32).astype(np.float64)  # exact (previous test)
    fused = (v * dx + nb).astype(np.float32)  # v*dx + nb is exact in float64 here: a single final rounding
    assert np.array_equal(fused, (s * dx).astype(np.float32))
