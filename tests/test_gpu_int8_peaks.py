"""The int8 measurement library (peaks/int8_peaks.cu, libb200q8_peaks.so) on the GPU.

The tcgen05 kind::i8 MMA the ceilings are timed with must compute the right thing: one M = 128, N = 256,
K = 32 MMA on known operands (A[r][k] = r % 7 - 3, B[n][k] = (n + 2k) % 5 - 2) is read back from TMEM and
must equal the exact int32 products.  The one-CTA latency probe must finish without a timed-out wait and
report plausible cycle counts (a back-to-back 128 x 128 x 32 MMA cannot beat the B200's nominal int8 rate
of about 15.5 k int8 ops per SM cycle, i.e. 68 cycles, by more than the clock-rounding margin).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def peaks(pkg):
    import torch

    from synthesize_cpp_b200 import build

    torch.cuda.init()
    L = ctypes.CDLL(build.PEAKS_LIB)
    L.b200q8p_tcgen05_check.argtypes = [ctypes.c_void_p]
    L.b200q8p_tcgen05_latency.argtypes = [ctypes.c_void_p]
    return L


def test_tcgen05_i8_mma_equals_exact_products(peaks):
    out = np.full((128, 256), -1, np.int32)
    assert peaks.b200q8p_tcgen05_check(out.ctypes.data) == 0
    a = (np.arange(128)[:, None] % 7 - 3) * np.ones((1, 32), np.int64)
    b = (np.arange(256)[:, None] + 2 * np.arange(32)[None, :]) % 5 - 2
    assert np.array_equal(out, (a @ b.T).astype(np.int32))


def test_tcgen05_latency_probe(peaks):
    lat = np.zeros(6, np.int64)
    assert peaks.b200q8p_tcgen05_latency(lat.ctypes.data) == 0
    ld_best, ld_mean, st_best, st_mean, mma1, mma32 = (int(v) for v in lat)
    assert 0 < ld_best <= ld_mean < 100000 and 0 < st_best <= st_mean < 100000
    assert 0 < mma1 < mma32 < 10_000_000
    assert (mma32 - mma1) / 31 >= 60  # 128 * 128 * 32 * 2 ops at <= ~15.5 k ops per cycle per SM
