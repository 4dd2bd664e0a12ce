"""b200q8_mul_mat_noalloc, the MUL_MAT entry point for callers that cannot
allocate device memory (a ggml backend mid-graph, a real-time streaming
callback that must not block on cudaMalloc).  It keeps its scratch in a fixed 1 MiB
device array inside the library instead of a caller workspace.

Checked through the C ABI, on calls made back to back (the array keeps each
call's contents when the next one runs), against the oracle's MUL_MAT and
against the existing entry point b200q8_mul_mat, within the tests' tolerance
of 1e-5 of the per-element abs-sum bound.  The sequence covers each path the
entry point can take (tensor-core GEMM with its records in the array, the
scratch-free streaming GEMV, the general kernel on activations quantized into
the array), a call whose footprint nearly fills the array, and calls whose
footprint only partly overwrites what the previous call left.
This file is collected last on purpose; it needs nothing from the others.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5
LIMIT = 1 << 20

# (K, N, M, seed), run back to back in this order
CALLS = [
    (1024, 768, 5, 11),      # tensor-core GEMM, records in the array
    (96, 33, 17, 12),        # general kernel, 1,734 B of quantized activations: a small part of the array
    (1024, 3072, 1, 13),     # the talker's gate shape at M = 1 (GEMM)
    (96, 33, 10280, 14),     # general kernel at 1,048,560 B, the largest M whose footprint fits
    (1024, 64, 963, 15),     # 1,047,744 B: the GEMM's records would not fit, so the scratch-free GEMV runs
    (160, 40, 9, 16),        # general kernel again, over what the near-limit call left
]


def noalloc(lib, w, k, x, mode=0):
    m, n = x.shape[0], w.shape[0]
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=x.device)
    st = lib.b200q8_mul_mat_noalloc(w.data_ptr(), k, n, w.stride(0), x.data_ptr(), m, x.stride(0) * 4,
                                    y.data_ptr(), y.stride(0) * 4, mode, torch.cuda.current_stream().cuda_stream)
    return st, y


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_noalloc_matches_oracle_and_mul_mat_on_calls_in_a_row(pkg, q8, O, dev, mode):
    from synthesize_cpp_b200 import _abi

    lib = _abi.lib()
    results = []
    for k, n, m, seed in CALLS:
        assert m * (k // 32) * 34 <= LIMIT
        w_np = O.quantize_rows(O.normal(seed, n * k, 0.05).reshape(n, k))
        x_np = np.asarray(np.random.default_rng(seed).standard_normal((m, k)), np.float32)
        w = torch.from_numpy(w_np).to(dev)
        x = torch.from_numpy(x_np).to(dev)
        st, y = noalloc(lib, w, k, x, mode)
        assert st == 0, _abi.last_error()
        results.append((w, x, y, w_np, x_np, k))
    torch.cuda.synchronize()
    assert q8.device_status(0) == 0
    for w, x, y, w_np, x_np, k in results:
        got = y.cpu().numpy().astype(np.float64)
        y_ref, bound = O.mul_mat(w_np, k, x_np, mode=mode)
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - y_ref) <= REL_TOL * bound + 1e-30), (k, x_np.shape[0])
        entry = q8.mul_mat(w, k, x, mode=mode).cpu().numpy()
        assert np.all(np.abs(got - entry) <= 2 * REL_TOL * bound + 1e-30), (k, x_np.shape[0])


def test_noalloc_rejects_sizes_beyond_its_array(pkg, dev):
    from synthesize_cpp_b200 import _abi

    lib = _abi.lib()
    for k, m in ((8192, 128), (1024, 964), (96, 10281)):  # one past the limit at each K
        assert m * (k // 32) * 34 > LIMIT
        w = torch.zeros((4, k // 32 * 34), dtype=torch.uint8, device=dev)
        x = torch.zeros((m, k), dtype=torch.float32, device=dev)
        st, _ = noalloc(lib, w, k, x)
        assert st == _abi.ERR_INVALID_ARG
        assert "static maximum" in _abi.last_error()[1]
