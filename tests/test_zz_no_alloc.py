"""b200q8_mul_mat_noalloc, the MUL_MAT entry point for callers that cannot
allocate device memory (a ggml backend mid-graph, a real-time streaming
callback that must not block on cudaMalloc).  It keeps its scratch in a fixed 1 MiB
device array inside the library instead of a caller workspace.

Checked through the C ABI against the existing entry point b200q8_mul_mat on
two calls in a row (the array keeps the first call's contents when the second
runs), within the tests' tolerance of 1e-5 of the per-element abs-sum bound.
This file is collected last on purpose; it needs nothing from the others.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5


def noalloc(lib, w, k, x, mode=0):
    m, n = x.shape[0], w.shape[0]
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device=x.device)
    st = lib.b200q8_mul_mat_noalloc(w.data_ptr(), k, n, w.stride(0), x.data_ptr(), m, x.stride(0) * 4,
                                    y.data_ptr(), y.stride(0) * 4, mode, torch.cuda.current_stream().cuda_stream)
    return st, y


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_mul_mat_on_two_calls(pkg, q8, O, dev, mode):
    from synthesize_cpp_b200 import _abi

    lib = _abi.lib()
    cases = [(1024, 768, 5, 11), (96, 33, 17, 12)]  # (K, N, M, seed): streaming-size and a general shape
    results = []
    for k, n, m, seed in cases:
        w_np = O.quantize_rows(O.normal(seed, n * k, 0.05).reshape(n, k))
        x_np = np.asarray(np.random.default_rng(seed).standard_normal((m, k)), np.float32)
        w = torch.from_numpy(w_np).to(dev)
        x = torch.from_numpy(x_np).to(dev)
        st, y = noalloc(lib, w, k, x, mode)
        assert st == 0, _abi.last_error()
        results.append((w, x, y, w_np, x_np, k))
    torch.cuda.synchronize()
    for w, x, y, w_np, x_np, k in results:
        ref_entry = q8.mul_mat(w, k, x, mode=mode).cpu().numpy()
        _, bound = O.mul_mat(w_np, k, x_np, mode=mode)
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got.astype(np.float64) - ref_entry) <= REL_TOL * bound + 1e-30)


def test_noalloc_rejects_sizes_beyond_its_array(pkg, dev):
    from synthesize_cpp_b200 import _abi

    lib = _abi.lib()
    k, m, n = 8192, 128, 4  # 128 * 256 * 34 = 1,114,112 bytes > 1 MiB
    w = torch.zeros((n, k // 32 * 34), dtype=torch.uint8, device=dev)
    x = torch.zeros((m, k), dtype=torch.float32, device=dev)
    st, _ = noalloc(lib, w, k, x)
    assert st == _abi.ERR_INVALID_ARG
    assert "static maximum" in _abi.last_error()[1]
