"""Large-M MUL_MAT on the tcgen05 tensor cores (gemm_tc.cu) through the C ABI, against the oracle.

The tcgen05 GEMM is off by default (the mma.sync GEMM measured faster); B200Q8_TC_MIN_M=<M> turns it on from
that M, read once per process.  test_tcgen05_gemm_cases therefore runs this file again in a fresh process with
B200Q8_TC_MIN_M=1024, where the cases below run: b200q8_mul_mat then sends M >= 1024 to the tcgen05 GEMM when
the workspace holds its planes (the size b200q8_mul_mat_workspace_size returns), and with one byte less the
same call runs the mma.sync GEMM.  Both are checked against the oracle at north_star's bound
|y - y_ref| <= 1e-5 * sum_b |dw*dx*isum_b|: ragged N and M (partial 128-row and 128-token tiles), K from one
256-wide chunk to 24, outliers, all three activation modes, strided activations and outputs, repeatability.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from test_gpu_mul_mat import activations, check_close, to_dev

pytestmark = pytest.mark.gpu

TC_MIN_M = 1024
TC_ON = os.environ.get("B200Q8_TC_MIN_M", "") == str(TC_MIN_M)
inner = pytest.mark.skipif(not TC_ON, reason="runs in the fresh process that test_tcgen05_gemm_cases starts")


@pytest.mark.skipif(TC_ON, reason="this is the inner process")
def test_tcgen05_gemm_cases():
    env = dict(os.environ, B200Q8_TC_MIN_M=str(TC_MIN_M))
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "-m", "gpu",
                        os.path.abspath(__file__)], env=env, cwd=os.path.dirname(os.path.dirname(__file__)),
                       capture_output=True, text=True, timeout=900)
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, tail
    assert " passed" in tail and "skipped" in tail, tail


def run(q8, wq, k, x, mode=0, out=None, short=False):
    m, n = x.shape[0], wq.shape[0]
    need = q8.workspace_size(k, n, m)
    ws = torch.empty(need - 1 if short else need, dtype=torch.uint8, device=x.device)
    return q8.mul_mat(wq, k, x, mode=mode, out=out, workspace=ws)


@inner
@pytest.mark.parametrize("n,k,m", [(3072, 1024, 1024), (1024, 3072, 1280), (1000, 2048, 1100), (33, 256, 1024),
                                   (2048, 1024, 2048), (130, 768, 1029), (6144, 2048, 1024)])
def test_tc_gemm_against_oracle(q8, O, dev, n, k, m):
    wq_np = O.quantize_rows(O.normal(n * 5 + k, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=m * 3 + k, outliers=True)
    wq, xd = to_dev(wq_np, dev), to_dev(x, dev)
    # the tcgen05 planes are part of the workspace the size query asks for
    assert q8.workspace_size(k, n, m) >= n * k + m * k
    y_ref, bound = O.mul_mat(wq_np, k, x)
    y_tc = run(q8, wq, k, xd).cpu().numpy()
    check_close(y_tc, y_ref, bound)
    # one byte short of the planes: the mma.sync GEMM, same bound
    y_mma = run(q8, wq, k, xd, short=True).cpu().numpy()
    check_close(y_mma, y_ref, bound)
    assert q8.device_status(0) == 0


@inner
@pytest.mark.parametrize("mode", [1, 2])
def test_tc_gemm_modes(q8, O, dev, mode):
    n, k, m = 1024, 1024, TC_MIN_M + 40
    wq_np = O.quantize_rows(O.normal(500 + mode, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=mode + 70)
    x[:, ::97] = 2.5 * np.float32(np.abs(x).max() / 127)  # near-ties in the quantizer
    y = run(q8, to_dev(wq_np, dev), k, to_dev(x, dev), mode=mode).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x, mode=mode)
    check_close(y, y_ref, bound)


@inner
def test_tc_gemm_strided_io(q8, O, dev):
    n, k, m = 520, 512, TC_MIN_M + 3
    wq_np = O.quantize_rows(O.normal(61, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=62, outliers=True)
    xbig = torch.zeros((m, k + 36), dtype=torch.float32, device=dev)  # row stride 548 floats (16-byte multiple)
    xbig[:, :k] = to_dev(x, dev)
    ybig = torch.full((m, n + 9), 7.0, dtype=torch.float32, device=dev)
    run(q8, to_dev(wq_np, dev), k, xbig[:, :k], out=ybig[:, :n])
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(ybig[:, :n].cpu().numpy(), y_ref, bound)
    assert torch.all(ybig[:, n:] == 7.0)


@inner
def test_tc_gemm_repeatable(q8, O, dev):
    # the same inputs give the same bits (fixed block order, no atomics)
    n, k, m = 2048, 2048, 1536
    wq = to_dev(O.quantize_rows(O.normal(91, n * k, 0.02).reshape(n, k)), dev)
    xd = to_dev(activations(m, k, seed=92), dev)
    a = run(q8, wq, k, xd)
    b = run(q8, wq, k, xd)
    assert torch.equal(a, b)
