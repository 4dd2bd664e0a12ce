"""MUL_MAT(Q8_0 W, F32 x) on the GPU through the C ABI against the oracle.

Tolerance: |y_gpu - y_ref| <= 1e-5 * sum_b |dw*dx*isum_b|
per element -- only the fp32 summation order may differ.  The activation codes
and scales themselves are bit-exact (any flipped code would move y by far more
than the bound).
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def check_close(y, y_ref, bound):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    lim = REL_TOL * bound + 1e-30
    bad = err > lim
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst ratio {(err / lim).max():.3g}"


def activations(m, k, seed, outliers=False):
    x = np.asarray(np.random.default_rng(seed).standard_normal((m, k)), np.float32)
    if outliers:  # config 3: 1 % of entries scaled by 20
        mask = np.random.default_rng(seed + 1).random((m, k)) < 0.01
        x[mask] *= 20
    return x


def test_config1_gemv(q8, O, dev):
    d = json.load(open(os.path.join(GOLDEN, "q8_seeded_digests.json")))["config1"]
    w = O.normal(0, 3072 * 1024, 0.02).reshape(3072, 1024)
    x = O.normal(1, 1024).reshape(1, 1024)
    wq = q8.quantize_rows(to_dev(w, dev))
    assert hashlib.sha256(wq.cpu().numpy().tobytes()).hexdigest() == d["w_q8_0_sha256"]
    assert q8.quantize_rows(to_dev(x, dev)).cpu().numpy().tobytes().hex() == d["x_q8_0_hex"]
    y = q8.mul_mat(wq, 1024, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq.cpu().numpy(), 1024, x)
    check_close(y, y_ref, bound)


SHAPES = [(2048, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (1024, 3072), (6144, 2048), (2048, 6144),
          (3072, 2048), (256, 256), (7, 512)]


@pytest.mark.parametrize("path", ["workspace", "no-workspace"])
@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 3, 8])
def test_decode_shapes(q8, O, dev, n, k, m, path):
    # with a workspace, M <= 8 runs on the tensor-core GEMM where the shape allows;
    # without one, on the streaming dp4a GEMV
    w = O.normal(n + k, n * k, 0.02).reshape(n, k)
    wq_np = O.quantize_rows(w)
    x = activations(m, k, seed=n * 7 + k + m)
    ws = None if path == "workspace" else torch.empty(0, dtype=torch.uint8, device=dev)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev), workspace=ws).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("mode", [1, 2])
def test_cpu_activation_modes(q8, O, dev, mode):
    n, k, m = 1024, 3072, 4
    wq_np = O.quantize_rows(O.normal(9, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=mode)
    x[:, ::97] = 2.5 * np.float32(np.abs(x).max() / 127)  # near-ties
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev), mode=mode).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x, mode=mode)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("m", [9, 16, 64])
def test_batched_with_outliers(q8, O, dev, m):
    n, k = 3072, 1024
    wq_np = O.quantize_rows(O.normal(31, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=m, outliers=True)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("n,k", [(1024, 1024), (3072, 1024), (1024, 3072), (2048, 2048), (1000, 2048), (33, 256),
                                 (6144, 2048)])
@pytest.mark.parametrize("m", [16, 20, 64, 256])
def test_tensor_core_gemm(q8, O, dev, n, k, m):
    # M > 8 runs the int8 mma.sync GEMM (config 3 shapes, outliers, ragged N and M)
    wq_np = O.quantize_rows(O.normal(n * 3 + k, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=m * 5 + k, outliers=True)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("n,k,m", [(1024, 1024, 72), (1000, 2048, 130), (3072, 1024, 1024), (256, 8192, 24),
                                   (48, 512, 9), (512, 1024, 4100)])
def test_tensor_core_gemm_token_chunks(q8, O, dev, n, k, m):
    # M > 64 splits tokens into chunks of <= 64 (72 -> 2 x 40, 130 -> 3 x 48); K up to 8192
    wq_np = O.quantize_rows(O.normal(n + 7 * k, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=m + k, outliers=True)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("m", [1, 5, 8])
def test_small_m_large_weight_on_tensor_cores(q8, O, dev, m):
    # M <= 8 with >= 16 MB of weights runs the tensor-core GEMM (one MMA per 16 rows x block)
    n, k = 8192, 2048
    wq_np = O.quantize_rows(O.normal(4242 + m, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=900 + m, outliers=True)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("mode", [1, 2])
def test_tensor_core_gemm_modes(q8, O, dev, mode):
    n, k, m = 3072, 1024, 24
    wq_np = O.quantize_rows(O.normal(77, n * k, 0.02).reshape(n, k))
    x = activations(m, k, seed=mode + 40)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev), mode=mode).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x, mode=mode)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("n,k,m", [(2, 32, 3), (1, 96, 4), (33, 160, 5), (5, 352, 17)])
def test_general_shapes(q8, O, dev, n, k, m):
    wq_np = O.quantize_rows(O.normal(n * k, n * k, 0.5).reshape(n, k))
    x = activations(m, k, seed=k)
    y = q8.mul_mat(to_dev(wq_np, dev), k, to_dev(x, dev)).cpu().numpy()
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(y, y_ref, bound)


@pytest.mark.parametrize("case", json.load(open(os.path.join(GOLDEN, "vits_q8_cases.json")))["cases"],
                         ids=lambda c: c["source"])
def test_vits_conv_q8_cases(q8, O, dev, case):
    k, n, m = case["k"], case["n"], case["m"]
    wq = q8.quantize_rows(to_dev(np.array(case["w_f32"], np.float32).reshape(n, k), dev))
    x = to_dev(np.array(case["x_f32"], np.float32).reshape(m, k), dev)
    y = q8.mul_mat(wq, k, x).cpu().numpy() + np.array(case["bias"], np.float32)[None, :]
    assert np.all(np.abs(y - np.array(case["expected"], np.float32)) < case["bound"])


def test_misaligned_weights_and_strided_io(q8, O, dev):
    n, k, m = 300, 1024, 5
    wq_np = O.quantize_rows(O.normal(8, n * k, 0.02).reshape(n, k))
    raw = torch.zeros(wq_np.size + 2, dtype=torch.uint8, device=dev)
    raw[2:] = to_dev(wq_np.ravel(), dev)
    w_view = raw[2:].view(n, -1)  # 2-byte aligned only: general path
    x = activations(m, k, seed=3)
    xbig = torch.zeros((m, k + 64), dtype=torch.float32, device=dev)
    xbig[:, :k] = to_dev(x, dev)
    ybig = torch.full((m, n + 20), 7.0, dtype=torch.float32, device=dev)
    q8.mul_mat(w_view, k, xbig[:, :k], out=ybig[:, :n])
    y_ref, bound = O.mul_mat(wq_np, k, x)
    check_close(ybig[:, :n].cpu().numpy(), y_ref, bound)
    assert torch.all(ybig[:, n:] == 7.0)
    # fast path with strided activations too
    y2 = q8.mul_mat(to_dev(wq_np, dev), k, xbig[:, :k]).cpu().numpy()
    check_close(y2, y_ref, bound)


def test_errors(q8, dev):
    w = torch.zeros((4, 34), dtype=torch.uint8, device=dev)
    with pytest.raises(q8.B200Q8Error) as e:
        q8.mul_mat(w, 33, torch.zeros((1, 33), device=dev))
    assert e.value.status == 1
    # the general path refuses to run without its workspace
    w2 = torch.zeros((4, 3 * 34), dtype=torch.uint8, device=dev)
    with pytest.raises(q8.B200Q8Error):
        q8.mul_mat(w2, 96, torch.zeros((2, 96), device=dev), workspace=torch.zeros(8, dtype=torch.uint8,
                                                                                    device=dev))
