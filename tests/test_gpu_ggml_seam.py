"""The ggml-backend seam (include/b200q8_ggml.h) on the GPU: nodes described
as ggml tensors, batched dims with ggml's broadcast rule, computed through
libb200q8_host.so -> libb200q8.so and checked against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_mul_mat_node_with_broadcast(pkg, O, dev):
    from synthesize_cpp_b200 import ggml_seam as G

    K, N, M, W2, X2 = 1024, 256, 3, 2, 4  # src0 ne2 = 2 broadcast over src1 ne2 = 4
    mats = [O.quantize_rows(O.normal(60 + i, N * K, 0.02).reshape(N, K)) for i in range(W2)]
    w = torch.from_numpy(np.stack(mats)).to(dev)                     # [2, N, K/32*34]
    xs = [np.asarray(np.random.default_rng(i).standard_normal((M, K)), np.float32) for i in range(X2)]
    x = torch.from_numpy(np.stack(xs)).to(dev)                       # [4, M, K]
    y = torch.zeros((X2, M, N), dtype=torch.float32, device=dev)
    tw, tx = G.q8_tensor(w, K), G.dense_tensor(x, G.TYPE_F32)
    ty = G.dense_tensor(y, G.TYPE_F32)
    ty.op = G.OP_MUL_MAT
    ty.src[0] = __import__("ctypes").pointer(tw)
    ty.src[1] = __import__("ctypes").pointer(tx)
    assert G.supports_op(ty)
    G.compute(ty)
    got = y.cpu().numpy()
    for i in range(X2):
        ref, bound = O.mul_mat(mats[i // (X2 // W2)], K, xs[i])
        assert np.all(np.abs(got[i].astype(np.float64) - ref) <= 1e-5 * bound + 1e-30)


def test_get_rows_node_batched(pkg, O, dev):
    import ctypes

    from synthesize_cpp_b200 import ggml_seam as G

    K, R, B = 1024, 64, 2
    tabs = [O.quantize_rows(O.normal(80 + i, R * K, 0.02).reshape(R, K)) for i in range(B)]
    t = torch.from_numpy(np.stack(tabs)).to(dev)                     # [B, R, K/32*34]
    ids_np = np.array([[3, 0, 63], [7, 7, 1]], dtype=np.int32)       # [B, 3]
    ids = torch.from_numpy(ids_np).to(dev)
    out = torch.zeros((B, 3, K), dtype=torch.float32, device=dev)
    tt, ti = G.q8_tensor(t, K), G.dense_tensor(ids, G.TYPE_I32)
    to = G.dense_tensor(out, G.TYPE_F32)
    to.op = G.OP_GET_ROWS
    to.src[0] = ctypes.pointer(tt)
    to.src[1] = ctypes.pointer(ti)
    assert G.supports_op(to)
    G.compute(to)
    got = out.cpu().numpy()
    for b in range(B):
        ref, st = O.get_rows(tabs[b], K, ids_np[b])
        assert st == 0 and np.array_equal(got[b], ref)
