"""The step with the reference's attention (b200q8_chain_run_at): q/k head RMS norms, NEOX RoPE, the F32 KV cache
and softmax attention over the cached prefix (src/arch/qwen3-tts/operations.cpp:86-135), against the oracle.

Per step, the attention output is checked against the oracle's attention computed from the GPU's own q, k, v (its
projections read back), with the oracle keeping its own cache of those rotated keys and values: that isolates the
attention kernels (fp32 vs the oracle's fp64 sums, CUDA's cosf/sinf/powf vs libm's).  The whole step is compared
with the oracle's attention chain, where quantization code flips -- carried from step to step by each side's
own cache -- make it a relative-L2 check."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_chain import H, HD, I, NH, NKV, EPS, make_model, upload

pytestmark = pytest.mark.gpu

Q, KV = NH * HD, NKV * HD
THETA = 1.0e6


def qk_norms(O, n_layers, seed=900):
    return np.stack([(1.0 + 0.2 * O.normal(seed + i, HD)).astype(np.float32) for i in range(2 * n_layers)])


def build(O, chain_mod, dev, n_layers, max_m, n_ctx, n_slots, seed):
    mats, norms, table = make_model(O, n_layers, seed=seed)
    qkn = qk_norms(O, n_layers, seed + 50)
    layers, t_table = upload(mats, norms, table, dev)
    for l, L in enumerate(layers):
        L["q_norm"] = torch.from_numpy(qkn[2 * l]).to(dev)
        L["k_norm"] = torch.from_numpy(qkn[2 * l + 1]).to(dev)
    ch = chain_mod.DecodeChain(layers, t_table, hidden=H, n_head=NH, n_kv=NKV, head_dim=HD, inter=I, eps=EPS,
                               max_m=max_m, attention=dict(rope_theta=THETA, n_ctx=n_ctx, n_slots=n_slots))
    return ch, mats, norms, table, qkn


def attention_ref(O, qkv, qkn_l, caches, pos):
    """Oracle attention for the tokens of one step from the GPU's own q|k|v rows; caches[m] = (kc, vc) lists."""
    out = np.empty((qkv.shape[0], Q), np.float32)
    for m in range(qkv.shape[0]):
        q = O.head_norm_rope(qkv[m, :Q], HD, qkn_l[0], EPS, int(pos[m]), THETA)
        k = O.head_norm_rope(qkv[m, Q:Q + KV], HD, qkn_l[1], EPS, int(pos[m]), THETA)
        v = qkv[m, Q + KV:].copy()
        kc, vc = caches[m]
        kc[int(pos[m])] = k
        vc[int(pos[m])] = v
        out[m] = O.attend(q, kc, vc, int(pos[m]) + 1, NH, NKV, HD)
    return out


def run_steps(O, chain_mod, dev, m, steps, n_layers=2, seed=1200, check_every=1, start=None):
    n_ctx = (max(start) if start is not None else 0) + steps + 1
    ch, mats, norms, table, qkn = build(O, chain_mod, dev, n_layers, max(8, m), n_ctx, m, seed)
    rng = np.random.default_rng(seed)
    k_ref = np.zeros((n_layers, m, n_ctx, KV), np.float32)
    v_ref = np.zeros_like(k_ref)
    gpu_caches = [[(np.zeros((n_ctx, KV), np.float32), np.zeros((n_ctx, KV), np.float32)) for _ in range(m)]
                  for _ in range(n_layers)]
    base = np.zeros(m, np.int32) if start is None else np.asarray(start, np.int32)
    h = torch.empty((m, H), device=dev)
    worst = 0.0
    for t in range(steps):
        pos = base + t
        x = rng.standard_normal((m, H)).astype(np.float32)
        ids = rng.integers(0, 64, m).astype(np.int32)
        ch.run_at(torch.from_numpy(ids).to(dev), torch.from_numpy(x).to(dev), torch.from_numpy(pos).to(dev), h)
        torch.cuda.synchronize(dev)
        for l in range(n_layers):
            qkv = ch.buffer(l, "qkv", m).cpu().numpy()[:, :Q + 2 * KV]
            att = ch.buffer(l, "attn", m).cpu().numpy()[:, :Q]
            ref = attention_ref(O, qkv, qkn[2 * l:2 * l + 2], gpu_caches[l], pos)
            err = np.abs(att - ref).max() / (np.abs(ref).max() + 1e-30)
            worst = max(worst, err)
            assert err < 2e-5, (t, l, err)
        want = O.decoder_chain_attn(mats, norms, qkn, table, ids, x, pos, k_ref, v_ref, hidden=H, n_head=NH,
                                    n_kv=NKV, head_dim=HD, inter=I, eps=EPS, theta=THETA)
        got = h.cpu().numpy()
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        cos = float(np.sum(got * want) / (np.linalg.norm(got) * np.linalg.norm(want)))
        # each side's cache carries its own quantization-code flips forward from step to step, so the
        # whole-step bound is looser than the single-step chain's (2e-3); the per-op checks above are tight
        assert rel < 1e-2 and cos > 0.9999, (t, rel, cos)
    ch.close()
    return worst


def test_single_stream_decode_over_positions(pkg, O, chain_mod, dev):
    run_steps(O, chain_mod, dev, m=1, steps=24)


def test_two_streams_at_different_positions(pkg, O, chain_mod, dev):
    run_steps(O, chain_mod, dev, m=2, steps=8, start=[0, 37])


def test_batched_path_with_attention(pkg, O, chain_mod, dev):
    # M > 8: stage + tensor-core GEMM per op, attention kernels between qkv and o
    run_steps(O, chain_mod, dev, m=12, steps=5, start=list(range(0, 60, 5)))


def test_explicit_slots_and_bad_positions(pkg, O, chain_mod, dev):
    from synthesize_cpp_b200 import q8

    ch, *_ = build(O, chain_mod, dev, 1, 8, 16, 4, seed=1400)
    x = torch.randn((2, H), device=dev)
    ids = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    h = torch.empty((2, H), device=dev)
    ch.run_at(ids, x, torch.tensor([0, 0], dtype=torch.int32, device=dev), h,
              slots=torch.tensor([3, 1], dtype=torch.int32, device=dev))
    assert q8.device_status(dev.index or 0) == 0
    ch.run_at(ids, x, torch.tensor([0, 16], dtype=torch.int32, device=dev), h,
              slots=torch.tensor([3, 1], dtype=torch.int32, device=dev))  # position 16 is outside n_ctx = 16
    assert q8.device_status(dev.index or 0, clear=True) == 1
    ch.run_at(ids, x, torch.tensor([0, 0], dtype=torch.int32, device=dev), h,
              slots=torch.tensor([3, 4], dtype=torch.int32, device=dev))  # slot 4 is outside n_slots = 4
    assert q8.device_status(dev.index or 0, clear=True) == 1
    ch.close()
