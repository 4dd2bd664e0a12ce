"""The step's output stage (b200q8_chain_step: final RMS norm + Q8_0 head) and the device-side decode frame
(b200q8_frame_run: talker step, greedy or replayed selection, the code predictor's prefill and steps) against the
oracle (src/arch/qwen3-tts/model.cpp:1310-1489, talker.cpp:135-185, code-predictor.cpp:34-80,
code-predictor-host.cpp:15-80).

The output stage is checked on the GPU's own residual stream: the norm bit-exact, the head within 1e-5 of its
abs-sum bound.  A frame is checked with the oracle replaying the GPU's codes (so both follow one path): every
greedy choice must be the oracle's argmax, or within a near-tie margin of it, since the two sides' logits differ
by the quantization-code flips the attention chain carries (relative L2 ~1e-3).  The selection rule itself (ties,
NaN, -inf, the repetition penalty) is checked bit-exactly through skip_talker, where the logits are inputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_chain import EPS, HD, H, I, KV, NH, NKV, Q, make_model, rms_norm, upload
from test_gpu_attention import THETA, qk_norms

pytestmark = pytest.mark.gpu

G = 4          # code groups per frame in these tests (16 in the 0.6B package)
TV = 384       # talker codec vocab / table rows
PV = 256       # predictor vocab / table rows


def stack(O, dev, n_layers, seed, vocab, n_heads, table_rows, chain_mod, *, n_ctx, n_slots, max_m):
    """A decoder stack with attention and an output desc: (DecodeChain, oracle dict)."""
    mats, norms, _ = make_model(O, n_layers, seed=seed)
    qkn = qk_norms(O, n_layers, seed + 50)
    table = O.quantize_rows(O.normal(seed + 70, table_rows * H, 0.5).reshape(table_rows, H))
    out_norm = (1.0 + 0.1 * O.normal(seed + 71, H)).astype(np.float32)
    heads = [O.quantize_rows(O.normal(seed + 80 + i, vocab * H, 0.02).reshape(vocab, H)) for i in range(n_heads)]
    layers, t_table = upload(mats, norms, table, dev)
    for l, L in enumerate(layers):
        L["q_norm"] = torch.from_numpy(qkn[2 * l]).to(dev)
        L["k_norm"] = torch.from_numpy(qkn[2 * l + 1]).to(dev)
    t_heads = [torch.from_numpy(h).to(dev) for h in heads]
    ch = chain_mod.DecodeChain(layers, t_table, hidden=H, n_head=NH, n_kv=NKV, head_dim=HD, inter=I, eps=EPS,
                               max_m=max_m, attention=dict(rope_theta=THETA, n_ctx=n_ctx, n_slots=n_slots),
                               output=dict(norm=torch.from_numpy(out_norm).to(dev), heads=t_heads))
    ref = dict(mats=mats, norms=norms, qkn=qkn, table=table, out_norm=out_norm, heads=heads, hidden=H, n_head=NH,
               n_kv=NKV, head_dim=HD, inter=I, eps=EPS, theta=THETA, vocab=vocab)
    return ch, ref


def t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("m", [1, 3, 12])
def test_step_output_stage(chain_mod, O, dev, m):
    ch, ref = stack(O, dev, 2, 3000, 512, 2, 64, chain_mod, n_ctx=4, n_slots=m, max_m=16)
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, H)).astype(np.float32)
    ids = rng.integers(0, 64, m).astype(np.int32)
    pos = np.zeros(m, np.int32)
    h = torch.empty((m, H), device=dev)
    hid = torch.empty((m, H), device=dev)
    lg = torch.empty((m, 512), device=dev)
    for head in (1, 0):
        ch.step(ids=t(ids, dev), x_in=t(x, dev), pos=t(pos + (1 - head), dev), h_out=h, hidden_out=hid, logits=lg,
                head=head)
        torch.cuda.synchronize(dev)
        hg, hidg, lgg = h.cpu().numpy(), hid.cpu().numpy(), lg.cpu().numpy()
        assert np.array_equal(hidg, rms_norm(hg, ref["out_norm"])), "final norm not bit-exact"
        y_ref, bound = O.mul_mat(ref["heads"][head], H, hidg)
        assert np.all(np.abs(lgg.astype(np.float64) - y_ref) <= 1e-5 * bound + 1e-30)
    # the residual stream matches the oracle's attention chain (two positions of one slot each)
    kc = np.zeros((2, m, 4, KV), np.float32)
    vc = np.zeros_like(kc)
    for p in (0, 1):
        want = O.decoder_chain_attn(ref["mats"], ref["norms"], ref["qkn"], ref["table"], ids, x,
                                    np.full(m, p, np.int32), kc, vc, hidden=H, n_head=NH, n_kv=NKV, head_dim=HD,
                                    inter=I, eps=EPS, theta=THETA)
    rel = np.linalg.norm(hg - want) / np.linalg.norm(want)
    assert rel < 1e-2, rel


def test_step_inputs_are_interchangeable(chain_mod, O, dev):
    """ids-only, x_in-only and table-override steps agree bit-for-bit with the equivalent explicit input."""
    m = 4
    ch, ref = stack(O, dev, 1, 3100, 256, 1, 64, chain_mod, n_ctx=2, n_slots=4 * m, max_m=8)
    rng = np.random.default_rng(7)
    ids = rng.integers(0, 64, m).astype(np.int32)
    other = O.quantize_rows(O.normal(3199, 32 * H, 0.5).reshape(32, H))
    ids2 = rng.integers(0, 32, m).astype(np.int32)
    pos = t(np.zeros(m, np.int32), dev)
    outs = []
    cases = [dict(ids=t(ids, dev)),
             dict(x_in=t(O.get_rows(ref["table"], H, ids)[0], dev)),
             dict(ids=t(ids2, dev), table=t(other, dev)),
             dict(x_in=t(O.get_rows(other, H, ids2)[0], dev))]
    for i, kw in enumerate(cases):
        h = torch.empty((m, H), device=dev)
        lg = torch.empty((m, 256), device=dev)
        ch.step(pos=pos, slots=t(np.arange(m, dtype=np.int32) + i * m, dev), h_out=h, logits=lg, m=m, **kw)
        outs.append((h, lg))
    torch.cuda.synchronize(dev)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[2][0], outs[3][0]) and torch.equal(outs[2][1], outs[3][1])
    assert not torch.equal(outs[0][0], outs[2][0])


def make_frame(O, dev, chain_mod, frame_mod, *, m, penalty=1.0, t_layers=2, p_layers=2):
    talker, tref = stack(O, dev, t_layers, 4000, TV, 1, TV, chain_mod, n_ctx=16, n_slots=m, max_m=max(8, m))
    pred, pref = stack(O, dev, p_layers, 5000, PV, G - 1, 8, chain_mod, n_ctx=G, n_slots=m, max_m=max(8, 2 * m))
    ptables = [O.quantize_rows(O.normal(6000 + g, PV * H, 0.5).reshape(PV, H)) for g in range(G - 1)]
    fr = frame_mod.Frame(talker, pred, [t(p, dev) for p in ptables], repetition_penalty=penalty)
    n_ctx_t = 16
    state = dict(tk=np.zeros((t_layers, m, n_ctx_t, KV), np.float32), tv=np.zeros((t_layers, m, n_ctx_t, KV), np.float32),
                 pk=np.zeros((p_layers, m, G, KV), np.float32), pv=np.zeros((p_layers, m, G, KV), np.float32),
                 history={})
    return fr, talker, tref, pref, ptables, state


def assert_choice(code, logits, margin):
    """code is the argmax of logits, or within `margin` of its value (a near-tie the two sides may split)."""
    best = int(np.argmax(logits))
    assert code == best or logits[best] - logits[code] <= margin, (code, best, logits[best] - logits[code])


@pytest.mark.parametrize("m,penalty", [(1, 1.0), (3, 1.0), (2, 1.5)])
def test_frame_greedy_against_oracle(chain_mod, frame_mod, O, dev, m, penalty):
    fr, _, tref, pref, ptables, state = make_frame(O, dev, chain_mod, frame_mod, m=m, penalty=penalty)
    rng = np.random.default_rng(11 + m)
    slots = np.arange(m, dtype=np.int32)[::-1].copy()
    prev = np.stack([rng.integers(0, TV, m)] + [rng.integers(0, PV, m) for _ in range(G - 1)], 1).astype(np.int32)
    codes = torch.empty((m, G), dtype=torch.int32, device=dev)
    hid = torch.empty((m, H), device=dev)
    tlog = torch.empty((m, TV), device=dev)
    hist = {}
    for f in range(4):
        text = rng.standard_normal((m, H)).astype(np.float32)
        pos = np.full(m, f, np.int32)
        fr.run(codes, text=t(text, dev), prev=t(prev, dev), pos=t(pos, dev), slots=t(slots, dev), hidden=hid,
               talker_logits=tlog)
        torch.cuda.synchronize(dev)
        got = codes.cpu().numpy()
        want, whid, wlog, wplog = O.frame(tref, pref, ptables, G, text, prev, pos, slots, state, replay=got,
                                          penalty=penalty)
        rel = np.linalg.norm(hid.cpu().numpy() - whid) / np.linalg.norm(whid)
        assert rel < 1e-2, (f, rel)
        rel = np.linalg.norm(tlog.cpu().numpy() - wlog) / np.linalg.norm(wlog)
        assert rel < 1e-2, (f, rel)
        for i in range(m):
            h = hist.setdefault(int(slots[i]), set())
            lv = wlog[i].copy()
            for c in h:
                lv[c] = lv[c] / np.float32(penalty) if lv[c] > 0 else lv[c] * np.float32(penalty)
            assert_choice(int(got[i, 0]), lv, 2e-2 * np.abs(lv).max())
            h.add(int(got[i, 0]))
            for g in range(1, G):
                assert_choice(int(got[i, g]), wplog[g - 1][i], 2e-2 * np.abs(wplog[g - 1][i]).max())
        prev = got


def test_frame_replay_and_prompt_pass(chain_mod, frame_mod, O, dev):
    """Frame 0 after a prompt pass through chain.step (skip_talker), then replayed frames: codes are the replayed
    ones and the talker follows the oracle."""
    m = 1
    fr, talker, tref, pref, ptables, state = make_frame(O, dev, chain_mod, frame_mod, m=m)
    rng = np.random.default_rng(5)
    P = 5
    prompt = rng.standard_normal((P, H)).astype(np.float32)
    ph = torch.empty((P, H), device=dev)
    plg = torch.empty((P, TV), device=dev)
    talker.step(x_in=t(prompt, dev), pos=t(np.arange(P, dtype=np.int32), dev),
                slots=t(np.zeros(P, np.int32), dev), hidden_out=ph, logits=plg)
    h0 = O.decoder_chain_attn(tref["mats"], tref["norms"], tref["qkn"], None, None, prompt,
                              np.arange(P, dtype=np.int32), state["tk"], state["tv"], slots=np.zeros(P, np.int32),
                              hidden=H, n_head=NH, n_kv=NKV, head_dim=HD, inter=I, eps=EPS, theta=THETA)
    codes = torch.empty((m, G), dtype=torch.int32, device=dev)
    fr.run(codes, hidden=ph[P - 1:], talker_logits=plg[P - 1:], skip_talker=True)
    torch.cuda.synchronize(dev)
    got = codes.cpu().numpy()
    hid_ref = O.rms_norm_rows(h0[P - 1:], tref["out_norm"], EPS)
    assert np.linalg.norm(ph[P - 1:].cpu().numpy() - hid_ref) / np.linalg.norm(hid_ref) < 1e-2
    # the frame's selection and predictor, fed the GPU's own prompt outputs
    _, _, _, wplog = O.frame(tref, pref, ptables, G, None, None, np.zeros(m, np.int32), np.zeros(m, np.int32), state,
                             replay=got, hidden_in=ph[P - 1:].cpu().numpy(), logits_in=plg[P - 1:].cpu().numpy())
    assert got[0, 0] == O.select_code(plg[P - 1].cpu().numpy())
    for g in range(1, G):
        assert_choice(int(got[0, g]), wplog[g - 1][0], 2e-2 * np.abs(wplog[g - 1][0]).max())
    prev = got
    hid = torch.empty((m, H), device=dev)
    for f in range(3):
        replay = np.stack([rng.integers(0, TV, m)] + [rng.integers(0, PV, m) for _ in range(G - 1)], 1).astype(np.int32)
        text = rng.standard_normal((m, H)).astype(np.float32)
        pos = np.full(m, P + f, np.int32)
        fr.run(codes, text=t(text, dev), prev=t(prev, dev), pos=t(pos, dev), replay=t(replay, dev), hidden=hid)
        torch.cuda.synchronize(dev)
        assert np.array_equal(codes.cpu().numpy(), replay)
        _, whid, _, _ = O.frame(tref, pref, ptables, G, text, prev, pos, np.zeros(m, np.int32), state, replay=replay)
        rel = np.linalg.norm(hid.cpu().numpy() - whid) / np.linalg.norm(whid)
        assert rel < 1e-2, (f, rel)
        prev = replay


def test_frame_selection_rule(chain_mod, frame_mod, O, dev):
    """Ties, NaN, -inf and the repetition penalty, bit-exactly against std::max_element's sequential rule."""
    m = 6
    fr, *_ = make_frame(O, dev, chain_mod, frame_mod, m=m, penalty=1.25, t_layers=1, p_layers=1)
    lg = (0.1 * np.random.default_rng(3).standard_normal((m, TV))).astype(np.float32)
    lg[0, 10] = lg[0, 200] = 9.0                      # tie: lower index
    lg[1, 0] = np.nan                                 # NaN first: index 0
    lg[2, 5] = np.nan; lg[2, 7] = 50.0                # NaN elsewhere never wins
    lg[3, :] = -np.inf                                # all -inf: index 0
    lg[4, 17] = 3.0; lg[4, 18] = 2.9                  # the penalty alternates the choice between 17 and 18
    lg[5, :] -= 2.0; lg[5, 30] = -0.5; lg[5, 31] = -0.6  # negative logits are multiplied by the penalty
    codes = torch.empty((m, G), dtype=torch.int32, device=dev)
    hid = torch.zeros((m, H), device=dev)
    hist = {}
    for rnd in range(3):
        fr.run(codes, hidden=hid, talker_logits=t(lg, dev), skip_talker=True)
        torch.cuda.synchronize(dev)
        got = codes.cpu().numpy()[:, 0]
        for i in range(m):
            h = hist.setdefault(i, set())
            assert got[i] == O.select_code(lg[i], h, 1.25), (rnd, i, got[i])
            h.add(int(got[i]))
    fr.reset_history()
    fr.run(codes, hidden=hid, talker_logits=t(lg, dev), skip_talker=True)
    torch.cuda.synchronize(dev)
    assert [int(c) for c in codes.cpu().numpy()[:, 0]] == [O.select_code(lg[i]) for i in range(m)]


def test_frame_with_input_projection(chain_mod, frame_mod, O, dev):
    """A predictor narrower than the talker (the 1.7B packages' small_to_mtp_projection): every predictor input row
    is projected, x = W * Q(x) + b, before its layers; greedy frames against the oracle replaying the GPU's codes."""
    m = 2
    HP = 512
    talker, tref = stack(O, dev, 2, 4000, TV, 1, TV, chain_mod, n_ctx=16, n_slots=m, max_m=8)
    # a narrower predictor: hidden 512, 4 query heads, 2 kv heads of 128, intermediate 1024
    shapes = [(4 * HD, HP), (2 * HD, HP), (2 * HD, HP), (HP, 4 * HD), (1024, HP), (1024, HP), (HP, 1024)]
    mats, norms = [], []
    for l in range(2):
        for j, (n, k) in enumerate(shapes):
            mats.append(O.quantize_rows(O.normal(7000 + 16 * l + j, n * k, 0.03).reshape(n, k)))
        for j in range(2):
            norms.append((1.0 + 0.1 * O.normal(7000 + 16 * l + 8 + j, HP)).astype(np.float32))
    norms = np.stack(norms)
    qkn = np.stack([(1.0 + 0.2 * O.normal(7100 + i, HD)).astype(np.float32) for i in range(4)])
    out_norm = (1.0 + 0.1 * O.normal(7200, HP)).astype(np.float32)
    heads = [O.quantize_rows(O.normal(7300 + g, PV * HP, 0.03).reshape(PV, HP)) for g in range(G - 1)]
    ptables = [O.quantize_rows(O.normal(7400 + g, PV * H, 0.5).reshape(PV, H)) for g in range(G - 1)]  # talker width
    proj_w = O.quantize_rows(O.normal(7500, HP * H, 0.03).reshape(HP, H))
    proj_b = (0.1 * O.normal(7501, HP)).astype(np.float32)
    keys = ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown")
    layers = [dict({k: t(mats[7 * l + j], dev) for j, k in enumerate(keys)}, norm_in=t(norms[2 * l], dev),
                   norm_post=t(norms[2 * l + 1], dev), q_norm=t(qkn[2 * l], dev), k_norm=t(qkn[2 * l + 1], dev))
              for l in range(2)]
    pred = chain_mod.DecodeChain(layers, t(heads[0], dev), hidden=HP, n_head=4, n_kv=2, head_dim=HD, inter=1024,
                                 eps=EPS, max_m=8, attention=dict(rope_theta=THETA, n_ctx=G, n_slots=m),
                                 output=dict(norm=t(out_norm, dev), heads=[t(h, dev) for h in heads]))
    fr = frame_mod.Frame(talker, pred, [t(p, dev) for p in ptables], projection=(t(proj_w, dev), t(proj_b, dev)))
    pref = dict(mats=mats, norms=norms, qkn=qkn, out_norm=out_norm, heads=heads, hidden=HP, n_head=4, n_kv=2,
                head_dim=HD, inter=1024, eps=EPS, theta=THETA, vocab=PV, proj_w=proj_w, proj_b=proj_b)
    state = dict(tk=np.zeros((2, m, 16, KV), np.float32), tv=np.zeros((2, m, 16, KV), np.float32),
                 pk=np.zeros((2, m, G, 2 * HD), np.float32), pv=np.zeros((2, m, G, 2 * HD), np.float32), history={})
    rng = np.random.default_rng(21)
    prev = np.stack([rng.integers(0, TV, m)] + [rng.integers(0, PV, m) for _ in range(G - 1)], 1).astype(np.int32)
    codes = torch.empty((m, G), dtype=torch.int32, device=dev)
    slots = np.arange(m, dtype=np.int32)
    for f in range(3):
        text = rng.standard_normal((m, H)).astype(np.float32)
        pos = np.full(m, f, np.int32)
        fr.run(codes, text=t(text, dev), prev=t(prev, dev), pos=t(pos, dev))
        torch.cuda.synchronize(dev)
        got = codes.cpu().numpy()
        _, _, _, wplog = O.frame(tref, pref, ptables, G, text, prev, pos, slots, state, replay=got)
        for i in range(m):
            for g in range(1, G):
                assert_choice(int(got[i, g]), wplog[g - 1][i], 2e-2 * np.abs(wplog[g - 1][i]).max())
        prev = got


TH, TROWS = 512, 300  # text hidden width and text vocabulary of these tests


def text_projection(O, dev, seed=8000):
    """The talker's text side: a Q8_0 text_embedding [TROWS, TH], fc1 [TH, TH] and fc2 [H, TH] with F32 biases;
    (device dict for Frame, oracle dict for O.text_projection)."""
    ref = dict(embedding=O.quantize_rows(O.normal(seed, TROWS * TH, 0.5).reshape(TROWS, TH)),
               fc1=O.quantize_rows(O.normal(seed + 1, TH * TH, 0.05).reshape(TH, TH)),
               fc1_bias=(0.1 * O.normal(seed + 2, TH)).astype(np.float32),
               fc2=O.quantize_rows(O.normal(seed + 3, H * TH, 0.05).reshape(H, TH)),
               fc2_bias=(0.1 * O.normal(seed + 4, H)).astype(np.float32), hidden=TH)
    return {k: t(v, dev) for k, v in ref.items() if k != "hidden"}, ref


def make_text_frame(O, dev, chain_mod, frame_mod, m):
    """make_frame's talker and predictor, and a frame over them with the text projection."""
    talker, tref = stack(O, dev, 2, 4000, TV, 1, TV, chain_mod, n_ctx=16, n_slots=m, max_m=max(8, m))
    pred, pref = stack(O, dev, 2, 5000, PV, G - 1, 8, chain_mod, n_ctx=G, n_slots=m, max_m=max(8, 2 * m))
    ptables = [O.quantize_rows(O.normal(6000 + g, PV * H, 0.5).reshape(PV, H)) for g in range(G - 1)]
    tp_dev, tp_ref = text_projection(O, dev)
    fr = frame_mod.Frame(talker, pred, [t(p, dev) for p in ptables], text_projection=tp_dev)
    tref["text"] = tp_ref
    state = dict(tk=np.zeros((2, m, 16, KV), np.float32), tv=np.zeros((2, m, 16, KV), np.float32),
                 pk=np.zeros((2, m, G, KV), np.float32), pv=np.zeros((2, m, G, KV), np.float32), history={})
    return fr, tref, pref, ptables, state


@pytest.mark.parametrize("m", [1, 5])
def test_text_rows_against_oracle(chain_mod, frame_mod, O, dev, q8, m):
    """b200q8_frame_text_rows (build_text_projection, talker.cpp:37-50) op by op: the Q8_0 GET_ROWS exact (it is
    checked through fc1), fc1 within its MUL_MAT bound with the bias and silu (expf on the device and in libm may
    differ by an ulp), fc2 on the GPU's own activation within its bound plus the bias's rounding."""
    fr, tref, *_ = make_text_frame(O, dev, chain_mod, frame_mod, m)
    tp = tref["text"]
    ids = np.random.default_rng(m).integers(0, TROWS, m).astype(np.int32)
    out = torch.empty((m, H), device=dev)
    h1 = torch.empty((m, TH), device=dev)
    fr.text_rows(t(ids, dev), out, h1)
    torch.cuda.synchronize(dev)
    h1g, outg = h1.cpu().numpy(), out.cpu().numpy()
    x = O.get_rows(tp["embedding"], TH, ids)[0]
    y1, b1 = O.mul_mat(tp["fc1"], TH, x)
    h1_ref = np.ascontiguousarray(y1, np.float32)
    O.lib().oracle_bias_silu_rows(h1_ref.ctypes.data, tp["fc1_bias"].ctypes.data, m, TH)
    # silu's slope is within [-0.1, 1.1]: the MUL_MAT bound carries through, plus an ulp of the bias add and
    # an ulp or two of expf
    z = np.abs(y1.astype(np.float64) + tp["fc1_bias"])
    assert np.all(np.abs(h1g - h1_ref) <= 1.2e-5 * b1 + 5e-7 * np.abs(h1_ref) + 2.4e-7 * z + 1e-30)
    y2, b2 = O.mul_mat(tp["fc2"], TH, h1g)
    want = y2 + tp["fc2_bias"]
    assert np.all(np.abs(outg - want) <= 1e-5 * b2 + 1.2e-7 * np.abs(want) + 1e-30)
    # the whole projection against the oracle's own: only fc2's activation codes can differ, rarely
    rel = np.linalg.norm(outg - O.text_projection(tp, ids)) / np.linalg.norm(outg)
    assert rel < 2e-3, rel
    # an id outside the vocabulary: a zero embedding row, reported in the device status
    bad = ids.copy()
    bad[0] = TROWS
    fr.text_rows(t(bad, dev), out)
    torch.cuda.synchronize(dev)
    assert q8.device_status(0) == 1
    assert q8.device_status(0) == 0
    fr.close()


def test_frame_from_text_ids(chain_mod, frame_mod, O, dev):
    """Frames run from text token ids: bit-identical to frames given the text rows b200q8_frame_text_rows computes,
    and greedy frames against the oracle's frame over the same ids (the oracle replaying the GPU's codes)."""
    m = 2
    runs = []
    for use_ids in (True, False):
        fr, tref, pref, ptables, state = make_text_frame(O, dev, chain_mod, frame_mod, m)
        rng = np.random.default_rng(31)
        prev = np.stack([rng.integers(0, TV, m)] + [rng.integers(0, PV, m) for _ in range(G - 1)], 1).astype(np.int32)
        codes = torch.empty((m, G), dtype=torch.int32, device=dev)
        hid = torch.empty((m, H), device=dev)
        tlog = torch.empty((m, TV), device=dev)
        rows = torch.empty((m, H), device=dev)
        seq = []
        for f in range(4):
            ids = rng.integers(0, TROWS, m).astype(np.int32)
            pos = np.full(m, f, np.int32)
            if use_ids:
                fr.run(codes, text_ids=t(ids, dev), prev=t(prev, dev), pos=t(pos, dev), hidden=hid, talker_logits=tlog)
            else:
                fr.text_rows(t(ids, dev), rows)
                fr.run(codes, text=rows, prev=t(prev, dev), pos=t(pos, dev), hidden=hid, talker_logits=tlog)
            torch.cuda.synchronize(dev)
            got = codes.cpu().numpy()
            seq.append((got.copy(), hid.cpu().numpy(), tlog.cpu().numpy()))
            if use_ids:
                _, whid, wlog, wplog = O.frame(tref, pref, ptables, G, None, prev, pos, np.arange(m, dtype=np.int32),
                                               state, replay=got, text_ids=ids)
                rel = np.linalg.norm(seq[-1][1] - whid) / np.linalg.norm(whid)
                assert rel < 1e-2, (f, rel)
                for i in range(m):
                    assert_choice(int(got[i, 0]), wlog[i], 2e-2 * np.abs(wlog[i]).max())
                    for g in range(1, G):
                        assert_choice(int(got[i, g]), wplog[g - 1][i], 2e-2 * np.abs(wplog[g - 1][i]).max())
            prev = got
        runs.append(seq)
        fr.close()
    for (c1, h1, l1), (c2, h2, l2) in zip(*runs):
        assert np.array_equal(c1, c2) and np.array_equal(h1, h2) and np.array_equal(l1, l2)
