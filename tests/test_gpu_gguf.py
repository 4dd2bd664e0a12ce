"""The talker step built from a Q8_MIXED-style package (b200q8_gguf_talker_chain) equals the step built from the
same Q8_0 bytes through b200q8_chain_create, and the oracle's step, on B200."""
from __future__ import annotations

import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

from test_gguf import write_package  # noqa: E402

pytestmark = pytest.mark.gpu

HP = dict(layers=2, hidden=256, heads=4, kv=2, head_dim=64, inter=512, vocab=64, eps=1e-6)


def tiny_talker(O, tmp_path):
    p = "synthesize.qwen3-tts.talker."
    kv = {p + "layer_count": ("uint32", HP["layers"]), p + "hidden_size": ("uint32", HP["hidden"]),
          p + "attention_head_count": ("uint32", HP["heads"]), p + "key_value_head_count": ("uint32", HP["kv"]),
          p + "head_dim": ("uint32", HP["head_dim"]), p + "intermediate_size": ("uint32", HP["inter"]),
          p + "codec_vocab_size": ("uint32", HP["vocab"]), p + "rms_norm_eps": ("float32", HP["eps"]),
          p + "text_vocab_size": ("uint32", 100), p + "text_hidden_size": ("uint32", 128)}
    H, Q, KV, I = HP["hidden"], HP["heads"] * HP["head_dim"], HP["kv"] * HP["head_dim"], HP["inter"]
    shapes = {"self_attn.q_proj": (Q, H), "self_attn.k_proj": (KV, H), "self_attn.v_proj": (KV, H),
              "self_attn.o_proj": (H, Q), "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H), "mlp.down_proj": (H, I)}
    tensors, layers = [], []
    seed = 300
    for l in range(HP["layers"]):
        b = f"talker.model.layers.{l}."
        L = {}
        for key, (n, k) in shapes.items():
            seed += 1
            q = O.quantize_rows(O.normal(seed, n * k, 0.05).reshape(n, k))
            tensors.append((b + key + ".weight", q, None, gguf.GGMLQuantizationType.Q8_0))
            L[key] = q
        for key in ("input_layernorm", "post_attn_norm"):
            seed += 1
            v = (1.0 + O.normal(seed, H, 0.1)).astype(np.float32)
            tensors.append((b + key + ".weight", v, None, None))
            L[key] = v
        layers.append(L)
    table = O.quantize_rows(O.normal(999, HP["vocab"] * H, 0.05).reshape(HP["vocab"], H))
    tensors.append(("talker.model.codec_embedding.weight", table, None, gguf.GGMLQuantizationType.Q8_0))
    tensors.append(("talker.model.norm.weight", np.ones(H, np.float32), None, None))
    path = tmp_path / "tiny_talker.gguf"
    write_package(path, kv, tensors)
    return path, layers, table


@pytest.mark.parametrize("m", [1, 2, 5, 9])
def test_package_chain_matches_direct_chain(pkg, O, chain_mod, dev, tmp_path, m):
    from synthesize_cpp_b200 import gguf as G
    from synthesize_cpp_b200.workloads import stream_inputs

    path, layers, table = tiny_talker(O, tmp_path)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    direct_layers = [{"wq": t(L["self_attn.q_proj"]), "wk": t(L["self_attn.k_proj"]), "wv": t(L["self_attn.v_proj"]),
                      "wo": t(L["self_attn.o_proj"]), "wgate": t(L["mlp.gate_proj"]), "wup": t(L["mlp.up_proj"]),
                      "wdown": t(L["mlp.down_proj"]), "norm_in": t(L["input_layernorm"]),
                      "norm_post": t(L["post_attn_norm"])} for L in layers]
    direct = chain_mod.DecodeChain(direct_layers, t(table), hidden=HP["hidden"], n_head=HP["heads"], n_kv=HP["kv"],
                                   head_dim=HP["head_dim"], inter=HP["inter"], eps=HP["eps"], max_m=max(8, m))
    with G.Package(path) as p:
        from_pkg = p.talker_chain(device=dev.index or 0, max_m=max(8, m))
    x_np, ids_np = stream_inputs(m, HP["hidden"], HP["vocab"])
    x, ids = t(x_np), t(ids_np)
    h1 = torch.empty((m, HP["hidden"]), device=dev)
    h2 = torch.empty((m, HP["hidden"]), device=dev)
    direct.run(ids, x, h1)
    from_pkg.run(ids, x, h2)
    torch.cuda.synchronize()
    assert torch.equal(h1, h2)
    # and the step is the oracle's step on these weights
    mats = [L[k] for L in layers for k in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                                           "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")]
    norms = np.stack([L[k] for L in layers for k in ("input_layernorm", "post_attn_norm")])
    ref = O.decoder_chain(mats, norms, table, ids_np, x_np, hidden=HP["hidden"], n_head=HP["heads"], n_kv=HP["kv"],
                          head_dim=HP["head_dim"], inter=HP["inter"], eps=HP["eps"])
    got = h2.cpu().numpy()
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < 2e-3
    direct.close()
    from_pkg.close()


DP = dict(hidden=256, heads=4, kv=2, head_dim=64, inter=512, t_layers=2, p_layers=2, t_vocab=96, p_vocab=64,
          groups=4, eps=1e-6, theta=1.0e4, penalty=1.2)


TEXT_HIDDEN, TEXT_VOCAB = 256, 120


def tiny_decoder_package(O, tmp_path, t_hidden=None, text=False):
    """A package with the talker (attention norms, final norm, codec head) and the code predictor (layers, norm,
    per-group tables and heads), named and keyed as the reference's catalog and loader expect.  t_hidden: a talker
    wider than the predictor, which then reads its input through small_to_mtp_projection."""
    H, Q, KV, I = DP["hidden"], DP["heads"] * DP["head_dim"], DP["kv"] * DP["head_dim"], DP["inter"]
    HT = t_hidden or H
    kv = {}
    for p, layers, vocab_key, vocab, hid in (("synthesize.qwen3-tts.talker.", DP["t_layers"], "codec_vocab_size",
                                              DP["t_vocab"], HT),
                                             ("synthesize.qwen3-tts.code_predictor.", DP["p_layers"], "vocab_size",
                                              DP["p_vocab"], H)):
        kv.update({p + "layer_count": ("uint32", layers), p + "hidden_size": ("uint32", hid),
                   p + "attention_head_count": ("uint32", DP["heads"]), p + "key_value_head_count": ("uint32", DP["kv"]),
                   p + "head_dim": ("uint32", DP["head_dim"]), p + vocab_key: ("uint32", vocab),
                   p + "code_group_count": ("uint32", DP["groups"])})
    t = "synthesize.qwen3-tts.talker."
    kv.update({t + "intermediate_size": ("uint32", I), t + "rms_norm_eps": ("float32", DP["eps"]),
               t + "rope_theta": ("float32", DP["theta"]), t + "rope_type": ("string", "1d"),
               "synthesize.qwen3-tts.sampling.repetition_penalty": ("float32", DP["penalty"])})
    shapes_of = lambda h: {"self_attn.q_proj": (Q, h), "self_attn.k_proj": (KV, h), "self_attn.v_proj": (KV, h),
                           "self_attn.o_proj": (h, Q), "mlp.gate_proj": (I, h), "mlp.up_proj": (I, h),
                           "mlp.down_proj": (h, I)}
    Q8 = gguf.GGMLQuantizationType.Q8_0
    tensors = []
    stacks = {}
    seed = [700]

    def q8(n, k, scale=0.05):
        seed[0] += 1
        return O.quantize_rows(O.normal(seed[0], n * k, scale).reshape(n, k))

    def vec(n, scale):
        seed[0] += 1
        return (1.0 + O.normal(seed[0], n, scale)).astype(np.float32)

    for name, prefix, n_layers, hid in (("talker", "talker.model.layers.", DP["t_layers"], HT),
                                        ("predictor", "talker.code_predictor.model.layers.", DP["p_layers"], H)):
        layers = []
        for l in range(n_layers):
            b = f"{prefix}{l}."
            L = {}
            for key, (n, k) in shapes_of(hid).items():
                L[key] = q8(n, k)
                tensors.append((b + key + ".weight", L[key], None, Q8))
            for key, n, sc in (("input_layernorm", hid, 0.1), ("post_attn_norm", hid, 0.1),
                               ("self_attn.q_norm", DP["head_dim"], 0.2), ("self_attn.k_norm", DP["head_dim"], 0.2)):
                L[key] = vec(n, sc)
                tensors.append((b + key + ".weight", L[key], None, None))
            layers.append(L)
        stacks[name] = layers
    ttable = q8(DP["t_vocab"], HT, 0.5)
    thead = q8(DP["t_vocab"], HT)
    tnorm = vec(HT, 0.1)
    tensors += [("talker.model.codec_embedding.weight", ttable, None, Q8), ("talker.codec_head.weight", thead, None, Q8),
                ("talker.model.norm.weight", tnorm, None, None)]
    ptables, pheads = [], []
    for g in range(DP["groups"] - 1):
        ptables.append(q8(DP["p_vocab"], HT, 0.5))  # the predictor's tables are at the talker's width
        pheads.append(q8(DP["p_vocab"], H))
        tensors += [(f"talker.code_predictor.model.codec_embedding.{g}.weight", ptables[-1], None, Q8),
                    (f"talker.code_predictor.lm_head.{g}.weight", pheads[-1], None, Q8)]
    pnorm = vec(H, 0.1)
    tensors.append(("talker.code_predictor.model.norm.weight", pnorm, None, None))
    proj = None
    if HT != H:
        proj = (q8(H, HT), (0.1 * O.normal(seed[0] + 1, H)).astype(np.float32))
        tensors += [("talker.code_predictor.small_to_mtp_projection.weight", proj[0], None, Q8),
                    ("talker.code_predictor.small_to_mtp_projection.bias", proj[1], None, None)]
    if text:  # the talker's text side (catalog.cpp:271-275)
        kv.update({t + "text_hidden_size": ("uint32", TEXT_HIDDEN), t + "text_vocab_size": ("uint32", TEXT_VOCAB)})
        tp = dict(embedding=q8(TEXT_VOCAB, TEXT_HIDDEN, 0.5), fc1=q8(TEXT_HIDDEN, TEXT_HIDDEN),
                  fc1_bias=(0.1 * O.normal(seed[0] + 2, TEXT_HIDDEN)).astype(np.float32), fc2=q8(HT, TEXT_HIDDEN),
                  fc2_bias=(0.1 * O.normal(seed[0] + 3, HT)).astype(np.float32))
        tensors += [("talker.model.text_embedding.weight", tp["embedding"], None, Q8),
                    ("talker.text_projection.linear_fc1.weight", tp["fc1"], None, Q8),
                    ("talker.text_projection.linear_fc1.bias", tp["fc1_bias"], None, None),
                    ("talker.text_projection.linear_fc2.weight", tp["fc2"], None, Q8),
                    ("talker.text_projection.linear_fc2.bias", tp["fc2_bias"], None, None)]
        proj = (proj, tp)
    path = tmp_path / "tiny_decoder.gguf"
    write_package(path, kv, tensors)
    return path, stacks, (ttable, thead, tnorm), (ptables, pheads, pnorm), proj


@pytest.mark.parametrize("t_hidden", [None, 512])
def test_package_decoder_matches_direct_frame(pkg, O, chain_mod, frame_mod, dev, tmp_path, t_hidden):
    from synthesize_cpp_b200 import gguf as G

    path, stacks, (ttable, thead, tnorm), (ptables, pheads, pnorm), proj = tiny_decoder_package(O, tmp_path, t_hidden)
    HT = t_hidden or DP["hidden"]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    keys = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj",
            "wgate": "mlp.gate_proj", "wup": "mlp.up_proj", "wdown": "mlp.down_proj", "norm_in": "input_layernorm",
            "norm_post": "post_attn_norm", "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm"}
    m, n_ctx = 2, 8
    mk = lambda layers: [{k: t(L[v]) for k, v in keys.items()} for L in layers]
    common = dict(n_head=DP["heads"], n_kv=DP["kv"], head_dim=DP["head_dim"], inter=DP["inter"], eps=DP["eps"])
    talker = chain_mod.DecodeChain(mk(stacks["talker"]), t(ttable), max_m=8, hidden=HT, **common,
                                   attention=dict(rope_theta=DP["theta"], n_ctx=n_ctx, n_slots=m),
                                   output=dict(norm=t(tnorm), heads=[t(thead)]))
    pred = chain_mod.DecodeChain(mk(stacks["predictor"]), t(pheads[0]), max_m=8, hidden=DP["hidden"], **common,
                                 attention=dict(rope_theta=DP["theta"], n_ctx=DP["groups"], n_slots=m),
                                 output=dict(norm=t(pnorm), heads=[t(h) for h in pheads]))
    direct = frame_mod.Frame(talker, pred, [t(p) for p in ptables], repetition_penalty=DP["penalty"],
                             projection=(t(proj[0]), t(proj[1])) if proj else None)
    with G.Package(path) as p:
        _, _, from_pkg = p.decoder(device=dev.index or 0, max_m=m, n_ctx=n_ctx, n_slots=m)
    rng = np.random.default_rng(9)
    prev = np.stack([rng.integers(0, DP["t_vocab"], m)] +
                    [rng.integers(0, DP["p_vocab"], m) for _ in range(DP["groups"] - 1)], 1).astype(np.int32)
    outs = []
    for fr in (direct, from_pkg):
        codes = torch.empty((m, DP["groups"]), dtype=torch.int32, device=dev)
        hid = torch.empty((m, HT), device=dev)
        lg = torch.empty((m, DP["t_vocab"]), device=dev)
        pv = t(prev)
        seq = []
        for f in range(5):
            text = t(np.random.default_rng(100 + f).standard_normal((m, HT)).astype(np.float32))
            fr.run(codes, text=text, prev=pv, pos=t(np.full(m, f, np.int32)), hidden=hid, talker_logits=lg)
            seq.append((codes.clone(), hid.clone(), lg.clone()))
            pv = codes.clone()
        torch.cuda.synchronize(dev)
        outs.append(seq)
    for (c1, h1, l1), (c2, h2, l2) in zip(*outs):
        assert torch.equal(c1, c2) and torch.equal(h1, h2) and torch.equal(l1, l2)
    from_pkg.close()
    direct.close()


def test_cpp_driver_runs_a_package_like_the_python_path(pkg, O, dev, tmp_path):
    """The C++ host driver (synth_b200_frames over b200q8h_decoder_load / b200q8h_decoder_run) loads a package with
    the talker's text projection and decodes frames from text token ids, reading each frame's codes back before
    the next; its codes equal those of the same package driven from Python (b200q8_gguf_decoder + frame runs from
    the same ids), and its stop code ends a stream where the codes say so."""
    import json
    import os
    import subprocess

    from synthesize_cpp_b200 import build
    from synthesize_cpp_b200 import gguf as G

    path, *_ = tiny_decoder_package(O, tmp_path, text=True)
    m, F, start = 3, 6, 2
    rng = np.random.default_rng(44)
    ids = rng.integers(0, TEXT_VOCAB, (F, m)).astype(np.int32)
    prev = np.stack([rng.integers(0, DP["t_vocab"], m)] +
                    [rng.integers(0, DP["p_vocab"], m) for _ in range(DP["groups"] - 1)], 1).astype(np.int32)
    ids.tofile(tmp_path / "ids.i32")
    prev.tofile(tmp_path / "prev.i32")

    def drive(stop_code):
        out = tmp_path / f"codes_{stop_code}.i32"
        r = subprocess.run([build.CLI, str(path), "--streams", str(m), "--frames", str(F), "--out", str(out),
                            "--text-ids", str(tmp_path / "ids.i32"), "--prev", str(tmp_path / "prev.i32"),
                            "--start-pos", str(start), "--stop-code", str(stop_code),
                            "--device", str(dev.index or 0)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        return np.fromfile(out, np.int32).reshape(F, m, DP["groups"]), json.loads(r.stdout.strip().splitlines()[-1])

    cpp, rep = drive(-1)
    assert rep["frames"] == [F] * m
    # the Python path over the same package and inputs
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    with G.Package(path) as p:
        talker, pred, fr = p.decoder(device=dev.index or 0, max_m=m, n_ctx=start + F, n_slots=m)
    codes = torch.empty((m, DP["groups"]), dtype=torch.int32, device=dev)
    pv = t(prev)
    py = []
    for f in range(F):
        fr.run(codes, text_ids=t(ids[f]), prev=pv, pos=t(np.full(m, start + f, np.int32)))
        torch.cuda.synchronize(dev)
        py.append(codes.cpu().numpy().copy())
        pv = codes.clone()
    fr.close()
    talker.close()
    pred.close()
    assert np.array_equal(cpp, np.stack(py))
    # a stop code: each stream ends at its first frame whose code 0 is it (the stop frame not counted)
    stop = int(cpp[2, 1, 0])
    cpp2, rep2 = drive(stop)
    want = [next((f for f in range(F) if cpp[f, s, 0] == stop), F) for s in range(m)]
    assert rep2["frames"] == want
    last = max(want) + 1 if max(want) < F else F
    assert np.array_equal(cpp2[:last], cpp[:last])
    assert os.path.exists(build.CLI)
