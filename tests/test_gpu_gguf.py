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
