"""CPU oracle for the Q8_0 hot path -- TEST INFRASTRUCTURE ONLY.

Two restatements of ggml's Q8_0 arithmetic as synthesize.cpp reaches it:

* ``q8_oracle.c`` (loaded here through ctypes): packing
  (``quantize_row_q8_0_ref``, reached from
  tools/synthesize-quantize/quantize.cpp:300-301), the three activation
  quantizer variants ggml-cpu's ``from_float`` may use, ``vec_dot_q8_0_q8_0``
  / MUL_MAT (operations.cpp:39-41,90-92,142), GET_ROWS (talker.cpp:44,86,
  code-predictor.cpp:31), the seeded normal stream (src/random-stream.cpp:10-48)
  and the decode-step chain.
* numpy / pure-Python versions of the packing and of the random stream,
  used to cross-check the C code and small cases.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module.  The product library never links or calls it.

Pinning: packing is checked byte-for-byte against gguf-py 0.19.0
(gguf/quants.py:378-394, rounding helper :43-47) through the fixtures in
tests/golden/; the random stream and thread policy are checked against the
reference's own sources compiled into oracle/_ref/ when that library exists.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libq8oracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libsynth_ref.so")

QK = 32
BLOCK_BYTES = 34
QUANT_REF = 0
QUANT_CPU_X86 = 1
QUANT_CPU_ARM = 2

_lib = None
_ref = None


def reference_root() -> str | None:
    """Where the reference tree is, if anywhere: $SYNTH_REFERENCE, else the "reference_path" that the
    repository's BASELINE.json records.  None when neither names an existing tree."""
    cands = [os.environ.get("SYNTH_REFERENCE")]
    try:
        import json

        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            cands.append(json.load(f).get("reference_path"))
    except (OSError, ValueError):
        pass
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "src")):
            return c
    return None


def build(reference: str | None = None) -> None:
    """Compile the oracle (and, when a reference tree is found, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    ref = reference or reference_root()
    if ref is not None:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        c_void_p, c_int64, c_size_t, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_int
        L.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.oracle_fp32_to_fp16.restype = ctypes.c_uint16
        L.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.oracle_fp16_to_fp32.restype = ctypes.c_float
        L.oracle_quantize_row_q8_0.argtypes = [c_void_p, c_void_p, c_int64, c_int]
        L.oracle_quantize_chunk_q8_0.argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_int64]
        L.oracle_quantize_chunk_q8_0.restype = c_size_t
        L.oracle_dequantize_row_q8_0.argtypes = [c_void_p, c_void_p, c_int64]
        L.oracle_vec_dot_q8_0_q8_0.argtypes = [c_int64, c_void_p, c_void_p, c_void_p]
        L.oracle_vec_dot_q8_0_q8_0.restype = ctypes.c_float
        L.oracle_mul_mat_q8_0_f32.argtypes = [c_void_p, c_int64, c_int64, c_size_t, c_void_p, c_int64, c_size_t,
                                              c_void_p, c_size_t, c_int, c_void_p, c_int]
        L.oracle_mul_mat_q8_0_q8_0.argtypes = [c_void_p, c_int64, c_int64, c_size_t, c_void_p, c_int64,
                                               c_void_p, c_size_t, c_void_p, c_int]
        L.oracle_get_rows_q8_0.argtypes = [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p]
        L.oracle_get_rows_q8_0.restype = c_int
        L.oracle_normal_fill.argtypes = [ctypes.c_uint64, c_void_p, c_size_t]
        L.oracle_uniform_fill.argtypes = [ctypes.c_uint64, c_void_p, c_size_t]
        L.oracle_normal_fill_scaled.argtypes = [ctypes.c_uint64, ctypes.c_float, c_void_p, c_size_t]
        L.oracle_normal_fill_scaled_many.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int]
        L.oracle_quantize_rows_mt.argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int]
        L.oracle_default_synthesis_threads.argtypes = [c_int]
        L.oracle_default_synthesis_threads.restype = c_int
        L.oracle_max_threads.restype = c_int
        L.oracle_decoder_chain.argtypes = [c_int, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                           ctypes.c_float, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                                           c_int, c_int]
        L.oracle_head_norm_rope.argtypes = [c_void_p, c_int64, c_int64, c_void_p, ctypes.c_float, ctypes.c_int32,
                                            ctypes.c_float, c_int]
        L.oracle_attend.argtypes = [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p]
        L.oracle_decoder_chain_attn.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                c_int64, c_int64, ctypes.c_float, ctypes.c_float, c_void_p, c_int64,
                                                c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                c_void_p, c_void_p, c_void_p, c_int, c_int]
        L.oracle_bias_silu_rows.argtypes = [c_void_p, c_void_p, c_int64, c_int64]
        L.oracle_rms_norm_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_int64, c_int64, ctypes.c_float]
        _lib = L
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own random stream / thread policy, if oracle/_ref was built."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB_PATH):
        R = ctypes.CDLL(REF_LIB_PATH)
        R.ref_normal_fill.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t]
        R.ref_uniform_fill.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t]
        R.ref_default_synthesis_threads.restype = ctypes.c_int
        R.ref_available_cpu_parallelism.restype = ctypes.c_int
        _ref = R
    return _ref


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def row_bytes(k: int) -> int:
    return k // QK * BLOCK_BYTES


# ------------------------------------------------------------------ C wrappers

def quantize_rows(x: np.ndarray, mode: int = QUANT_REF) -> np.ndarray:
    """x: float32 [rows, K] -> uint8 [rows, K/32*34] (ggml block_q8_0 rows)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    out = np.empty((rows, row_bytes(k)), dtype=np.uint8)
    L = lib()
    xr = x.reshape(rows, k)
    for r in range(rows):
        L.oracle_quantize_row_q8_0(_ptr(xr[r]), _ptr(out[r]), k, mode)
    return out


def quantize_rows_mt(x: np.ndarray, mode: int = QUANT_REF, threads: int = 0) -> np.ndarray:
    """quantize_rows on OpenMP threads (bytes identical; for building large fixtures)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    rows = x.size // k
    out = np.empty((rows, row_bytes(k)), dtype=np.uint8)
    lib().oracle_quantize_rows_mt(_ptr(x), _ptr(out), rows, k, mode, threads)
    return out


def quantize_chunk(src: np.ndarray, start: int, nrows: int, n_per_row: int) -> tuple[np.ndarray, int]:
    """ggml_quantize_chunk(Q8_0, ...) on a flat float32 buffer; returns (dst, bytes written)."""
    src = np.ascontiguousarray(src, dtype=np.float32).ravel()
    total_rows = src.size // n_per_row
    dst = np.zeros(total_rows * row_bytes(n_per_row), dtype=np.uint8)
    n = lib().oracle_quantize_chunk_q8_0(_ptr(src), _ptr(dst), start, nrows, n_per_row)
    return dst, n


def dequantize_rows(q: np.ndarray, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8).reshape(-1, row_bytes(k))
    out = np.empty((q.shape[0], k), dtype=np.float32)
    L = lib()
    for r in range(q.shape[0]):
        L.oracle_dequantize_row_q8_0(_ptr(q[r]), _ptr(out[r]), k)
    return out


def mul_mat(w_q: np.ndarray, k: int, x: np.ndarray, mode: int = QUANT_REF, threads: int = 0,
            want_bound: bool = True):
    """ggml_mul_mat(W Q8_0 [N rows], x F32 [M, K]) -> (y [M, N], bound [M, N])."""
    w_q = np.ascontiguousarray(w_q, dtype=np.uint8)
    n = w_q.shape[0]
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    bound = np.empty((m, n), dtype=np.float64) if want_bound else None
    lib().oracle_mul_mat_q8_0_f32(_ptr(w_q), k, n, w_q.shape[1], _ptr(x), m, k * 4, _ptr(y), n * 4, mode,
                                  _ptr(bound) if bound is not None else None, threads)
    return y, bound


def mul_mat_q8(w_q: np.ndarray, k: int, xq: np.ndarray, threads: int = 0):
    """MUL_MAT with already-quantized activations xq [M, K/32*34]."""
    w_q = np.ascontiguousarray(w_q, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8).reshape(-1, row_bytes(k))
    n, m = w_q.shape[0], xq.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    bound = np.empty((m, n), dtype=np.float64)
    lib().oracle_mul_mat_q8_0_q8_0(_ptr(w_q), k, n, w_q.shape[1], _ptr(xq), m, _ptr(y), n * 4, _ptr(bound), threads)
    return y, bound


def get_rows(table_q: np.ndarray, k: int, ids: np.ndarray) -> tuple[np.ndarray, int]:
    table_q = np.ascontiguousarray(table_q, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, k), dtype=np.float32)
    st = lib().oracle_get_rows_q8_0(_ptr(table_q), k, table_q.shape[0], _ptr(ids), ids.size, _ptr(out))
    return out, st


def normal(seed: int, count: int, scale: float | None = None) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    if scale is None:
        lib().oracle_normal_fill(seed, _ptr(out), count)
    else:
        lib().oracle_normal_fill_scaled(seed, scale, _ptr(out), count)
    return out


def normal_many(seeds, scales, counts, threads: int = 0) -> list:
    """[normal(seeds[j], counts[j], scales[j]) for j] filled on OpenMP threads (same values)."""
    n = len(seeds)
    outs = [np.empty(c, dtype=np.float32) for c in counts]
    s = (ctypes.c_uint64 * n)(*seeds)
    f = (ctypes.c_float * n)(*scales)
    p = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    c = (ctypes.c_size_t * n)(*counts)
    lib().oracle_normal_fill_scaled_many(n, s, f, p, c, threads)
    return outs


def uniform(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().oracle_uniform_fill(seed, _ptr(out), count)
    return out


def default_synthesis_threads(available: int) -> int:
    return lib().oracle_default_synthesis_threads(available)


def decoder_chain(weights_q, norms: np.ndarray, table_q: np.ndarray, ids: np.ndarray, x_in: np.ndarray, *,
                  hidden: int, n_head: int, n_kv: int, head_dim: int, inter: int, eps: float = 1e-6,
                  mode: int = QUANT_REF, threads: int = 0) -> np.ndarray:
    """The decode-step chain; weights_q: list of n_layers*7 uint8 arrays (q,k,v,o,gate,up,down)."""
    n_layers = len(weights_q) // 7
    ptrs = (ctypes.c_void_p * len(weights_q))(*[_ptr(np.ascontiguousarray(w)) for w in weights_q])
    norms = np.ascontiguousarray(norms, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    x_in = np.ascontiguousarray(x_in, dtype=np.float32).reshape(-1, hidden)
    m = x_in.shape[0]
    h = np.empty((m, hidden), dtype=np.float32)
    lib().oracle_decoder_chain(n_layers, ptrs, _ptr(norms), hidden, n_head, n_kv, head_dim, inter, eps,
                               _ptr(table_q), table_q.shape[0], _ptr(ids), _ptr(x_in), m, _ptr(h), mode, threads)
    return h


def head_norm_rope(x: np.ndarray, head_dim: int, w, eps: float, pos: int, theta: float, rope: bool = True) -> np.ndarray:
    """Per-head RMS norm (w: [head_dim] or None) then NEOX RoPE at pos; x: [..., n_heads*head_dim] (one token)."""
    y = np.array(x, dtype=np.float32, copy=True).ravel()
    wp = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    lib().oracle_head_norm_rope(_ptr(y), y.size // head_dim, head_dim, None if wp is None else _ptr(wp), eps, pos,
                                theta, 1 if rope else 0)
    return y


def attend(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, npos: int, n_head: int, n_kv: int,
           head_dim: int) -> np.ndarray:
    """One token's attention over npos cached rows (kc, vc: [>=npos, n_kv*head_dim])."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(kc, dtype=np.float32)
    vc = np.ascontiguousarray(vc, dtype=np.float32)
    out = np.empty(n_head * head_dim, np.float32)
    lib().oracle_attend(_ptr(q), _ptr(kc), _ptr(vc), npos, n_head, n_kv, head_dim, _ptr(out))
    return out


def decoder_chain_attn(weights_q, norms: np.ndarray, qk_norms: np.ndarray, table_q: np.ndarray | None,
                       ids: np.ndarray | None, x_in: np.ndarray, pos: np.ndarray, kcache: np.ndarray,
                       vcache: np.ndarray, *, hidden: int, n_head: int, n_kv: int, head_dim: int, inter: int,
                       eps: float = 1e-6, theta: float = 1e6, mode: int = QUANT_REF, threads: int = 0,
                       slots: np.ndarray | None = None) -> np.ndarray:
    """The decode step with the reference's attention; kcache/vcache [n_layers, n_slots, n_ctx, n_kv*head_dim]
    float32, updated in place (token m uses slot slots[m], default m, at position pos[m]).  table_q None: h = x_in."""
    n_layers = len(weights_q) // 7
    ptrs = (ctypes.c_void_p * len(weights_q))(*[_ptr(np.ascontiguousarray(w)) for w in weights_q])
    norms = np.ascontiguousarray(norms, dtype=np.float32)
    qk_norms = np.ascontiguousarray(qk_norms, dtype=np.float32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    x_in = np.ascontiguousarray(x_in, dtype=np.float32).reshape(-1, hidden)
    assert kcache.flags.c_contiguous and vcache.flags.c_contiguous and kcache.dtype == np.float32
    m = x_in.shape[0]
    if slots is not None:
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        assert slots.min() >= 0 and slots.max() < kcache.shape[1]
    else:
        assert m <= kcache.shape[1]
    if table_q is not None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
    h = np.empty((m, hidden), dtype=np.float32)
    lib().oracle_decoder_chain_attn(n_layers, ptrs, _ptr(norms), _ptr(qk_norms), hidden, n_head, n_kv, head_dim,
                                    inter, eps, theta, _ptr(table_q) if table_q is not None else None,
                                    table_q.shape[0] if table_q is not None else 0,
                                    _ptr(ids) if table_q is not None else None, _ptr(x_in), _ptr(pos),
                                    _ptr(slots) if slots is not None else None, m, kcache.shape[1], kcache.shape[2],
                                    _ptr(kcache), _ptr(vcache), _ptr(h), mode, threads)
    return h


def rms_norm_rows(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm(x) * w per row (ggml_rms_norm: sum of squares in double, scale 1/sqrtf(mean + eps))."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, n = x.reshape(-1, x.shape[-1]).shape
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty((rows, n), dtype=np.float32)
    lib().oracle_rms_norm_rows(_ptr(x), _ptr(w), _ptr(y), rows, n, eps)
    return y


def select_code(logits: np.ndarray, history: set | None = None, penalty: float = 1.0) -> int:
    """The reference's greedy choice (sample == false): std::max_element over the logits after the repetition
    penalty (src/arch/qwen3-tts/code-predictor-host.cpp:45-49,51-69,71-80), in float32, sequentially."""
    v = np.array(logits, dtype=np.float32)
    if history and penalty > 1.0:
        p = np.float32(penalty)
        for c in history:
            if 0 <= c < v.size:
                v[c] = v[c] / p if v[c] > 0 else v[c] * p
    best = 0
    for i in range(1, v.size):
        if v[best] < v[i]:
            best = i
    return best


def text_projection(tp: dict, ids: np.ndarray, mode: int = QUANT_REF, threads: int = 0, want_h1: bool = False):
    """The talker's text rows for text token ids (build_text_projection, src/arch/qwen3-tts/talker.cpp:37-50):
    GET_ROWS from the Q8_0 text_embedding, fc1 (Q8_0 MUL_MAT) + bias, silu, fc2 + bias.  tp: dict(embedding, fc1,
    fc1_bias, fc2, fc2_bias, hidden = the text width).  Returns the rows [M, talker hidden] (and, with want_h1,
    silu(fc1 + b1) [M, text hidden] as well)."""
    Th = tp["hidden"]
    x = get_rows(tp["embedding"], Th, np.asarray(ids, np.int32))[0]
    h1 = np.ascontiguousarray(mul_mat(tp["fc1"], Th, x, mode, threads, want_bound=False)[0])
    lib().oracle_bias_silu_rows(_ptr(h1), _ptr(np.ascontiguousarray(tp["fc1_bias"], np.float32)), h1.shape[0], Th)
    out = (mul_mat(tp["fc2"], Th, h1, mode, threads, want_bound=False)[0] + tp["fc2_bias"]).astype(np.float32)
    return (out, h1) if want_h1 else out


def frame(talker: dict, predictor: dict, ptables: list, groups: int, text: np.ndarray | None, prev: np.ndarray | None,
          pos: np.ndarray, slots: np.ndarray, state: dict, *, replay: np.ndarray | None = None, penalty: float = 1.0,
          hidden_in: np.ndarray | None = None, logits_in: np.ndarray | None = None, mode: int = QUANT_REF,
          threads: int = 0, text_ids: np.ndarray | None = None):
    """One decode frame for M streams (src/arch/qwen3-tts/model.cpp:1310-1489 with request.sample == false or
    replay codes): talker step on sum(code embeddings) + text, greedy/replayed code 0, predictor prefill over
    [hidden, ttable[code 0]] at positions 0, 1 and G-2 single-position predictor steps.  talker / predictor: dicts
    with mats, norms, qkn, table (talker only), out_norm, heads (list of Q8_0 arrays), hidden, n_head, n_kv,
    head_dim, inter, eps, theta, vocab; the predictor's may hold proj_w / proj_b (its input projection), the
    talker's "text" (a text_projection dict; then text_ids [M] may replace text).  state: {"tk", "tv", "pk", "pv" caches, "history": {slot: set}} updated in
    place.  hidden_in / logits_in: the talker's outputs when its step already ran (the prompt pass).
    Returns (codes [M, G] int32, talker hidden [M, H], talker logits [M, V], predictor logits: a list of G-1
    arrays [M, V_p], the one each acoustic code was chosen from)."""
    T, P = talker, predictor
    H = T["hidden"]
    M = pos.shape[0]
    dims = lambda c: dict(hidden=c["hidden"], n_head=c["n_head"], n_kv=c["n_kv"], head_dim=c["head_dim"],
                          inter=c["inter"], eps=c["eps"], theta=c["theta"], mode=mode, threads=threads)
    if hidden_in is None and text_ids is not None:  # text rows through the talker's text projection
        text = text_projection(T["text"], text_ids, mode, threads)
    if hidden_in is None:
        x = np.empty((M, H), np.float32)
        for m in range(M):
            acc = get_rows(ptables[0], H, prev[m, 1:2])[0][0]
            for g in range(2, groups):
                acc = (acc + get_rows(ptables[g - 1], H, prev[m, g:g + 1])[0][0]).astype(np.float32)
            acc = (acc + get_rows(T["table"], H, prev[m, 0:1])[0][0]).astype(np.float32)
            x[m] = (acc + text[m]).astype(np.float32)
        h = decoder_chain_attn(T["mats"], T["norms"], T["qkn"], None, None, x, pos, state["tk"], state["tv"],
                               slots=slots, **dims(T))
        hid = rms_norm_rows(h, T["out_norm"], T["eps"])
        logits = mul_mat(T["heads"][0], H, hid, mode, threads, want_bound=False)[0]
    else:
        hid, logits = hidden_in, logits_in
    codes = np.zeros((M, groups), np.int32)
    for m in range(M):
        if replay is not None:
            codes[m, 0] = replay[m, 0]
        else:
            hist = state["history"].setdefault(int(slots[m]), set())
            codes[m, 0] = select_code(logits[m], hist, penalty)
            hist.add(int(codes[m, 0]))
    def project(x):  # a predictor narrower than the talker: x = W * Q(x) + b (code-predictor.cpp:49-58)
        if "proj_w" not in P:
            return x
        return (mul_mat(P["proj_w"], H, x, mode, threads, want_bound=False)[0] + P["proj_b"]).astype(np.float32)

    # predictor prefill: two positions per stream
    xp = np.empty((2 * M, H), np.float32)
    xp[0::2] = hid
    xp[1::2] = get_rows(T["table"], H, codes[:, 0])[0]
    xp = project(xp)
    pp = np.tile(np.array([0, 1], np.int32), M)
    ps = np.repeat(np.asarray(slots, np.int32), 2)
    h = decoder_chain_attn(P["mats"], P["norms"], P["qkn"], None, None, xp, pp, state["pk"], state["pv"], slots=ps,
                           **dims(P))
    Hp = P["hidden"]
    lg = mul_mat(P["heads"][0], Hp, rms_norm_rows(h[1::2], P["out_norm"], P["eps"]), mode, threads, want_bound=False)[0]
    plogits = [lg]
    for m in range(M):
        codes[m, 1] = replay[m, 1] if replay is not None else select_code(lg[m])
    for g in range(1, groups - 1):
        x = project(get_rows(ptables[g - 1], H, codes[:, g])[0])
        h = decoder_chain_attn(P["mats"], P["norms"], P["qkn"], None, None, x, np.full(M, g + 1, np.int32),
                               state["pk"], state["pv"], slots=slots, **dims(P))
        lg = mul_mat(P["heads"][g], Hp, rms_norm_rows(h, P["out_norm"], P["eps"]), mode, threads, want_bound=False)[0]
        plogits.append(lg)
        for m in range(M):
            codes[m, g + 1] = replay[m, g + 1] if replay is not None else select_code(lg[m])
    return codes, hid, logits, plogits


# ---------------------------------------------------- numpy / Python restatements

def np_roundf(v: np.ndarray) -> np.ndarray:
    """Round half away from zero (C roundf), in float32."""
    a = np.abs(v)
    f = np.floor(a)
    r = f + (a - f >= np.float32(0.5)).astype(np.float32)
    return np.copysign(r, v).astype(np.float32)


def quantize_rows_np(x: np.ndarray) -> np.ndarray:
    """numpy restatement of quantize_row_q8_0_ref for finite inputs."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.reshape(-1, x.shape[-1]).shape
    blocks = x.reshape(-1, QK)
    amax = np.abs(blocks).max(axis=1, keepdims=True)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np_roundf((blocks * idv).astype(np.float32)).astype(np.int8)
    out = np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
    return out.reshape(rows, row_bytes(k))


class PyNormalStream:
    """Pure-Python restatement of synth::NormalRandomStream (src/random-stream.cpp:10-48)."""

    M64 = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = seed & self.M64
        self.spare = None

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & self.M64
        v = self.state
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & self.M64
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & self.M64
        return v ^ (v >> 31)

    def uniform_open(self) -> float:
        return ((self.next_u64() >> 11) + 0.5) * (1.0 / 9007199254740992.0)

    def next(self) -> float:
        if self.spare is not None:
            s, self.spare = self.spare, None
            return s
        while True:
            first = 2.0 * self.uniform_open() - 1.0
            second = 2.0 * self.uniform_open() - 1.0
            radius = first * first + second * second
            if not (radius >= 1.0 or radius == 0.0):
                break
        scale = math.sqrt(-2.0 * math.log(radius) / radius)
        self.spare = float(np.float32(second * scale))
        return float(np.float32(first * scale))

    def fill(self, count: int) -> np.ndarray:
        return np.array([self.next() for _ in range(count)], dtype=np.float32)
