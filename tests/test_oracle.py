"""The CPU oracle against the golden fixtures and the reference's own code.

Pins: gguf-py 0.19.0's Q8_0 packing (tests/golden/q8_pack_fixtures.json,
q8_seeded_digests.json), the reference's NormalRandomStream and thread policy
(src/random-stream.cpp, src/cpu-parallelism.cpp compiled into oracle/_ref
when the reference tree is present), and the Q8_0 cases of
tests/vits_conv_test.cpp:293-313 with the reference's own bound.
"""
from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import pytest

pytestmark = pytest.mark.filterwarnings("ignore:overflow encountered in cast")

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


PACK = load("q8_pack_fixtures.json")


@pytest.mark.parametrize("name", sorted(PACK["cases"]))
def test_packing_matches_gguf_py(O, name):
    case = PACK["cases"][name]
    x = np.frombuffer(bytes.fromhex(case["x_f32_hex"]), np.float32).reshape(1, -1)
    golden = bytes.fromhex(case["q8_0_hex"])
    assert O.quantize_rows(x, O.QUANT_REF).tobytes() == golden
    if np.all(np.isfinite(x)):
        assert O.quantize_rows_np(x).tobytes() == golden


def test_quantize_test_probe(O):
    # tests/synthesize_quantize_test.cpp:273-278: dequantised probe 100 within 0.2 of (100+1)/7
    case = PACK["cases"]["synthesize_quantize_test_i_plus_1_over_7"]
    q = np.frombuffer(bytes.fromhex(case["q8_0_hex"]), np.uint8)
    deq = O.dequantize_rows(q, case["k"])[0]
    probe = case["probe"]
    assert abs(deq[probe["index"]] - probe["expected"]) < probe["bound"]


def test_quantize_chunk_semantics(O):
    src = (np.arange(4 * 64, dtype=np.float32) + 1) / np.float32(7)
    dst, n = O.quantize_chunk(src, 2 * 64, 2, 64)
    assert n == 2 * 68
    assert np.all(dst[: 2 * 68] == 0)
    assert dst[2 * 68:].tobytes() == O.quantize_rows(src.reshape(4, 64)[2:]).tobytes()


def test_seeded_config1_digests(O):
    d = load("q8_seeded_digests.json")["config1"]
    w = O.normal(d["w_seed"], 3072 * 1024, d["w_scale"]).reshape(3072, 1024)
    x = O.normal(d["x_seed"], 1024).reshape(1, 1024)
    assert hashlib.sha256(w.tobytes()).hexdigest() == d["w_f32_sha256"]
    assert hashlib.sha256(x.tobytes()).hexdigest() == d["x_f32_sha256"]
    assert hashlib.sha256(O.quantize_rows(w).tobytes()).hexdigest() == d["w_q8_0_sha256"]
    assert O.quantize_rows(x).tobytes().hex() == d["x_q8_0_hex"]
    assert [float(v) for v in O.normal(0, 8)] == d["first_normals_seed0"]


@pytest.mark.parametrize("seed", [0, 1, 7, 42, 2**63 + 5])
def test_rng_restatements_agree(O, seed):
    c = O.normal(seed, 301)
    py = O.PyNormalStream(seed).fill(301)
    assert np.array_equal(c, py)
    ref = O.ref_lib()
    if ref is not None:
        r = np.empty(301, np.float32)
        ref.ref_normal_fill(seed, r.ctypes.data, 301)
        assert np.array_equal(c, r)
        u = np.empty(33, np.float32)
        ref.ref_uniform_fill(seed, u.ctypes.data, 33)
        assert np.array_equal(O.uniform(seed, 33), u)


def test_thread_policy(O):
    # src/cpu-parallelism.cpp:93-99
    assert [O.default_synthesis_threads(n) for n in (1, 2, 3, 4, 8, 20)] == [1, 1, 1, 2, 4, 10]
    ref = O.ref_lib()
    if ref is not None:
        assert ref.ref_default_synthesis_threads() == O.default_synthesis_threads(ref.ref_available_cpu_parallelism())


@pytest.mark.parametrize("case", load("vits_q8_cases.json")["cases"], ids=lambda c: c["source"])
def test_vits_conv_q8_cases(O, case):
    k, n, m = case["k"], case["n"], case["m"]
    w = np.array(case["w_f32"], np.float32).reshape(n, k)
    x = np.array(case["x_f32"], np.float32).reshape(m, k)
    y, _ = O.mul_mat(O.quantize_rows(w), k, x)
    y = y + np.array(case["bias"], np.float32)[None, :]
    assert np.all(np.abs(y - np.array(case["expected"], np.float32)) < case["bound"])


def test_fp16_conversion_matches_numpy(O):
    L = O.lib()
    rng = np.random.default_rng(5)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.exp(rng.uniform(-30, 15, 20000)).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.98e-8, 5.96e-8, 6.1e-5, np.inf, -np.inf],
                 np.float32),
    ])
    for v in vals:
        h = L.oracle_fp32_to_fp16(float(v))
        assert h == int(np.array([v], np.float32).astype(np.float16).view(np.uint16)[0]), v
        back = L.oracle_fp16_to_fp32(h)
        assert back == float(np.array([h], np.uint16).view(np.float16).astype(np.float32)[0])


def test_activation_modes_differ_only_at_ties(O):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    ref = O.quantize_rows(x, O.QUANT_REF)
    arm = O.quantize_rows(x, O.QUANT_CPU_ARM)
    x86 = O.quantize_rows(x, O.QUANT_CPU_X86)
    # scales identical in every mode
    for a in (arm, x86):
        assert np.array_equal(a.reshape(-1, 34)[:, :2], ref.reshape(-1, 34)[:, :2])
    # codes differ by at most one step
    for a in (arm, x86):
        da = a.reshape(-1, 34)[:, 2:].view(np.int8).astype(int) - ref.reshape(-1, 34)[:, 2:].view(np.int8).astype(int)
        assert np.abs(da).max() <= 1
    # on exact ties REF rounds away from zero, the SIMD forms to even
    t = np.zeros((1, 32), np.float32)
    t[0, 0] = 127.0
    t[0, 1] = 2.5
    t[0, 2] = -2.5
    assert O.quantize_rows(t, O.QUANT_REF)[0, 3:5].view(np.int8).tolist() == [3, -3]
    assert O.quantize_rows(t, O.QUANT_CPU_ARM)[0, 3:5].view(np.int8).tolist() == [2, -2]
    assert O.quantize_rows(t, O.QUANT_CPU_X86)[0, 3:5].view(np.int8).tolist() == [2, -2]


def test_nan_follows_reference_fold(O):
    # amax = MAX(amax, |x|) with MAX(a,b) = a > b ? a : b: a NaN is replaced by the next value
    x = np.linspace(-1, 1, 32).astype(np.float32)
    x[3] = np.nan
    q = O.quantize_rows(x.reshape(1, 32))[0]
    d = np.array(q[:2]).view(np.float16)[0]
    assert d == np.float16(np.float32(1.0) / np.float32(127))
    assert q[2 + 3] == 0  # NaN code stored as 0
    x[31] = np.nan
    q = O.quantize_rows(x.reshape(1, 32))[0]
    assert (int(q[0]) | (int(q[1]) << 8)) == 0x7E00 and np.all(q[2:] == 0)


def test_mul_mat_bound_is_respected(O):
    rng = np.random.default_rng(3)
    k, n, m = 1024, 64, 3
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    wq, xq = O.quantize_rows(w), O.quantize_rows(x)
    y, bound = O.mul_mat(wq, k, x)
    # exact value from the codes in float64
    wd = wq.reshape(n, -1, 34)
    xd = xq.reshape(m, -1, 34)
    dw = wd[:, :, :2].copy().view(np.float16)[..., 0].astype(np.float64)
    dx = xd[:, :, :2].copy().view(np.float16)[..., 0].astype(np.float64)
    qw = wd[:, :, 2:].view(np.int8).astype(np.int64)
    qx = xd[:, :, 2:].view(np.int8).astype(np.int64)
    isum = np.einsum("nbi,mbi->mnb", qw, qx)
    exact = np.einsum("mnb,nb,mb->mn", isum.astype(np.float64), dw, dx)
    assert np.all(np.abs(y - exact) <= 1e-5 * bound)
    assert math.isclose(float(bound[0, 0]), float(np.sum(np.abs(isum[0, 0] * dw[0] * dx[0]))), rel_tol=1e-12)
