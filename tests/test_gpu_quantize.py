"""Packing and activation quantization on the GPU, through the C ABI, against
the CPU oracle and the gguf-py golden bytes: bit-exact in every case."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.filterwarnings("ignore:overflow encountered in cast")]

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PACK = json.load(open(os.path.join(GOLDEN, "q8_pack_fixtures.json")))


def to_dev(a, dev):
    return torch.from_numpy(np.array(a, copy=True, order="C")).to(dev)


@pytest.mark.parametrize("name", sorted(PACK["cases"]))
def test_golden_packing(q8, dev, name):
    case = PACK["cases"][name]
    x = np.frombuffer(bytes.fromhex(case["x_f32_hex"]), np.float32).reshape(1, -1)
    got = q8.quantize_rows(to_dev(x, dev), q8.QUANT_REF).cpu().numpy().tobytes()
    assert got == bytes.fromhex(case["q8_0_hex"])


def random_rows(rows, k, seed, outliers=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    x *= np.exp(rng.uniform(-8, 8, (rows, 1))).astype(np.float32)
    if outliers:
        mask = rng.random((rows, k)) < 0.01
        x[mask] *= 20
    # exact ties: blocks whose amax is 127*2^e and values at half-steps
    t = rows // 3
    if t:
        x[:t, ::32] = 127.0
        x[:t, 1::32] = 2.5
        x[:t, 2::32] = -0.5
    return x


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("rows,k", [(1, 32), (3, 160), (7, 256), (64, 1024), (5, 3072), (33, 2048)])
def test_modes_match_oracle(q8, O, dev, mode, rows, k):
    x = random_rows(rows, k, seed=rows * 1000 + k + mode)
    got = q8.quantize_rows(to_dev(x, dev), mode).cpu().numpy()
    assert np.array_equal(got, O.quantize_rows(x, mode))


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_strided_and_unaligned_rows(q8, O, dev, mode):
    x = random_rows(9, 352, seed=11)
    big = torch.zeros((9, 400), dtype=torch.float32, device=dev)
    big[:, 1:353] = to_dev(x, dev)
    view = big[:, 1:353]  # row stride 1600 B, base not 16-byte aligned
    got = q8.quantize_rows(view, mode).cpu().numpy()
    assert np.array_equal(got, O.quantize_rows(x, mode))


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_non_finite_inputs(q8, O, dev, mode):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((16, 64)).astype(np.float32)
    x[0, 3] = np.nan
    x[1, 31] = np.nan
    x[2, 0] = np.inf
    x[3, 5] = -np.inf
    x[4, :32] = np.nan
    x[5, 40] = np.nan
    x[5, 50] = np.nan
    x[6, :] = 1e-42  # fp32 subnormals: 1/d overflows to inf
    x[7, 7] = 3e38
    got = q8.quantize_rows(to_dev(x, dev), mode).cpu().numpy()
    assert np.array_equal(got, O.quantize_rows(x, mode))


def test_ragged_tail_and_chunk(q8, O, dev):
    x = random_rows(3, 160, seed=4)  # 15 blocks: one 8-block run + a 7-block tail
    assert np.array_equal(q8.quantize_rows(to_dev(x, dev)).cpu().numpy(), O.quantize_rows(x))
    src = random_rows(6, 256, seed=6).ravel()
    dst = torch.zeros(6 * 272, dtype=torch.uint8, device=dev)
    n = q8.quantize_chunk(to_dev(src, dev), dst, 2 * 256, 3, 256)
    ref, nref = O.quantize_chunk(src, 2 * 256, 3, 256)
    assert n == nref == 3 * 272
    assert np.array_equal(dst.cpu().numpy(), ref)


def test_large_packing_and_round_trip(q8, O, dev):
    # a 1.7B-shaped gate matrix (6144 x 2048): bit-exact, and dequant(quant(x))
    # lands within half a step of x everywhere
    w = O.normal(77, 6144 * 2048, 0.02).reshape(6144, 2048)
    wq = q8.quantize_rows(to_dev(w, dev))
    assert np.array_equal(wq.cpu().numpy(), O.quantize_rows(w))
    back = q8.dequantize_rows(wq, 2048).cpu().numpy()
    d = wq.cpu().numpy().reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float32).reshape(6144, 64, 1)
    err = np.abs(back.reshape(6144, 64, 32) - w.reshape(6144, 64, 32))
    # half a step plus the fp16 rounding of d (127 * 2^-11 * d)
    assert np.all(err <= 0.57 * d + 1e-12)


def test_bad_arguments_raise(q8, dev):
    x = torch.zeros((2, 33), dtype=torch.float32, device=dev)
    with pytest.raises(q8.B200Q8Error) as e:
        q8.quantize_rows(x)
    assert e.value.status == 1


def test_quantize_chunk_host_matches_oracle(q8, O):
    # the quantize tool's call on host buffers: start offset, several chunks, bytes as the reference
    rows, k = 1200, 3072  # 14.7 MB of F32, one chunk; a start offset into src and dst
    src = O.normal(91, rows * k, 0.05)
    dst = np.zeros(rows * (k // 32 * 34), np.uint8)
    n = q8.quantize_chunk_host(src, dst, 200 * k, 1000, k)
    ref, nref = O.quantize_chunk(src, 200 * k, 1000, k)
    assert n == nref == 1000 * (k // 32 * 34)
    assert np.array_equal(dst, ref)


def test_quantize_chunk_host_shapes_and_release(q8, O):
    # staging is kept between calls and must serve any row width; a row wider
    # than the default staging grows it; release frees it and the next call re-creates it
    for rows, k in [(7, 32), (300, 1024), (2, 9 * 1024 * 1024), (513, 6144)]:
        src = O.normal(rows + k, rows * k, 0.3)
        dst = np.zeros(rows * (k // 32 * 34), np.uint8)
        assert q8.quantize_chunk_host(src, dst, 0, rows, k) == dst.size
        ref, _ = O.quantize_chunk(src, 0, rows, k)
        assert np.array_equal(dst, ref), (rows, k)
    q8.quantize_chunk_host_release()
    src = O.normal(5, 64 * 2048, 1.0)
    dst = np.zeros(64 * (2048 // 32 * 34), np.uint8)
    q8.quantize_chunk_host(src, dst, 0, 64, 2048)
    assert np.array_equal(dst, O.quantize_chunk(src, 0, 64, 2048)[0])


def test_quantize_chunk_host_many_chunks(q8, O):
    rows, k = 12000, 4096  # 196 MB of F32: seven 32 MB chunks through both staging buffers
    src = np.asarray(np.random.default_rng(3).standard_normal(rows * k), np.float32)
    dst = np.zeros(rows * (k // 32 * 34), np.uint8)
    assert q8.quantize_chunk_host(src, dst, 0, rows, k) == dst.size
    ref, _ = O.quantize_chunk(src, 0, rows, k)
    assert np.array_equal(dst, ref)


def _bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def _special16(rng, n, dtype):
    """Random 16-bit values with every class present: normals over a wide range, subnormals, zeros of both
    signs, infinities and NaNs."""
    if dtype == "f16":
        v = (rng.standard_normal(n) * np.exp(rng.uniform(-12, 10, n))).astype(np.float16)
        bits = v.view(np.uint16).copy()
        sub = rng.integers(1, 0x400, n // 50, dtype=np.uint16)
        specials = np.array([0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E00, 0x3C00, 0xBC00], np.uint16)
    else:
        v = (rng.standard_normal(n) * np.exp(rng.uniform(-60, 60, n))).astype(np.float32)
        bits = (v.view(np.uint32) >> 16).astype(np.uint16)
        sub = rng.integers(1, 0x80, n // 50, dtype=np.uint16)
        specials = np.array([0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x3F80, 0xBF80], np.uint16)
    pos = rng.choice(n, sub.size + specials.size * 3, replace=False)
    bits[pos[:sub.size]] = sub
    bits[pos[sub.size:]] = np.tile(specials, 3)
    return bits


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_quantize_rows_16bit_sources(q8, O, dev, dtype, mode):
    # F16 / BF16 rows are widened exactly and quantized like F32 (the quantize tool's dequantize_to_f32 path)
    rng = np.random.default_rng(17 + mode)
    rows, k = 96, 1024 + 512  # dense path with a ragged 8-block tail per row
    bits = _special16(rng, rows * k, dtype)
    f32 = bits.view(np.float16).astype(np.float32) if dtype == "f16" else _bf16_bits_to_f32(bits)
    t = torch.from_numpy(bits.view(np.int16).copy()).to(dev)
    x = t.view(torch.float16 if dtype == "f16" else torch.bfloat16).view(rows, k)
    got = q8.quantize_rows(x, mode=mode).cpu().numpy()
    ref = O.quantize_rows(f32.reshape(rows, k), mode=mode)
    assert np.array_equal(got, ref)
    # strided rows (general per-block path)
    xs = torch.zeros((rows, k + 64), dtype=x.dtype, device=dev)
    xs[:, :k] = x
    got2 = q8.quantize_rows(xs[:, :k], mode=mode).cpu().numpy()
    assert np.array_equal(got2, ref)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_quantize_chunk_host_16bit_sources(q8, O, dtype):
    rng = np.random.default_rng(5)
    rows, k = 3000, 2048  # 12 MB of 16-bit source
    bits = _special16(rng, rows * k, dtype)
    f32 = bits.view(np.float16).astype(np.float32) if dtype == "f16" else _bf16_bits_to_f32(bits)
    src = bits.view(np.float16) if dtype == "f16" else torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    dst = np.zeros(rows * (k // 32 * 34), np.uint8)
    n = q8.quantize_chunk_host_typed(src, dst, 100 * k, rows - 100, k)
    ref, nref = O.quantize_chunk(f32, 100 * k, rows - 100, k)
    assert n == nref
    assert np.array_equal(dst[100 * (k // 32 * 34):], ref[100 * (k // 32 * 34):])


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_nan_fold_out_of_range_codes(q8, O, dev, mode):
    # ggml's amax fold skips every value before a block's last NaN, so x*id can leave int8 (low byte of the
    # int32 kept) and even int32 (stored as 0, x86's cvttss2si result); GPU and oracle agree on both
    rng = np.random.default_rng(23 + mode)
    x = rng.uniform(-1, 1, (64, 32)).astype(np.float32)
    x[:, 0] = rng.uniform(-9e3, 9e3, 64)          # int32 range after scaling: low byte kept
    x[:, 1] = rng.uniform(-8e4, 8e4, 64)
    x[:, 2] = np.float32(3e12) * np.sign(rng.uniform(-1, 1, 64))  # beyond int32: 0
    x[::2, 3] = np.nan
    x[1::2, 7] = np.nan
    x = x.reshape(2, 1024)
    got = q8.quantize_rows(torch.from_numpy(x).to(dev), mode=mode).cpu().numpy()
    ref = O.quantize_rows(x, mode=mode)
    assert np.array_equal(got, ref)
    codes = ref.reshape(-1, 34)[:, 2:].view(np.int8)
    assert np.all(codes[::2, 2] == 0)
