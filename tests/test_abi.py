"""The C ABI library loads and exports what include/b200q8.h declares, and its
argument checks answer with synth_status_t codes -- all without a GPU (no
compute call is made)."""
from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest


def test_every_declared_symbol_is_exported(pkg):
    from synthesize_cpp_b200 import _abi

    L = _abi.lib()
    declared = _abi.header_symbols()
    assert len(declared) >= 13
    for name in declared:
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_gguf_header_is_exported(pkg):
    import os

    from synthesize_cpp_b200 import _abi

    hdr = os.path.join(os.path.dirname(_abi.HEADER), "b200q8_gguf.h")
    declared = _abi.header_symbols(hdr)
    assert declared == ["b200q8_gguf_close", "b200q8_gguf_decoder", "b200q8_gguf_find_tensor", "b200q8_gguf_get_f32",
                        "b200q8_gguf_get_str",
                        "b200q8_gguf_get_u32", "b200q8_gguf_open", "b200q8_gguf_talker_chain", "b200q8_gguf_tensor",
                        "b200q8_gguf_tensor_count"]
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_ggml_seam_header_is_exported_by_the_host_library(pkg):
    import os

    from synthesize_cpp_b200 import _abi, host

    hdr = os.path.join(os.path.dirname(_abi.HEADER), "b200q8_ggml.h")
    declared = _abi.header_symbols(hdr)
    assert declared == ["b200q8_ggml_compute_node", "b200q8_ggml_graph_compute", "b200q8_ggml_supports_op",
                        "b200q8_ggml_workspace_size"]
    L = host.lib()
    for name in declared:
        assert hasattr(L, name), name


def test_ggml_supports_op_rules(pkg):
    from synthesize_cpp_b200 import ggml_seam as G

    K, N, M = 1024, 3072, 3
    w = G.tensor(G.TYPE_Q8_0, [K, N], [34, K // 32 * 34])
    x = G.tensor(G.TYPE_F32, [K, M], [4, K * 4])
    y = G.tensor(G.TYPE_F32, [N, M], [4, N * 4], op=G.OP_MUL_MAT, src=(w, x))
    assert G.supports_op(y)
    assert G.lib().b200q8_ggml_workspace_size(y) == pkg.lib().b200q8_mul_mat_workspace_size(K, N, M)
    # F16 weights, odd K, shape mismatch, strided elements: refused (ggml-cpu keeps them)
    w16 = G.tensor(G.TYPE_F16, [K, N], [2, K * 2])
    assert not G.supports_op(G.tensor(G.TYPE_F32, [N, M], [4, N * 4], op=G.OP_MUL_MAT, src=(w16, x)))
    wodd = G.tensor(G.TYPE_Q8_0, [40, N], [34, 68])
    xodd = G.tensor(G.TYPE_F32, [40, M], [4, 160])
    assert not G.supports_op(G.tensor(G.TYPE_F32, [N, M], [4, N * 4], op=G.OP_MUL_MAT, src=(wodd, xodd)))
    assert not G.supports_op(G.tensor(G.TYPE_F32, [N + 1, M], [4, N * 4 + 4], op=G.OP_MUL_MAT, src=(w, x)))
    xs = G.tensor(G.TYPE_F32, [K, M], [8, K * 8])
    assert not G.supports_op(G.tensor(G.TYPE_F32, [N, M], [4, N * 4], op=G.OP_MUL_MAT, src=(w, xs)))
    # broadcast over dim 2: src0 ne2 = 2, src1 ne2 = 4 is fine, 3 is not
    w3 = G.tensor(G.TYPE_Q8_0, [K, N, 2], [34, K // 32 * 34, N * K // 32 * 34])
    x4 = G.tensor(G.TYPE_F32, [K, M, 4], [4, K * 4, K * M * 4])
    assert G.supports_op(G.tensor(G.TYPE_F32, [N, M, 4], [4, N * 4, N * M * 4], op=G.OP_MUL_MAT, src=(w3, x4)))
    x3 = G.tensor(G.TYPE_F32, [K, M, 3], [4, K * 4, K * M * 4])
    assert not G.supports_op(G.tensor(G.TYPE_F32, [N, M, 3], [4, N * 4, N * M * 4], op=G.OP_MUL_MAT, src=(w3, x3)))
    # GET_ROWS of a Q8_0 table by I32 ids
    table = G.tensor(G.TYPE_Q8_0, [K, 3072], [34, K // 32 * 34])
    ids = G.tensor(G.TYPE_I32, [5], [4])
    assert G.supports_op(G.tensor(G.TYPE_F32, [K, 5], [4, K * 4], op=G.OP_GET_ROWS, src=(table, ids)))
    ids16 = G.tensor(G.TYPE_F16, [5], [2])
    assert not G.supports_op(G.tensor(G.TYPE_F32, [K, 5], [4, K * 4], op=G.OP_GET_ROWS, src=(table, ids16)))
    assert not G.supports_op(G.tensor(G.TYPE_F32, [K, 5], [4, K * 4], op=99, src=(table, ids)))


def test_version_and_workspace(pkg):
    from synthesize_cpp_b200 import _abi

    L = _abi.lib()
    assert L.b200q8_version() == 100
    # K % 256 == 0: room for the tensor-core path's staged activation records,
    # (K / 256) chunks x 8 token slots x 288 bytes for M <= 8
    assert L.b200q8_mul_mat_workspace_size(1024, 3072, 1) == 4 * 8 * 288
    assert L.b200q8_mul_mat_workspace_size(1024, 3072, 64) == 4 * 64 * 288
    # other K: the quantized activations of the general path, M rows of K/32 blocks
    assert L.b200q8_mul_mat_workspace_size(96, 10, 3) == 256 * ((3 * 3 * 34 + 255) // 256)
    assert L.b200q8_mul_mat_workspace_size(33, 1, 1) == 0


def test_workspace_counts_the_tcgen05_planes_only_when_switched_on(pkg):
    """B200Q8_TC_MIN_M (read once per process, so checked in a fresh one) makes the workspace query add the
    tcgen05 GEMM's planes from that M on: int8 codes of W and x, fp32 scales of both and -1.5*2^23*dx for x
    (rows padded to 4), each plane 256-aligned.  Below that M, and without the variable, the sizes stay the mma.sync path's."""
    import os
    import sys

    code = (
        "import sys; sys.path.insert(0, %r); import __graft_entry__ as g; g.load_package();"
        "from synthesize_cpp_b200 import _abi; L = _abi.lib();"
        "print(L.b200q8_mul_mat_workspace_size(1024, 3072, 2048), L.b200q8_mul_mat_workspace_size(1024, 3072, 1023),"
        " L.b200q8_mul_mat_workspace_size(2048, 33, 1030))"
    ) % os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    al = lambda v: (v + 255) // 256 * 256
    planes = lambda k, n, m: (al(n * k) + al(k // 32 * ((n + 3) // 4 * 4) * 4) + al(m * k)
                              + 2 * al(k // 32 * ((m + 3) // 4 * 4) * 4))
    on = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                        env=dict(os.environ, B200Q8_TC_MIN_M="1024"), check=True).stdout.split()
    off = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         env={k: v for k, v in os.environ.items() if k != "B200Q8_TC_MIN_M"},
                         check=True).stdout.split()
    on, off = [int(v) for v in on], [int(v) for v in off]
    assert on[0] == max(off[0], planes(1024, 3072, 2048))
    assert on[0] > off[0]
    assert on[1] == off[1]  # M below the threshold
    assert on[2] == max(off[2], planes(2048, 33, 1030))


def test_invalid_arguments_report_status_and_message(pkg):
    from synthesize_cpp_b200 import _abi

    L = _abi.lib()
    st = L.b200q8_mul_mat(None, 33, 4, 34, None, 1, 0, None, 0, 0, None, 0, None)
    assert st == _abi.ERR_INVALID_ARG
    code, msg = _abi.last_error()
    assert code == _abi.ERR_INVALID_ARG and "multiple of 32" in msg
    assert L.b200q8_mul_mat(None, 64, 4, 68, None, 1, 0, None, 0, 7, None, 0, None) == _abi.ERR_INVALID_ARG
    assert "mode" in _abi.last_error()[1]
    assert L.b200q8_quantize_rows(None, 2, 48, 0, None, 0, 0, None) == _abi.ERR_INVALID_ARG
    assert L.b200q8_quantize_chunk(None, None, 5, 1, 32, None, None) == _abi.ERR_INVALID_ARG
    assert L.b200q8_get_rows(None, 40, 1, 0, None, 1, None, 0, None) == _abi.ERR_INVALID_ARG
    assert L.b200q8_dequantize_rows(None, 1, 31, 0, None, 0, None) == _abi.ERR_INVALID_ARG
    h = ctypes.c_void_p()
    assert L.b200q8_chain_create(None, 0, ctypes.byref(h)) == _abi.ERR_INVALID_ARG
    p = ctypes.c_void_p()
    assert L.b200q8_chain_buffer(None, 0, 0, ctypes.byref(p), None) == _abi.ERR_INVALID_ARG
    # empty work is a successful no-op
    assert L.b200q8_mul_mat(None, 64, 0, 68, None, 1, 0, None, 0, 0, None, 0, None) == _abi.OK
    assert L.b200q8_quantize_rows(None, 0, 64, 0, None, 0, 0, None) == _abi.OK


def test_chain_desc_validation(pkg):
    from synthesize_cpp_b200 import _abi

    L = _abi.lib()
    layers = (_abi.Layer * 1)()
    desc = _abi.ChainDesc(1, 1000, 16, 8, 128, 3072, 1e-6, 1, 0, ctypes.cast(layers, ctypes.POINTER(_abi.Layer)),
                          1, 10)
    h = ctypes.c_void_p()
    assert L.b200q8_chain_create(ctypes.byref(desc), 0, ctypes.byref(h)) == _abi.ERR_INVALID_ARG  # hidden % 256
    desc.hidden = 1024
    assert L.b200q8_chain_create(ctypes.byref(desc), 0, ctypes.byref(h)) == _abi.ERR_INVALID_ARG  # null weights
    assert "null" in _abi.last_error()[1]


def test_host_stream_matches_oracle_and_reference(pkg, O):
    from synthesize_cpp_b200 import host

    for seed in (0, 1, 42, 12345):
        a = host.normal(seed, 1000)
        assert np.array_equal(a, O.normal(seed, 1000))
        assert np.array_equal(host.normal(seed, 100, 0.02), O.normal(seed, 100, 0.02))
    outs = [np.empty(n, np.float32) for n in (5, 1000, 77)]
    host.normal_many([3, 4, 5], [1.0, 0.5, 2.0], outs, threads=3)
    for o, s, f in zip(outs, (3, 4, 5), (1.0, 0.5, 2.0)):
        assert np.array_equal(o, O.normal(s, o.size, f) if f != 1.0 else O.normal(s, o.size))
    assert [host.default_threads(n) for n in (1, 2, 3, 16)] == [1, 1, 1, 8]
    ref = O.ref_lib()
    if ref is not None:
        r = np.empty(500, np.float32)
        ref.ref_normal_fill(77, r.ctypes.data, 500)
        assert np.array_equal(host.normal(77, 500), r)


def test_product_library_does_not_link_the_oracle(pkg):
    from synthesize_cpp_b200 import _abi, host

    for path in (_abi.LIB_PATH, host.HOST_LIB):
        deps = subprocess.run(["ldd", path], capture_output=True, text=True).stdout
        assert "q8oracle" not in deps and "synth_ref" not in deps
        syms = subprocess.run(["nm", "-D", path], capture_output=True, text=True).stdout
        assert "oracle_" not in syms


@pytest.mark.parametrize("name", ["q8", "chain", "workloads", "host"])
def test_modules_import_without_gpu(pkg, name):
    import importlib

    importlib.import_module("synthesize_cpp_b200." + name)


def test_host_driver_header_is_exported_and_checks_arguments(pkg, tmp_path):
    """include/b200q8_host.h: every function exported by libb200q8_host.so; argument and file errors answer with
    status codes and a message before any device is touched; the command-line driver prints its usage."""
    import os

    from synthesize_cpp_b200 import _abi, build, host

    hdr = os.path.join(os.path.dirname(_abi.HEADER), "b200q8_host.h")
    declared = _abi.header_symbols(hdr)
    assert declared == ["b200q8h_decoder_free", "b200q8h_decoder_info_get", "b200q8h_decoder_load",
                        "b200q8h_decoder_run", "b200q8h_last_error"]
    out = subprocess.run(["nm", "-D", "--defined-only", host.HOST_LIB], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported
    L = host.lib()
    L.b200q8h_decoder_load.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p]
    L.b200q8h_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    buf = ctypes.create_string_buffer(512)
    h = ctypes.c_void_p()
    assert L.b200q8h_decoder_load(b"x.gguf", None, ctypes.byref(h)) == _abi.ERR_INVALID_ARG
    assert L.b200q8h_last_error(buf, 512) == _abi.ERR_INVALID_ARG and b"null" in buf.value

    class Params(ctypes.Structure):
        _fields_ = [("device", ctypes.c_int32), ("max_streams", ctypes.c_int64), ("n_ctx", ctypes.c_int64),
                    ("mode", ctypes.c_int32)]

    missing = str(tmp_path / "missing.gguf").encode()
    assert L.b200q8h_decoder_load(missing, ctypes.byref(Params(0, 1, 16, 0)), ctypes.byref(h)) != _abi.OK
    L.b200q8h_last_error(buf, 512)
    assert b"decoder_load" in buf.value and not h.value
    r = subprocess.run([build.CLI], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr
