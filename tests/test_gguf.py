"""The library's GGUF reader (include/b200q8_gguf.h) on files written by gguf-py 0.19.0, the writer version the
reference's conversion environment pins (scripts/envs/qwen3-tts/uv.lock:291-293).  Host code only: no GPU."""
from __future__ import annotations

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def write_package(path, kv, tensors):
    w = gguf.GGUFWriter(str(path), "synthesize")
    for key, (kind, value) in kv.items():
        getattr(w, "add_" + kind)(key, value)
    for name, arr, raw_shape, raw_dtype in tensors:
        w.add_tensor(name, arr, raw_shape=raw_shape, raw_dtype=raw_dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture()
def pkg_mod(pkg):
    from synthesize_cpp_b200 import gguf as G

    return G


def sample(tmp_path):
    rng = np.random.default_rng(7)
    f32 = rng.standard_normal((3, 64)).astype(np.float32)
    f16 = rng.standard_normal((5, 32)).astype(np.float16)
    q8 = rng.integers(0, 256, (4, 2 * 34), dtype=np.uint8)
    i32 = rng.integers(-9, 9, (7,), dtype=np.int32)
    kv = {"synthesize.test.count": ("uint32", 28), "synthesize.test.eps": ("float32", 1e-6),
          "synthesize.test.name": ("string", "qwen3-tts talker"), "synthesize.test.flag": ("bool", True),
          "synthesize.test.big": ("int64", -5), "synthesize.test.list": ("array", ["a", "bc", "def"]),
          "synthesize.test.nums": ("array", [1, 2, 3, 4])}
    tensors = [("a.f32", f32, None, None), ("b.f16", f16, None, None),
               ("c.q8", q8, None, gguf.GGMLQuantizationType.Q8_0), ("d.i32", i32, None, None)]
    path = tmp_path / "sample.gguf"
    write_package(path, kv, tensors)
    return path, {"a.f32": f32, "b.f16": f16, "c.q8": q8, "d.i32": i32}


def test_reads_what_gguf_py_wrote(pkg_mod, tmp_path):
    path, arrays = sample(tmp_path)
    with pkg_mod.Package(path) as p:
        assert len(p) == 4
        assert p.get_u32("synthesize.test.count") == 28
        assert p.get_f32("synthesize.test.eps") == np.float32(1e-6)
        assert p.get_str("synthesize.test.name") == "qwen3-tts talker"
        expect = {"a.f32": (0, [64, 3]), "b.f16": (1, [32, 5]), "c.q8": (8, [64, 4]), "d.i32": (26, [7, 1])}
        for name, (typ, ne) in expect.items():
            t = p.info(name)
            assert t.name.decode() == name and t.type == typ
            assert list(t.ne)[:2] == ne and list(t.ne)[2:] == [1, 1]
            assert t.nbytes == arrays[name].nbytes
            assert p.tensor_bytes(name).tobytes() == arrays[name].tobytes()
        assert p.find("absent") == -1
        # gguf-py's own reader sees the same bytes for every tensor
        r = gguf.GGUFReader(str(path))
        for rt in r.tensors:
            assert np.asarray(rt.data).view(np.uint8).tobytes() == p.tensor_bytes(rt.name).tobytes()


def test_missing_keys_and_types_are_errors(pkg_mod, tmp_path):
    from synthesize_cpp_b200._abi import B200Q8Error

    path, _ = sample(tmp_path)
    with pkg_mod.Package(path) as p:
        for call in (lambda: p.get_u32("synthesize.test.nope"), lambda: p.get_u32("synthesize.test.eps"),
                     lambda: p.get_f32("synthesize.test.count"), lambda: p.get_str("synthesize.test.count")):
            with pytest.raises(B200Q8Error) as e:
                call()
            assert e.value.status == 1


def test_malformed_files_are_rejected(pkg_mod, tmp_path):
    from synthesize_cpp_b200._abi import B200Q8Error

    path, _ = sample(tmp_path)
    data = path.read_bytes()
    cases = {"truncated_data": data[:-40], "truncated_header": data[:60], "not_gguf": b"GGML" + data[4:],
             "version_1": data[:4] + (1).to_bytes(4, "little") + data[8:],
             "huge_count": data[:8] + (2**60).to_bytes(8, "little") + data[16:], "empty": b""}
    for name, blob in cases.items():
        bad = tmp_path / f"{name}.gguf"
        bad.write_bytes(blob)
        with pytest.raises(B200Q8Error) as e:
            pkg_mod.Package(bad)
        assert e.value.status == 1, name


def test_talker_chain_reports_missing_tensors_without_a_gpu(pkg_mod, tmp_path):
    # hyperparameters present, tensors absent: the loader fails on the first missing tensor before any CUDA call
    from synthesize_cpp_b200._abi import B200Q8Error

    p = "synthesize.qwen3-tts.talker."
    kv = {p + k: ("uint32", v) for k, v in [("layer_count", 1), ("hidden_size", 256), ("attention_head_count", 4),
                                               ("key_value_head_count", 2), ("head_dim", 64),
                                               ("intermediate_size", 512), ("codec_vocab_size", 64)]}
    kv[p + "rms_norm_eps"] = ("float32", 1e-6)
    path = tmp_path / "talker.gguf"
    write_package(path, kv, [("talker.model.norm.weight", np.ones(256, np.float32), None, None)])
    with pkg_mod.Package(path) as pk:
        with pytest.raises(B200Q8Error) as e:
            pk.talker_chain()
        assert e.value.status == 1


def _decoder_meta(p_hidden=256, with_pred=True):
    kv = {}
    t, pp = "synthesize.qwen3-tts.talker.", "synthesize.qwen3-tts.code_predictor."
    kv.update({t + "layer_count": ("uint32", 1), t + "hidden_size": ("uint32", 256),
               t + "attention_head_count": ("uint32", 4), t + "key_value_head_count": ("uint32", 2),
               t + "head_dim": ("uint32", 64), t + "intermediate_size": ("uint32", 512),
               t + "codec_vocab_size": ("uint32", 64), t + "rms_norm_eps": ("float32", 1e-6),
               t + "rope_theta": ("float32", 1e4), t + "code_group_count": ("uint32", 4)})
    if with_pred:
        kv.update({pp + "layer_count": ("uint32", 1), pp + "hidden_size": ("uint32", p_hidden),
                   pp + "attention_head_count": ("uint32", 4), pp + "key_value_head_count": ("uint32", 2),
                   pp + "head_dim": ("uint32", 64), pp + "vocab_size": ("uint32", 32),
                   pp + "code_group_count": ("uint32", 4)})
    return kv


@pytest.mark.parametrize("case,status", [("width", 1), ("no_predictor", 1)])
def test_decoder_refusals_before_any_upload(pkg_mod, tmp_path, case, status):
    """b200q8_gguf_decoder reports a predictor of another width without its small_to_mtp_projection tensors, and a
    package without the predictor's keys, as INVALID_ARG before touching a device."""
    import ctypes

    path = tmp_path / f"{case}.gguf"
    write_package(path, _decoder_meta(p_hidden=512 if case == "width" else 256, with_pred=case != "no_predictor"),
                  [("talker.model.norm.weight", np.ones(256, np.float32), None, None)])
    with pkg_mod.Package(path) as p:
        L = pkg_mod._bind()
        t, pr, f = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        st = L.b200q8_gguf_decoder(p._h, 0, 2, 0, 8, 2, ctypes.byref(t), ctypes.byref(pr), ctypes.byref(f))
        assert st == status
        assert not t.value and not pr.value and not f.value
