"""GGUF packages on the B200 Q8_0 path (include/b200q8_gguf.h) from Python.

The package reader the reference uses is ggml's (src/gguf-metadata.cpp:12-46);
this wraps the library's own bounds-checked reader and the talker step built
from a Qwen3-TTS package (hyperparameters of src/arch/qwen3-tts/weights.cpp:
128-138, tensor names of src/arch/qwen3-tts/catalog.cpp:239-281).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._abi import check, lib
from .q8 import QUANT_REF

# bytes per element (or per 32-element block for Q8_0) of the ggml types the reader sizes
_NP = {0: np.float32, 1: np.float16, 24: np.int8, 25: np.int16, 26: np.int32, 27: np.int64, 28: np.float64}


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int32), ("n_dims", ctypes.c_int32),
                ("ne", ctypes.c_int64 * 4), ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("data", ctypes.c_void_p)]


def _bind():
    L = lib()
    if getattr(L, "_gguf_bound", False):
        return L
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    L.b200q8_gguf_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
    L.b200q8_gguf_open.restype = i32
    L.b200q8_gguf_close.argtypes = [vp]
    L.b200q8_gguf_close.restype = None
    L.b200q8_gguf_tensor_count.argtypes = [vp]
    L.b200q8_gguf_tensor_count.restype = i64
    L.b200q8_gguf_find_tensor.argtypes = [vp, ctypes.c_char_p]
    L.b200q8_gguf_find_tensor.restype = i64
    L.b200q8_gguf_tensor.argtypes = [vp, i64, ctypes.POINTER(TensorInfo)]
    L.b200q8_gguf_tensor.restype = i32
    L.b200q8_gguf_get_u32.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)]
    L.b200q8_gguf_get_u32.restype = i32
    L.b200q8_gguf_get_f32.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float)]
    L.b200q8_gguf_get_f32.restype = i32
    L.b200q8_gguf_get_str.argtypes = [vp, ctypes.c_char_p, ctypes.c_char_p, sz]
    L.b200q8_gguf_get_str.restype = i32
    L.b200q8_gguf_talker_chain.argtypes = [vp, i32, i64, i32, ctypes.POINTER(vp)]
    L.b200q8_gguf_talker_chain.restype = i32
    L.b200q8_gguf_decoder.argtypes = [vp, i32, i64, i32, i64, i64, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                      ctypes.POINTER(vp)]
    L.b200q8_gguf_decoder.restype = i32
    L._gguf_bound = True
    return L


class Package:
    """An open GGUF file; tensor data stays memory-mapped until close()."""

    def __init__(self, path: str):
        L = _bind()
        h = ctypes.c_void_p()
        check(L.b200q8_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    def __len__(self) -> int:
        return int(_bind().b200q8_gguf_tensor_count(self._h))

    def find(self, name: str) -> int:
        return int(_bind().b200q8_gguf_find_tensor(self._h, name.encode()))

    def info(self, index_or_name) -> TensorInfo:
        i = self.find(index_or_name) if isinstance(index_or_name, str) else index_or_name
        t = TensorInfo()
        check(_bind().b200q8_gguf_tensor(self._h, i, ctypes.byref(t)))
        return t

    def tensor_bytes(self, index_or_name) -> np.ndarray:
        """The tensor's bytes (a copy out of the mapping)."""
        t = self.info(index_or_name)
        return np.ctypeslib.as_array(ctypes.cast(t.data, ctypes.POINTER(ctypes.c_uint8)), (t.nbytes,)).copy()

    def get_u32(self, key: str) -> int:
        v = ctypes.c_uint32()
        check(_bind().b200q8_gguf_get_u32(self._h, key.encode(), ctypes.byref(v)))
        return int(v.value)

    def get_f32(self, key: str) -> float:
        v = ctypes.c_float()
        check(_bind().b200q8_gguf_get_f32(self._h, key.encode(), ctypes.byref(v)))
        return float(v.value)

    def get_str(self, key: str, max_len: int = 4096) -> str:
        buf = ctypes.create_string_buffer(max_len)
        check(_bind().b200q8_gguf_get_str(self._h, key.encode(), buf, max_len))
        return buf.value.decode()

    def talker_chain(self, device: int = 0, max_m: int = 8, mode: int = QUANT_REF):
        """The package's talker decode step on `device` (a chain.DecodeChain)."""
        from .chain import DecodeChain

        p = "synthesize.qwen3-tts.talker."
        h = ctypes.c_void_p()
        check(_bind().b200q8_gguf_talker_chain(self._h, device, max_m, mode, ctypes.byref(h)))
        return DecodeChain.from_handle(h, hidden=self.get_u32(p + "hidden_size"),
                                       n_layers=self.get_u32(p + "layer_count"),
                                       device=torch.device("cuda", device))

    def decoder(self, device: int = 0, max_m: int = 8, n_ctx: int = 4096, n_slots: int = 8,
                mode: int = QUANT_REF):
        """(talker, predictor, frame): the package's talker step with attention and codec head, its code predictor
        and the decode frame over both (b200q8_gguf_decoder)."""
        from .chain import DecodeChain
        from .frame import Frame

        t, pr, f = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        check(_bind().b200q8_gguf_decoder(self._h, device, max_m, mode, n_ctx, n_slots, ctypes.byref(t),
                                          ctypes.byref(pr), ctypes.byref(f)))
        dev = torch.device("cuda", device)
        tp, pp = "synthesize.qwen3-tts.talker.", "synthesize.qwen3-tts.code_predictor."
        talker = DecodeChain.from_handle(t, hidden=self.get_u32(tp + "hidden_size"),
                                         n_layers=self.get_u32(tp + "layer_count"), device=dev)
        talker.vocab = self.get_u32(tp + "codec_vocab_size")
        predictor = DecodeChain.from_handle(pr, hidden=self.get_u32(pp + "hidden_size"),
                                            n_layers=self.get_u32(pp + "layer_count"), device=dev)
        predictor.vocab = self.get_u32(pp + "vocab_size")
        frame = Frame.from_handle(f, talker, predictor, groups=self.get_u32(tp + "code_group_count"))
        return talker, predictor, frame

    def close(self) -> None:
        if self._h:
            _bind().b200q8_gguf_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
