"""ctypes binding of libb200q8.so (include/b200q8.h).

The product path: every call goes through the C ABI into the sm_100a kernels.
There is no fallback: if the library is missing or cannot be loaded, calls
raise.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libb200q8.so")
HEADER = os.path.join(ROOT, "include", "b200q8.h")

OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 8
ERR_OOM = 16
ERR_BACKEND = 17
ERR_INTERNAL = 20
ERR_DEVICE_TIMEOUT = 21

QUANT_REF = 0
QUANT_CPU_X86 = 1
QUANT_CPU_ARM = 2

_lib: ctypes.CDLL | None = None


class B200Q8Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"b200q8 status {status}: {message}")
        self.status = status


class Layer(ctypes.Structure):
    _fields_ = [("wq", ctypes.c_void_p), ("wk", ctypes.c_void_p), ("wv", ctypes.c_void_p),
                ("wo", ctypes.c_void_p), ("wgate", ctypes.c_void_p), ("wup", ctypes.c_void_p),
                ("wdown", ctypes.c_void_p), ("norm_in", ctypes.c_void_p), ("norm_post", ctypes.c_void_p)]


class AttentionDesc(ctypes.Structure):
    _fields_ = [("rope_theta", ctypes.c_float), ("n_ctx", ctypes.c_int64), ("n_slots", ctypes.c_int64),
                ("q_norm", ctypes.POINTER(ctypes.c_void_p)), ("k_norm", ctypes.POINTER(ctypes.c_void_p))]


class OutputDesc(ctypes.Structure):
    _fields_ = [("norm", ctypes.c_void_p), ("heads", ctypes.POINTER(ctypes.c_void_p)), ("n_heads", ctypes.c_int32),
                ("vocab", ctypes.c_int64)]


class ChainDesc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("hidden", ctypes.c_int64), ("n_head", ctypes.c_int64),
                ("n_kv", ctypes.c_int64), ("head_dim", ctypes.c_int64), ("inter", ctypes.c_int64),
                ("eps", ctypes.c_float), ("max_m", ctypes.c_int64), ("mode", ctypes.c_int32),
                ("layers", ctypes.POINTER(Layer)), ("table", ctypes.c_void_p), ("table_rows", ctypes.c_int64),
                ("attention", ctypes.POINTER(AttentionDesc)), ("output", ctypes.POINTER(OutputDesc))]


class StepArgs(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("ids", ctypes.c_void_p), ("table", ctypes.c_void_p),
                ("table_rows", ctypes.c_int64), ("x_in", ctypes.c_void_p), ("pos", ctypes.c_void_p),
                ("slots", ctypes.c_void_p), ("h_out", ctypes.c_void_p), ("hidden_out", ctypes.c_void_p),
                ("logits", ctypes.c_void_p), ("head", ctypes.c_int32)]


class FrameDesc(ctypes.Structure):
    _fields_ = [("talker", ctypes.c_void_p), ("predictor", ctypes.c_void_p), ("groups", ctypes.c_int32),
                ("tables", ctypes.POINTER(ctypes.c_void_p)), ("table_rows", ctypes.c_int64),
                ("repetition_penalty", ctypes.c_float), ("input_projection", ctypes.c_void_p),
                ("input_projection_bias", ctypes.c_void_p), ("text_embedding", ctypes.c_void_p),
                ("text_rows", ctypes.c_int64), ("text_hidden", ctypes.c_int64), ("text_fc1", ctypes.c_void_p),
                ("text_fc1_bias", ctypes.c_void_p), ("text_fc2", ctypes.c_void_p), ("text_fc2_bias", ctypes.c_void_p)]


class FrameArgs(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("skip_talker", ctypes.c_int32), ("text", ctypes.c_void_p),
                ("prev", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("slots", ctypes.c_void_p),
                ("replay", ctypes.c_void_p), ("codes", ctypes.c_void_p), ("hidden", ctypes.c_void_p),
                ("talker_logits", ctypes.c_void_p), ("text_ids", ctypes.c_void_p)]


def header_symbols(header: str = HEADER) -> list[str]:
    """Every function a public header declares."""
    text = open(header).read()
    return sorted(set(re.findall(r"^\S[^\n;]*?\b(b200q8h?_\w+)\s*\(", text, flags=re.M)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run __graft_entry__.build() (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    L.b200q8_version.restype = i32
    L.b200q8_last_error.argtypes = [ctypes.c_char_p, sz]
    L.b200q8_last_error.restype = i32
    L.b200q8_device_status.argtypes = [i32, i32]
    L.b200q8_device_status.restype = i32
    L.b200q8_quantize_rows.argtypes = [vp, i64, i64, sz, vp, sz, i32, vp]
    L.b200q8_quantize_rows.restype = i32
    L.b200q8_quantize_chunk.argtypes = [vp, vp, i64, i64, i64, ctypes.POINTER(sz), vp]
    L.b200q8_quantize_chunk.restype = i32
    L.b200q8_quantize_chunk_host.argtypes = [vp, vp, i64, i64, i64, ctypes.POINTER(sz), i32]
    L.b200q8_quantize_chunk_host.restype = i32
    L.b200q8_quantize_rows_typed.argtypes = [vp, i32, i64, i64, sz, vp, sz, i32, vp]
    L.b200q8_quantize_rows_typed.restype = i32
    L.b200q8_quantize_chunk_host_typed.argtypes = [vp, i32, vp, i64, i64, i64, ctypes.POINTER(sz), i32]
    L.b200q8_quantize_chunk_host_typed.restype = i32
    L.b200q8_chain_inject_epoch_skew.argtypes = [vp, i32]
    L.b200q8_chain_inject_epoch_skew.restype = i32
    L.b200q8_quantize_chunk_host_release.argtypes = []
    L.b200q8_quantize_chunk_host_release.restype = None
    L.b200q8_dequantize_rows.argtypes = [vp, i64, i64, sz, vp, sz, vp]
    L.b200q8_dequantize_rows.restype = i32
    L.b200q8_get_rows.argtypes = [vp, i64, i64, sz, vp, i64, vp, sz, vp]
    L.b200q8_get_rows.restype = i32
    L.b200q8_mul_mat_workspace_size.argtypes = [i64, i64, i64]
    L.b200q8_mul_mat_workspace_size.restype = sz
    L.b200q8_mul_mat.argtypes = [vp, i64, i64, sz, vp, i64, sz, vp, sz, i32, vp, sz, vp]
    L.b200q8_mul_mat.restype = i32
    L.b200q8_mul_mat_noalloc.argtypes = [vp, i64, i64, sz, vp, i64, sz, vp, sz, i32, vp]
    L.b200q8_mul_mat_noalloc.restype = i32
    L.b200q8_chain_create.argtypes = [ctypes.POINTER(ChainDesc), i32, ctypes.POINTER(vp)]
    L.b200q8_chain_create.restype = i32
    L.b200q8_chain_run.argtypes = [vp, vp, vp, vp, i64, vp]
    L.b200q8_chain_run.restype = i32
    L.b200q8_chain_run_at.argtypes = [vp, vp, vp, vp, vp, vp, i64, vp]
    L.b200q8_chain_run_at.restype = i32
    L.b200q8_chain_buffer.argtypes = [vp, i32, i32, ctypes.POINTER(vp), ctypes.POINTER(i64)]
    L.b200q8_chain_buffer.restype = i32
    L.b200q8_chain_destroy.argtypes = [vp]
    L.b200q8_chain_destroy.restype = None
    L.b200q8_chain_step.argtypes = [vp, ctypes.POINTER(StepArgs), vp]
    L.b200q8_chain_step.restype = i32
    L.b200q8_frame_create.argtypes = [ctypes.POINTER(FrameDesc), ctypes.POINTER(vp)]
    L.b200q8_frame_create.restype = i32
    L.b200q8_frame_run.argtypes = [vp, ctypes.POINTER(FrameArgs), vp]
    L.b200q8_frame_run.restype = i32
    L.b200q8_frame_text_rows.argtypes = [vp, vp, i64, vp, vp, vp]
    L.b200q8_frame_text_rows.restype = i32
    L.b200q8_frame_reset_history.argtypes = [vp, i32, vp]
    L.b200q8_frame_reset_history.restype = i32
    L.b200q8_frame_destroy.argtypes = [vp]
    L.b200q8_frame_destroy.restype = None
    _lib = L
    return L


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(1024)
    code = lib().b200q8_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        _, msg = last_error()
        raise B200Q8Error(status, msg)
