"""The Q8_0 ops of synthesize.cpp's hot path on B200, over the C ABI.

Names, argument meaning and error behaviour follow the ggml calls the
reference makes on this path:

* ``mul_mat(w, x)``           ggml_mul_mat(Q8_0 W, F32 x)
                              (src/arch/qwen3-tts/operations.cpp:39-41,90-92,142)
* ``get_rows(table, ids)``    ggml_get_rows(Q8_0 table, I32 ids)
                              (talker.cpp:44,86, code-predictor.cpp:31)
* ``quantize_chunk(...)``     ggml_quantize_chunk(GGML_TYPE_Q8_0, ...)
                              (tools/synthesize-quantize/quantize.cpp:300-301)
* ``quantize_rows`` / ``dequantize_rows``  the Q8_0 type traits' from_float /
                              to_float (quantize.cpp:67-83)

Tensors are torch CUDA tensors in ggml's memory order: a Q8_0 matrix with
ne = [K, N] is a uint8 tensor [N, K/32*34]; F32 activations with ne = [K, M]
are float32 [M, K] (rows may be strided); results are [M, N].  Work is
enqueued on torch's current stream.  Every call goes through
libb200q8.so; a failure raises B200Q8Error with the library's message.
"""
from __future__ import annotations

import ctypes

import torch

from ._abi import QUANT_CPU_ARM, QUANT_CPU_X86, QUANT_REF, B200Q8Error, check, lib

QK = 32
BLOCK_BYTES = 34

__all__ = ["QK", "BLOCK_BYTES", "QUANT_REF", "QUANT_CPU_X86", "QUANT_CPU_ARM", "B200Q8Error", "row_bytes",
           "quantize_rows", "quantize_chunk", "quantize_chunk_host", "quantize_chunk_host_typed", "quantize_chunk_host_release", "dequantize_rows", "get_rows", "mul_mat", "workspace_size",
           "device_status", "stream_ptr"]


def row_bytes(k: int) -> int:
    return k // QK * BLOCK_BYTES


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("b200q8 ops take CUDA tensors (no CPU path exists)")


def _row_stride_bytes(t: torch.Tensor) -> int:
    return (t.stride(0) if t.dim() > 1 else t.shape[-1]) * t.element_size()


SRC_TYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 30}  # ggml type ids


def quantize_rows(x: torch.Tensor, mode: int = QUANT_REF, out: torch.Tensor | None = None) -> torch.Tensor:
    """F32 / F16 / BF16 [rows, K] -> Q8_0 uint8 [rows, K/32*34] (16-bit values widened to fp32 exactly)."""
    _need_cuda(x)
    if x.dtype not in SRC_TYPES or x.stride(-1) != 1:
        raise ValueError("quantize_rows: x must be float32, float16 or bfloat16 with unit inner stride")
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    rows, k = x2.shape
    if out is None:
        out = torch.empty((rows, row_bytes(k)), dtype=torch.uint8, device=x.device)
    if x.dtype == torch.float32:
        check(lib().b200q8_quantize_rows(x2.data_ptr(), rows, k, _row_stride_bytes(x2), out.data_ptr(),
                                         _row_stride_bytes(out), mode, stream_ptr()))
    else:
        check(lib().b200q8_quantize_rows_typed(x2.data_ptr(), SRC_TYPES[x.dtype], rows, k, _row_stride_bytes(x2),
                                               out.data_ptr(), _row_stride_bytes(out), mode, stream_ptr()))
    return out


def quantize_chunk(src: torch.Tensor, dst: torch.Tensor, start: int, nrows: int, n_per_row: int) -> int:
    """ggml_quantize_chunk(Q8_0, src, dst, start, nrows, n_per_row, NULL); returns bytes written."""
    _need_cuda(src, dst)
    written = ctypes.c_size_t(0)
    check(lib().b200q8_quantize_chunk(src.data_ptr(), dst.data_ptr(), start, nrows, n_per_row,
                                      ctypes.byref(written), stream_ptr()))
    return int(written.value)


def quantize_chunk_host(src, dst, start: int, nrows: int, n_per_row: int, device: int = 0) -> int:
    """ggml_quantize_chunk(Q8_0, ...) on host numpy/torch-CPU buffers (the quantize tool's call); returns bytes written."""
    import numpy as np

    def ptr(a):
        return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()

    written = ctypes.c_size_t(0)
    check(lib().b200q8_quantize_chunk_host(ptr(src), ptr(dst), start, nrows, n_per_row, ctypes.byref(written), device))
    return int(written.value)


def quantize_chunk_host_typed(src, dst, start: int, nrows: int, n_per_row: int, device: int = 0) -> int:
    """quantize_chunk_host for an F32 / F16 / BF16 host source (numpy float32/float16 array, or a CPU torch
    tensor of float32/float16/bfloat16); returns bytes written."""
    import numpy as np

    if isinstance(src, np.ndarray):
        st = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}[src.dtype]
        sp = src.ctypes.data
    else:
        st = SRC_TYPES[src.dtype]
        sp = src.data_ptr()
    dp = dst.ctypes.data if isinstance(dst, np.ndarray) else dst.data_ptr()
    written = ctypes.c_size_t(0)
    check(lib().b200q8_quantize_chunk_host_typed(sp, st, dp, start, nrows, n_per_row, ctypes.byref(written), device))
    return int(written.value)


def quantize_chunk_host_release() -> None:
    """Frees the pinned and device staging quantize_chunk_host keeps between calls."""
    lib().b200q8_quantize_chunk_host_release()


def dequantize_rows(q: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(q)
    rows = q.shape[0]
    if out is None:
        out = torch.empty((rows, k), dtype=torch.float32, device=q.device)
    check(lib().b200q8_dequantize_rows(q.data_ptr(), rows, k, _row_stride_bytes(q), out.data_ptr(),
                                       _row_stride_bytes(out), stream_ptr()))
    return out


def get_rows(table: torch.Tensor, k: int, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_get_rows(Q8_0 table [rows, K/32*34], I32 ids [n]) -> F32 [n, K]."""
    _need_cuda(table, ids)
    if ids.dtype != torch.int32:
        raise ValueError("get_rows: ids must be int32 (GGML_TYPE_I32)")
    n = ids.numel()
    if out is None:
        out = torch.empty((n, k), dtype=torch.float32, device=table.device)
    check(lib().b200q8_get_rows(table.data_ptr(), k, table.shape[0], _row_stride_bytes(table), ids.data_ptr(), n,
                                out.data_ptr(), _row_stride_bytes(out), stream_ptr()))
    return out


def workspace_size(k: int, n: int, m: int) -> int:
    return int(lib().b200q8_mul_mat_workspace_size(k, n, m))


def mul_mat(w: torch.Tensor, k: int, x: torch.Tensor, mode: int = QUANT_REF, out: torch.Tensor | None = None,
            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """ggml_mul_mat(Q8_0 W [N, K/32*34], F32 x [M, K]) -> F32 [M, N]."""
    _need_cuda(w, x)
    if x.dtype != torch.float32 or x.stride(-1) != 1:
        raise ValueError("mul_mat: x must be float32 with unit inner stride")
    x2 = x.reshape(-1, k) if x.dim() != 2 else x
    m = x2.shape[0]
    n = w.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    need = workspace_size(k, n, m)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib().b200q8_mul_mat(w.data_ptr(), k, n, _row_stride_bytes(w), x2.data_ptr(), m, _row_stride_bytes(x2),
                               out.data_ptr(), _row_stride_bytes(out), mode,
                               workspace.data_ptr() if workspace is not None else None,
                               workspace.numel() if workspace is not None else 0, stream_ptr()))
    return out


def device_status(device: int = 0, clear: bool = True) -> int:
    """Synchronises the device and returns (and by default clears) its kernel status word."""
    return int(lib().b200q8_device_status(device, 1 if clear else 0))

