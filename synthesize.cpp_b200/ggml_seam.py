"""The ggml-backend seam (include/b200q8_ggml.h) from Python: descriptors
mirroring ggml_tensor for MUL_MAT / GET_ROWS nodes, supports_op and
graph_compute over libb200q8_host.so."""
from __future__ import annotations

import ctypes

import torch

from . import host
from ._abi import check
from .q8 import stream_ptr

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_I32 = 0, 1, 8, 26
OP_NONE, OP_MUL_MAT, OP_GET_ROWS = 0, 1, 2


class GgmlTensor(ctypes.Structure):
    pass


GgmlTensor._fields_ = [("type", ctypes.c_int32), ("op", ctypes.c_int32), ("ne", ctypes.c_int64 * 4),
                       ("nb", ctypes.c_size_t * 4), ("data", ctypes.c_void_p),
                       ("src", ctypes.POINTER(GgmlTensor) * 2)]

_bound = False


def lib() -> ctypes.CDLL:
    global _bound
    L = host.lib()
    if not _bound:
        P = ctypes.POINTER(GgmlTensor)
        L.b200q8_ggml_supports_op.argtypes = [P]
        L.b200q8_ggml_supports_op.restype = ctypes.c_int32
        L.b200q8_ggml_workspace_size.argtypes = [P]
        L.b200q8_ggml_workspace_size.restype = ctypes.c_size_t
        L.b200q8_ggml_compute_node.argtypes = [P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_void_p]
        L.b200q8_ggml_compute_node.restype = ctypes.c_int32
        L.b200q8_ggml_graph_compute.argtypes = [ctypes.POINTER(P), ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t,
                                                ctypes.c_int32, ctypes.c_void_p]
        L.b200q8_ggml_graph_compute.restype = ctypes.c_int32
        _bound = True
    return L


def tensor(type_: int, ne, nb, data: int = 0, op: int = OP_NONE, src=(None, None)) -> GgmlTensor:
    """A descriptor with ggml's ne (innermost first) and byte strides nb."""
    ne = list(ne) + [1] * (4 - len(ne))
    nb = list(nb) + [nb[-1] * ne[len(nb) - 1]] * (4 - len(nb)) if len(nb) < 4 else list(nb)
    t = GgmlTensor()
    t.type, t.op, t.data = type_, op, data
    for i in range(4):
        t.ne[i] = ne[i]
        t.nb[i] = nb[i]
    for i, s in enumerate(src):
        t.src[i] = ctypes.pointer(s) if s is not None else ctypes.POINTER(GgmlTensor)()
    return t


def q8_tensor(t: torch.Tensor, k: int) -> GgmlTensor:
    """Q8_0 uint8 tensor [..., rows, k/32*34] -> descriptor ne = [k, rows, ...]."""
    shape = list(t.shape)
    rows = shape[-2] if len(shape) >= 2 else 1
    outer = list(reversed(shape[:-2]))
    ne = [k, rows] + outer
    nb = [34, t.stride(-2)] + [t.stride(d) for d in reversed(range(len(shape) - 2))]
    return tensor(TYPE_Q8_0, ne, nb, t.data_ptr())


def dense_tensor(t: torch.Tensor, type_: int) -> GgmlTensor:
    """A row-major torch tensor [..., d1, d0] -> descriptor ne = [d0, d1, ...]."""
    es = t.element_size()
    ne = list(reversed(t.shape))
    nb = [t.stride(d) * es for d in reversed(range(t.dim()))]
    return tensor(type_, ne, nb, t.data_ptr())


def supports_op(node: GgmlTensor) -> bool:
    return bool(lib().b200q8_ggml_supports_op(ctypes.byref(node)))


def compute(node: GgmlTensor, mode: int = 0, workspace: torch.Tensor | None = None) -> None:
    L = lib()
    need = L.b200q8_ggml_workspace_size(ctypes.byref(node))
    if workspace is None and need:
        workspace = torch.empty(need, dtype=torch.uint8, device="cuda")
    check(L.b200q8_ggml_compute_node(ctypes.byref(node), workspace.data_ptr() if workspace is not None else None,
                                     workspace.numel() if workspace is not None else 0, mode, stream_ptr()))
