"""The talker-shaped decode step (b200q8_chain_*) from Python.

Mirrors the caller side of the reference's per-frame talker step
(src/arch/qwen3-tts/talker.cpp:135-185 build_talker_step, computed through
model.cpp:101-126 GraphRun::run): weights stay resident on the device, each
run() is one step for M tokens.
"""
from __future__ import annotations

import ctypes

import torch

from ._abi import AttentionDesc, ChainDesc, Layer, OutputDesc, StepArgs, check, lib
from .q8 import QUANT_REF, stream_ptr

BUFFERS = {"n1": 0, "qkv": 1, "attn": 2, "o": 3, "h1": 4, "n2": 5, "gu": 6, "s": 7, "down": 8, "h": 9}


class DecodeChain:
    """layers: list of dicts with torch CUDA tensors wq, wk, wv, wo, wgate, wup, wdown (uint8 Q8_0 rows) and
    norm_in, norm_post (float32 [hidden]); table: uint8 Q8_0 [table_rows, hidden/32*34]."""

    def __init__(self, layers, table: torch.Tensor, *, hidden: int, n_head: int, n_kv: int, head_dim: int,
                 inter: int, eps: float = 1e-6, max_m: int = 8, mode: int = QUANT_REF, attention: dict | None = None,
                 output: dict | None = None):
        """attention: None for the single-cached-position step, or dict(rope_theta, n_ctx, n_slots) with each layer
        dict also holding q_norm and k_norm (float32 [head_dim]); such a chain runs through run_at / step.
        output: None, or dict(norm=float32 [hidden], heads=[uint8 Q8_0 [vocab, hidden/32*34], ...]): the final
        RMS norm and the heads step() applies."""
        self._keep = (layers, table)
        arr = (Layer * len(layers))()
        for i, L in enumerate(layers):
            arr[i] = Layer(*[L[k].data_ptr() for k in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown",
                                                       "norm_in", "norm_post")])
        self._arr = arr
        attn_ptr = None
        if attention is not None:
            qn = (ctypes.c_void_p * len(layers))(*[L["q_norm"].data_ptr() for L in layers])
            kn = (ctypes.c_void_p * len(layers))(*[L["k_norm"].data_ptr() for L in layers])
            self._attn = (AttentionDesc(attention["rope_theta"], attention["n_ctx"], attention["n_slots"],
                                        ctypes.cast(qn, ctypes.POINTER(ctypes.c_void_p)),
                                        ctypes.cast(kn, ctypes.POINTER(ctypes.c_void_p))), qn, kn)
            attn_ptr = ctypes.pointer(self._attn[0])
        out_ptr = None
        self.vocab = 0
        if output is not None:
            heads = (ctypes.c_void_p * len(output["heads"]))(*[h.data_ptr() for h in output["heads"]])
            self.vocab = output["heads"][0].shape[0]
            self._out = (OutputDesc(output["norm"].data_ptr(), ctypes.cast(heads, ctypes.POINTER(ctypes.c_void_p)),
                                    len(output["heads"]), self.vocab), heads, output)
            out_ptr = ctypes.pointer(self._out[0])
        desc = ChainDesc(len(layers), hidden, n_head, n_kv, head_dim, inter, eps, max_m, mode,
                         ctypes.cast(arr, ctypes.POINTER(Layer)), table.data_ptr(), table.shape[0], attn_ptr, out_ptr)
        handle = ctypes.c_void_p()
        check(lib().b200q8_chain_create(ctypes.byref(desc), table.device.index or 0, ctypes.byref(handle)))
        self._h = handle
        self.hidden = hidden
        self.n_layers = len(layers)
        self.device = table.device

    @classmethod
    def from_handle(cls, handle: ctypes.c_void_p, *, hidden: int, n_layers: int, device: torch.device,
                    keep=None) -> "DecodeChain":
        """Wraps a chain the library already built (b200q8_gguf_talker_chain)."""
        self = cls.__new__(cls)
        self._keep = keep
        self._arr = None
        self._h = handle
        self.hidden = hidden
        self.n_layers = n_layers
        self.device = device
        return self

    def run(self, ids: torch.Tensor, x_in: torch.Tensor, h_out: torch.Tensor) -> torch.Tensor:
        m = ids.numel()
        check(lib().b200q8_chain_run(self._h, ids.data_ptr(), x_in.data_ptr(), h_out.data_ptr(), m, stream_ptr()))
        return h_out

    def run_at(self, ids: torch.Tensor, x_in: torch.Tensor, pos: torch.Tensor, h_out: torch.Tensor,
               slots: torch.Tensor | None = None) -> torch.Tensor:
        """One step with attention: token m at position pos[m] of stream slot slots[m] (default slot m)."""
        m = ids.numel()
        check(lib().b200q8_chain_run_at(self._h, ids.data_ptr(), x_in.data_ptr(), pos.data_ptr(),
                                        slots.data_ptr() if slots is not None else None, h_out.data_ptr(), m,
                                        stream_ptr()))
        return h_out

    def step(self, *, ids: torch.Tensor | None = None, x_in: torch.Tensor | None = None,
             table: torch.Tensor | None = None, pos: torch.Tensor | None = None, slots: torch.Tensor | None = None,
             h_out: torch.Tensor | None = None, hidden_out: torch.Tensor | None = None,
             logits: torch.Tensor | None = None, head: int = 0, m: int | None = None) -> None:
        """b200q8_chain_step: h0 = x_in + table[ids] (either may be absent), the layers, then the output stage into
        hidden_out / logits when either is given."""
        if m is None:
            m = ids.numel() if ids is not None else x_in.shape[0]
        p = lambda t: t.data_ptr() if t is not None else None
        a = StepArgs(m, p(ids), p(table), table.shape[0] if table is not None else 0, p(x_in), p(pos), p(slots),
                     p(h_out), p(hidden_out), p(logits), head)
        check(lib().b200q8_chain_step(self._h, ctypes.byref(a), stream_ptr()))

    def buffer(self, layer: int, name: str, m: int) -> torch.Tensor:
        """A copy of one activation buffer of the last run, [m, width] float32 on the device."""
        ptr = ctypes.c_void_p()
        stride = ctypes.c_int64()
        check(lib().b200q8_chain_buffer(self._h, layer, BUFFERS[name], ctypes.byref(ptr), ctypes.byref(stride)))

        class _View:
            __cuda_array_interface__ = {"shape": (m, stride.value), "typestr": "<f4", "data": (ptr.value, False),
                                        "version": 3, "strides": None}

        return torch.as_tensor(_View(), device=self.device).clone()

    def close(self) -> None:
        if self._h:
            lib().b200q8_chain_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
