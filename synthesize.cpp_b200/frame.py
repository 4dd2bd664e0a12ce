"""One decode frame of Qwen3-TTS (talker + code predictor) on the device (b200q8_frame_*).

Mirrors the reference's per-frame loop (src/arch/qwen3-tts/model.cpp:1310-1489) with greedy selection
(request.sample == false) or replayed codes: one run() is the talker step and the code predictor's
code_group_count - 1 calls for M streams, replayed as one CUDA graph.
"""
from __future__ import annotations

import ctypes

import torch

from ._abi import FrameArgs, FrameDesc, check, lib
from .chain import DecodeChain
from .q8 import stream_ptr


class Frame:
    """talker / predictor: DecodeChain objects built with attention and output descs; tables: the predictor's
    G-1 codec tables (uint8 Q8_0 [rows, hidden/32*34] CUDA tensors)."""

    def __init__(self, talker: DecodeChain, predictor: DecodeChain, tables: list[torch.Tensor], *,
                 repetition_penalty: float = 1.0, projection: tuple[torch.Tensor, torch.Tensor] | None = None,
                 text_projection: dict | None = None):
        """projection: (W uint8 Q8_0 [predictor hidden, talker hidden/32*34], bias float32 [predictor hidden]) for a
        predictor narrower than the talker.  text_projection: dict(embedding=uint8 Q8_0 [text rows, text hidden/32*34],
        fc1=uint8 Q8_0 [text hidden, text hidden/32*34], fc1_bias=float32 [text hidden], fc2=uint8 Q8_0 [talker
        hidden, text hidden/32*34], fc2_bias=float32 [talker hidden]) for frames run from text token ids."""
        self._keep = (talker, predictor, tables, projection, text_projection)
        self.groups = len(tables) + 1
        arr = (ctypes.c_void_p * len(tables))(*[t.data_ptr() for t in tables])
        pw, pb = (projection[0].data_ptr(), projection[1].data_ptr()) if projection is not None else (None, None)
        tp = text_projection
        text = (None, 0, 0, None, None, None, None) if tp is None else (
            tp["embedding"].data_ptr(), tp["embedding"].shape[0], tp["embedding"].shape[1] // 34 * 32,
            tp["fc1"].data_ptr(), tp["fc1_bias"].data_ptr(), tp["fc2"].data_ptr(), tp["fc2_bias"].data_ptr())
        desc = FrameDesc(talker._h, predictor._h, self.groups, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)),
                         tables[0].shape[0], repetition_penalty, pw, pb, *text)
        handle = ctypes.c_void_p()
        check(lib().b200q8_frame_create(ctypes.byref(desc), ctypes.byref(handle)))
        self._h = handle

    @classmethod
    def from_handle(cls, handle: ctypes.c_void_p, talker: DecodeChain, predictor: DecodeChain, *,
                    groups: int) -> "Frame":
        """Wraps a frame the library already built (b200q8_gguf_decoder); keeps the chains alive while it lives."""
        self = cls.__new__(cls)
        self._keep = (talker, predictor)
        self.groups = groups
        self._h = handle
        return self

    def run(self, codes: torch.Tensor, *, text: torch.Tensor | None = None, prev: torch.Tensor | None = None,
            pos: torch.Tensor | None = None, slots: torch.Tensor | None = None, replay: torch.Tensor | None = None,
            hidden: torch.Tensor | None = None, talker_logits: torch.Tensor | None = None,
            skip_talker: bool = False, text_ids: torch.Tensor | None = None) -> torch.Tensor:
        """codes: int32 [M, G] out.  Without skip_talker: text [M, hidden] (or text_ids int32 [M] through the
        frame's text projection), prev [M, G], pos [M]."""
        p = lambda t: t.data_ptr() if t is not None else None
        a = FrameArgs(codes.shape[0], 1 if skip_talker else 0, p(text), p(prev), p(pos), p(slots), p(replay),
                      p(codes), p(hidden), p(talker_logits), p(text_ids))
        check(lib().b200q8_frame_run(self._h, ctypes.byref(a), stream_ptr()))
        return codes

    def text_rows(self, text_ids: torch.Tensor, out: torch.Tensor, h1: torch.Tensor | None = None) -> torch.Tensor:
        """The talker's text rows for text token ids through the frame's text projection (b200q8_frame_text_rows):
        out float32 [M, hidden]; h1 (optional) float32 [M, text hidden] gets silu(fc1(.) + b1)."""
        check(lib().b200q8_frame_text_rows(self._h, text_ids.data_ptr(), text_ids.numel(),
                                           h1.data_ptr() if h1 is not None else None, out.data_ptr(), stream_ptr()))
        return out

    def reset_history(self, slot: int = -1) -> None:
        check(lib().b200q8_frame_reset_history(self._h, slot, stream_ptr()))

    def close(self) -> None:
        if self._h:
            lib().b200q8_frame_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
