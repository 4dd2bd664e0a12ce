"""Synthetic Qwen3-TTS-shaped Q8_0 models on the device.

Weights are 0.02 * N(0,1) from the seeded normal stream (one seed per
tensor: base + 16*layer + index, index 0..6 = q,k,v,o,gate,up,down; 8 and 9
are the two RMS-norm weight vectors, 1 + 0.1 * N(0,1)), packed to Q8_0 on the
GPU by b200q8_quantize_rows.  Each layer's q|k|v and gate|up rows are laid
out contiguously, which is the layout the step chain streams without a copy.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import host
from .q8 import quantize_rows, row_bytes
from .shapes import (OUTLIER_SCALE, PREDICTOR_06B, STREAM_SEED, TALKER_06B, TALKER_17B, Shape,  # noqa: F401
                     outlier_positions, stream_ids)


@dataclass
class DeviceModel:
    shape: Shape
    layers: list = field(default_factory=list)  # dicts of torch tensors (views into blocks)
    blocks: list = field(default_factory=list)  # owning tensors
    table: torch.Tensor | None = None


def build_model(shape: Shape, device: torch.device, seed: int = 1000, threads: int = 0) -> DeviceModel:
    dm = DeviceModel(shape)
    mats = shape.matrices()
    H = shape.hidden
    for l in range(shape.n_layers):
        f32 = [np.empty(n * k, np.float32) for n, k in mats]
        norms = [np.empty(H, np.float32) for _ in range(2)]
        host.normal_many([seed + 16 * l + j for j in range(7)] + [seed + 16 * l + 8, seed + 16 * l + 9],
                         [0.02] * 7 + [0.1, 0.1], f32 + norms, threads)
        # q|k|v in one block, gate|up in one block, o and down alone
        groups = [(0, 1, 2), (3,), (4, 5), (6,)]
        views = {}
        for g in groups:
            k = mats[g[0]][1]
            rows = sum(mats[j][0] for j in g)
            blk = torch.empty((rows, row_bytes(k)), dtype=torch.uint8, device=device)
            dm.blocks.append(blk)
            r = 0
            for j in g:
                n = mats[j][0]
                src = torch.from_numpy(f32[j].reshape(n, k)).to(device)
                quantize_rows(src, out=blk[r:r + n])
                views[j] = blk[r:r + n]
                r += n
        keys = ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown")
        L = {key: views[j] for j, key in enumerate(keys)}
        L["norm_in"] = torch.from_numpy(1.0 + norms[0]).to(device)
        L["norm_post"] = torch.from_numpy(1.0 + norms[1]).to(device)
        dm.layers.append(L)
    tab = host.normal(seed - 1, shape.table_rows * H, 0.02).reshape(shape.table_rows, H)
    dm.table = quantize_rows(torch.from_numpy(tab).to(device))
    torch.cuda.synchronize(device)
    return dm


def stream_inputs(m: int, hidden: int, table_rows: int, first_stream: int = 0, seed: int = STREAM_SEED,
                  outliers: bool = False):
    """Per-stream N(0,1) activations (stream s from seed + s) and token ids; with outliers, the 1 % of entries
    shapes.outlier_positions names are scaled by 20."""
    x = np.stack([host.normal(seed + first_stream + s, hidden) for s in range(m)]).astype(np.float32)
    if outliers:
        x.reshape(-1)[outlier_positions(m, hidden, first_stream)] *= np.float32(OUTLIER_SCALE)
    ids = np.asarray(stream_ids(m, table_rows, first_stream), dtype=np.int32)
    return x, ids


def host_copy(dm: DeviceModel):
    """Host (numpy) copies of every Q8_0 matrix in oracle order, the norms and the table."""
    mats, norms = [], []
    for L in dm.layers:
        for key in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown"):
            mats.append(L[key].cpu().numpy())
        norms.append(L["norm_in"].cpu().numpy())
        norms.append(L["norm_post"].cpu().numpy())
    return mats, np.stack(norms), dm.table.cpu().numpy()


# ---------------------------------------------------------------- decode frame

@dataclass
class FrameShape:
    """One Qwen3-TTS decode frame: the talker step with its codec head, then groups - 1 code-predictor calls
    (src/arch/qwen3-tts/model.cpp:1310-1489); 0.6B package shapes."""
    talker: Shape
    predictor: Shape
    groups: int = 16
    talker_vocab: int = 3072
    predictor_vocab: int = 2048
    rope_theta: float = 1.0e6

    def weight_bytes(self) -> int:
        H = self.talker.hidden
        head_t = self.talker_vocab * row_bytes(H)
        head_p = self.predictor_vocab * row_bytes(self.predictor.hidden)
        return self.talker.weight_bytes() + head_t + (self.groups - 1) * (self.predictor.weight_bytes() + head_p)

    def weights(self) -> int:
        H = self.talker.hidden
        return (self.talker.weights() + self.talker_vocab * H +
                (self.groups - 1) * (self.predictor.weights() + self.predictor_vocab * self.predictor.hidden))

    def stream_bytes(self, talker_pos: float) -> float:
        """Per-stream algorithmic bytes beyond the weights: every MUL_MAT's F32 input and output, the KV rows the
        attention reads and writes, the embedding rows read and the codes written."""
        T, P, G = self.talker, self.predictor, self.groups
        act = lambda s: sum((k + n) * 4 for n, k in s.matrices()) * s.n_layers
        head = lambda s, v: (s.hidden + v) * 4
        kv_row = lambda s: 2 * s.kv_dim * 4
        talker = act(T) + head(T, self.talker_vocab) + T.n_layers * kv_row(T) * (talker_pos + 2)
        # predictor: prefill (2 positions: reads 1 + 2 cached rows) then G-2 calls at positions 2..G-1
        pred_positions_read = 3 + sum(g + 2 for g in range(1, G - 1))
        pred = ((G) * act(P) + (G - 1) * head(P, self.predictor_vocab) +
                P.n_layers * kv_row(P) * (pred_positions_read + G))
        emb = G * row_bytes(T.hidden) + 2 * row_bytes(T.hidden)
        return talker + pred + emb + G * 4

    def frame_bytes(self, m: int, talker_pos: float) -> float:
        return self.weight_bytes() + m * self.stream_bytes(talker_pos)

    def frame_ops(self, m: int) -> int:
        return 2 * m * (self.talker.weights() + self.talker_vocab * self.talker.hidden +
                        (self.groups - 1) * (self.predictor.weights() + self.predictor_vocab * self.predictor.hidden)
                        + self.predictor.weights())  # the prefill's second position


FRAME_06B = FrameShape(TALKER_06B, PREDICTOR_06B)


def _norm_vec(seed: int, n: int, scale: float, device) -> torch.Tensor:
    return torch.from_numpy((1.0 + host.normal(seed, n, scale)).astype(np.float32)).to(device)


def _q8(seed: int, rows: int, k: int, scale: float, device) -> torch.Tensor:
    return quantize_rows(torch.from_numpy(host.normal(seed, rows * k, scale).reshape(rows, k)).to(device))


@dataclass
class FrameModel:
    shape: FrameShape
    talker: DeviceModel
    predictor: DeviceModel
    t_out: dict
    p_out: dict
    ptables: list


def build_frame_model(fs: FrameShape, device: torch.device) -> FrameModel:
    """Talker (seed 1000) and code predictor (seed 3000) weights as build_model makes them, plus the q/k head norms
    (1 + 0.2 N), the final norms (1 + 0.1 N), the Q8_0 heads (0.02 N) and the predictor's codec tables (0.02 N)."""
    t = build_model(fs.talker, device, seed=1000)
    p = build_model(fs.predictor, device, seed=3000)
    for dm, base in ((t, 1000), (p, 3000)):
        for l, L in enumerate(dm.layers):
            L["q_norm"] = _norm_vec(base + 16 * l + 10, dm.shape.head_dim, 0.2, device)
            L["k_norm"] = _norm_vec(base + 16 * l + 11, dm.shape.head_dim, 0.2, device)
    H = fs.talker.hidden
    t_out = dict(norm=_norm_vec(2990, H, 0.1, device), heads=[_q8(2991, fs.talker_vocab, H, 0.02, device)])
    p_out = dict(norm=_norm_vec(4990, H, 0.1, device),
                 heads=[_q8(5000 + g, fs.predictor_vocab, H, 0.02, device) for g in range(fs.groups - 1)])
    ptables = [_q8(6000 + g, fs.predictor.table_rows, H, 0.02, device) for g in range(fs.groups - 1)]
    torch.cuda.synchronize(device)
    return FrameModel(fs, t, p, t_out, p_out, ptables)


def frame_host_copy(fm: FrameModel):
    """Oracle dicts (oracle.frame's talker / predictor arguments) and the predictor tables, on the host."""
    out = []
    for dm, o, vocab in ((fm.talker, fm.t_out, fm.shape.talker_vocab),
                         (fm.predictor, fm.p_out, fm.shape.predictor_vocab)):
        mats, norms, table = host_copy(dm)
        s = dm.shape
        qkn = np.stack([L[k].cpu().numpy() for L in dm.layers for k in ("q_norm", "k_norm")])
        out.append(dict(mats=mats, norms=norms, qkn=qkn, table=table, out_norm=o["norm"].cpu().numpy(),
                        heads=[h.cpu().numpy() for h in o["heads"]], hidden=s.hidden, n_head=s.n_head, n_kv=s.n_kv,
                        head_dim=s.head_dim, inter=s.inter, eps=s.eps, theta=fm.shape.rope_theta, vocab=vocab))
    return out[0], out[1], [t.cpu().numpy() for t in fm.ptables]
