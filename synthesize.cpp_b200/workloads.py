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


@dataclass
class Shape:
    name: str
    n_layers: int
    hidden: int
    n_head: int
    n_kv: int
    head_dim: int
    inter: int
    table_rows: int = 3072
    eps: float = 1e-6

    @property
    def q_dim(self) -> int:
        return self.n_head * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv * self.head_dim

    def matrices(self):
        """(rows N, K) of q,k,v,o,gate,up,down."""
        H, Q, KV, I = self.hidden, self.q_dim, self.kv_dim, self.inter
        return [(Q, H), (KV, H), (KV, H), (H, Q), (I, H), (I, H), (H, I)]

    def weight_bytes(self) -> int:
        return self.n_layers * sum(n * row_bytes(k) for n, k in self.matrices())

    def weights(self) -> int:
        return self.n_layers * sum(n * k for n, k in self.matrices())

    def step_bytes(self, m: int) -> int:
        """Algorithmic HBM bytes of one step for m tokens: every Q8_0 weight once, every MUL_MAT's F32 input and
        output once, plus the GET_ROWS row read (34/32 B per value) and written (4 B per value)."""
        act = sum((k + n) * 4 for n, k in self.matrices()) * self.n_layers * m
        emb = (row_bytes(self.hidden) + 4 * self.hidden) * m
        return self.weight_bytes() + act + emb

    def step_flops(self, m: int) -> int:
        return 2 * self.weights() * m


TALKER_06B = Shape("qwen3-tts-0.6b-talker", 28, 1024, 16, 8, 128, 3072)
TALKER_17B = Shape("qwen3-tts-1.7b-talker", 28, 2048, 16, 8, 128, 6144)


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


def stream_inputs(m: int, hidden: int, table_rows: int, first_stream: int = 0, seed: int = 5000):
    """Per-stream N(0,1) activations (stream s from seed + s) and token ids."""
    x = np.stack([host.normal(seed + first_stream + s, hidden) for s in range(m)]).astype(np.float32)
    ids = ((np.arange(m) + first_stream) * 7919 % table_rows).astype(np.int32)
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
