"""Qwen3-TTS-shaped workload geometry: layer shapes, bytes and ops.

Pure arithmetic with no torch, no ctypes and no native library, so that a CPU
harness can state the same workload as the device path without loading it.
The talker shapes follow the reference's decoder layer
(src/arch/qwen3-tts/operations.cpp:39-41,90-92,142): per layer the q, k, v, o,
gate, up and down projections, stored as Q8_0 rows of K/32 blocks of 34 bytes.
"""
from __future__ import annotations

from dataclasses import dataclass

QK = 32
BLOCK_BYTES = 34


def row_bytes(k: int) -> int:
    """Bytes of one Q8_0 row of k values (k % 32 == 0)."""
    return k // QK * BLOCK_BYTES


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
PREDICTOR_06B = Shape("qwen3-tts-0.6b-code-predictor", 5, 1024, 16, 8, 128, 3072, table_rows=2048)


def stream_ids(m: int, table_rows: int, first_stream: int = 0):
    """Token ids of streams first_stream .. first_stream+m-1 (a fixed spread over the table)."""
    return [(s + first_stream) * 7919 % table_rows for s in range(m)]


STREAM_SEED = 5000  # stream s draws its N(0,1) activations from seed STREAM_SEED + s
OUTLIER_SEED = 77
OUTLIER_SCALE = 20.0


def outlier_positions(m: int, hidden: int, first_stream: int = 0):
    """Flat indices into an [m, hidden] activation batch of the 1 % of entries that config 3 scales by 20 to
    exercise outlier block scales: drawn without repeats from a second seeded stream (numpy's PCG64 seeded with
    OUTLIER_SEED + first_stream), sorted."""
    import numpy as np

    total = m * hidden
    rng = np.random.default_rng(OUTLIER_SEED + first_stream)
    return np.sort(rng.choice(total, size=total // 100, replace=False))


def partition_streams(total: int, world: int, rank: int, batch: int) -> tuple[int, list[int]]:
    """Rank `rank`'s contiguous share of `total` streams as batches of at most `batch`:
    returns (first stream index, [batch sizes])."""
    if world < 1 or not 0 <= rank < world or batch < 1 or total < 0:
        raise ValueError("bad partition arguments")
    base, rem = divmod(total, world)
    mine = base + (1 if rank < rem else 0)
    first = rank * base + min(rank, rem)
    return first, [min(batch, mine - o) for o in range(0, mine, batch)]
