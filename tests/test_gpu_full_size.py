"""The decode step at the BASELINE configurations' own sizes, against the oracle.

* config 2: the 28-layer 0.6B talker step at M = 1 and 2 (single-launch persistent kernel) and 8 (tensor-core
  chain, the chain's own choice from M = 3);
* config 3: the same 28 layers at M = 16, 64 and 256 through the tensor-core chain;
* config 4: the 28-layer 1.7B-shaped step at M = 1 (persistent) and M = 32 (tensor-core chain).

The models are the bench's own (seeds 1000 + 16*layer + index, 0.02*N(0,1) weights packed by the oracle's
quantize_row_q8_0_ref; the packing itself is pinned bit-exact elsewhere), so the per-layer hand-off buffers, the
reuse of the step's epochs over 28 layers and the weight stream's layer-to-layer ring are exercised at full depth.
Layers 0, 13 and 27 are checked op by op on the GPU's own intermediates; every layer is checked against the
oracle's layer on the GPU's own input to it (2e-3 relative L2 per token); the whole step is checked against the
oracle's chain end to end, with the bound that the chain's own sensitivity over 28 layers calls for
(chain_checks.e2e_bounds).  Inputs are the bench's seeded streams (plus config 3's 1 % outliers at 20x).
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from chain_checks import Dims, check_end_to_end, check_layer, check_teacher_forced

pytestmark = pytest.mark.gpu

D06 = Dims(1024, 16, 8, 128, 3072)
D17 = Dims(2048, 16, 8, 128, 6144)
LAYERS = 28
CHECKED = (0, 13, 27)
TABLE_ROWS = 3072


def oracle_model(O, d: Dims, seed=1000):
    mats, norms = [], []
    shp = d.shapes()
    for l in range(LAYERS):
        seeds = [seed + 16 * l + j for j in range(7)] + [seed + 16 * l + 8, seed + 16 * l + 9]
        vals = O.normal_many(seeds, [0.02] * 7 + [0.1, 0.1], [n * k for n, k in shp] + [d.hidden] * 2)
        mats += [O.quantize_rows_mt(vals[j].reshape(n, k)) for j, (n, k) in enumerate(shp)]
        norms += [1.0 + vals[7], 1.0 + vals[8]]
    table = O.quantize_rows_mt(O.normal(seed - 1, TABLE_ROWS * d.hidden, 0.02).reshape(TABLE_ROWS, d.hidden))
    return mats, np.stack(norms).astype(np.float32), table


def upload(mats, norms, table, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    keys = ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown")
    layers = []
    for l in range(len(mats) // 7):
        L = {k: t(mats[7 * l + j]) for j, k in enumerate(keys)}
        L["norm_in"] = t(norms[2 * l])
        L["norm_post"] = t(norms[2 * l + 1])
        layers.append(L)
    return layers, t(table)


def stream_inputs(O, m, hidden, outliers=False):
    """The bench's streams 0..m-1 (seed 5000 + s, ids s*7919 % 3072); with outliers, the 1 % of entries that
    config 3 scales by 20 (shapes.outlier_positions, as the bench applies them)."""
    S = shapes()
    x = np.stack(O.normal_many([S.STREAM_SEED + s for s in range(m)], [1.0] * m, [hidden] * m)).astype(np.float32)
    ids = np.asarray(S.stream_ids(m, TABLE_ROWS), dtype=np.int32)
    if outliers:
        x.reshape(-1)[S.outlier_positions(m, hidden)] *= np.float32(S.OUTLIER_SCALE)
    return x, ids


def shapes():
    import importlib

    import __graft_entry__

    __graft_entry__.load_package()
    return importlib.import_module(__graft_entry__.PKG_NAME + ".shapes")


def make_chain(chain_mod, layers, t_table, d: Dims, path, max_m):
    old = os.environ.get("B200Q8_CHAIN_PER_OP")
    os.environ["B200Q8_CHAIN_PER_OP"] = "1" if path == "per_op" else "0"
    try:
        return chain_mod.DecodeChain(layers, t_table, max_m=max_m, **d.kw())
    finally:
        if old is None:
            del os.environ["B200Q8_CHAIN_PER_OP"]
        else:
            os.environ["B200Q8_CHAIN_PER_OP"] = old


@pytest.fixture(scope="module")
def model06(O, dev):
    mats, norms, table = oracle_model(O, D06)
    layers, t_table = upload(mats, norms, table, dev)
    return mats, norms, table, layers, t_table


@pytest.fixture(scope="module")
def model17(O, dev):
    mats, norms, table = oracle_model(O, D17)
    layers, t_table = upload(mats, norms, table, dev)
    return mats, norms, table, layers, t_table


def run_and_check(O, chain_mod, q8, dev, model, d: Dims, m, path, outliers=False):
    mats, norms, table, layers, t_table = model
    ch = make_chain(chain_mod, layers, t_table, d, path, max_m=max(8, m))
    x_in, ids = stream_inputs(O, m, d.hidden, outliers)
    h_out = torch.full((m, d.hidden), float("nan"), dtype=torch.float32, device=dev)
    ch.run(torch.from_numpy(ids).to(dev), torch.from_numpy(x_in).to(dev), h_out)
    torch.cuda.synchronize()
    assert q8.device_status(0) == 0
    got = h_out.cpu().numpy()
    emb, _ = O.get_rows(table, d.hidden, ids)
    for l in CHECKED:
        h = (x_in + emb).astype(np.float32) if l == 0 else ch.buffer(l - 1, "h", m).cpu().numpy()
        check_layer(O, ch, mats, norms, l, m, h, d, h_next=got if l == LAYERS - 1 else None)
    check_teacher_forced(O, ch, mats, norms, (x_in + emb).astype(np.float32), got, d)
    check_end_to_end(O, mats, norms, table, ids, x_in, got, d)
    # a replay of the same inputs is bit-identical (the per-launch epochs advance over all 28 layers)
    again = torch.empty_like(h_out)
    ch.run(torch.from_numpy(ids).to(dev), torch.from_numpy(x_in).to(dev), again)
    torch.cuda.synchronize()
    assert torch.equal(again, h_out)
    ch.close()


@pytest.mark.parametrize("m", [1, 2, 8])
def test_config2_28_layers(O, chain_mod, q8, dev, model06, m):
    run_and_check(O, chain_mod, q8, dev, model06, D06, m, "auto")


@pytest.mark.parametrize("m", [16, 64, 256])
def test_config3_tensor_core_chain_28_layers(O, chain_mod, q8, dev, model06, m):
    run_and_check(O, chain_mod, q8, dev, model06, D06, m, "per_op", outliers=True)


def test_config4_persistent_28_layers_m1(O, chain_mod, q8, dev, model17):
    run_and_check(O, chain_mod, q8, dev, model17, D17, 1, "persistent")


def test_config4_tensor_core_chain_28_layers_m32(O, chain_mod, q8, dev, model17):
    run_and_check(O, chain_mod, q8, dev, model17, D17, 32, "per_op")
