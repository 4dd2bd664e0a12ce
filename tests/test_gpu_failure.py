"""Failure detection on the GPU without a GPU fault: the persistent step's hand-off waits are made to run out
(host-side fault injection: the step's CTAs are given disagreeing epochs, so no wait is ever satisfied), and the
kernel must end on its own within its bounded waits, report B200Q8_ERR_DEVICE_TIMEOUT through the device status
word, leave the context usable, and compute correctly once the chain is restored."""
from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from test_gpu_chain import H, HD, I, NH, NKV, make_model, upload

pytestmark = pytest.mark.gpu

DEVICE_TIMEOUT = 21


@pytest.mark.parametrize("m", [1, 2])
def test_step_wait_timeout_is_reported_and_recoverable(pkg, O, chain_mod, dev, m):
    from synthesize_cpp_b200 import _abi, q8

    mats, norms, table = make_model(O, 2, seed=700)
    layers, t_table = upload(mats, norms, table, dev)
    ch = chain_mod.DecodeChain(layers, t_table, hidden=H, n_head=NH, n_kv=NKV, head_dim=HD, inter=I, max_m=2)
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((m, H)).astype(np.float32)).to(dev)
    ids = torch.from_numpy(rng.integers(0, 64, m).astype(np.int32)).to(dev)
    h_ok = torch.empty((m, H), device=dev)
    ch.run(ids, x, h_ok)
    assert q8.device_status(dev.index or 0) == 0

    L = _abi.lib()
    assert L.b200q8_chain_inject_epoch_skew(ch._h, 1) == 0
    h_bad = torch.full((m, H), float("nan"), device=dev)
    t0 = time.perf_counter()
    ch.run(ids, x, h_bad)
    torch.cuda.synchronize(dev)
    dt = time.perf_counter() - t0
    assert q8.device_status(dev.index or 0, clear=True) == DEVICE_TIMEOUT
    assert dt < 15.0, dt  # bounded waits (about a second each, in parallel), not a hang

    assert L.b200q8_chain_inject_epoch_skew(ch._h, 0) == 0
    h2 = torch.empty((m, H), device=dev)
    for _ in range(2):
        ch.run(ids, x, h2)
    torch.cuda.synchronize(dev)
    assert q8.device_status(dev.index or 0) == 0
    assert torch.equal(h2, h_ok)
    ch.close()
