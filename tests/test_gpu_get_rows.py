"""GET_ROWS and dequantization on the GPU through the C ABI: bit-exact with
the oracle (q * fp32(d) is exact in fp32)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_get_rows_matches_oracle(q8, O, dev):
    k, rows = 1024, 3072  # the talker codec_embedding shape (ne = [1024, 3072])
    table = O.quantize_rows(O.normal(21, rows * k, 0.02).reshape(rows, k))
    ids = np.array([0, 3071, 17, 17, 1500], dtype=np.int32)
    got = q8.get_rows(torch.from_numpy(table).to(dev), k, torch.from_numpy(ids).to(dev)).cpu().numpy()
    ref, st = O.get_rows(table, k, ids)
    assert st == 0
    assert np.array_equal(got, ref)
    assert q8.device_status(0) == 0


def test_text_embedding_row(q8, O, dev):
    # one row of a [2048, 151936]-shaped table: only the addressed rows are built
    k = 2048
    rows = O.quantize_rows(O.normal(5, 4 * k, 0.02).reshape(4, k))
    table = torch.zeros((151936, k // 32 * 34), dtype=torch.uint8, device=dev)
    table[151935] = torch.from_numpy(rows[3]).to(dev)
    ids = torch.tensor([151935], dtype=torch.int32, device=dev)
    got = q8.get_rows(table, k, ids).cpu().numpy()
    assert np.array_equal(got[0], O.dequantize_rows(rows[3], k)[0])


def test_out_of_range_ids_zero_fill_and_report(q8, O, dev):
    k = 64
    table = O.quantize_rows(O.normal(3, 8 * k).reshape(8, k))
    ids = np.array([1, -1, 8, 7], dtype=np.int32)
    got = q8.get_rows(torch.from_numpy(table).to(dev), k, torch.from_numpy(ids).to(dev)).cpu().numpy()
    ref, st = O.get_rows(table, k, ids)
    assert st == -1
    assert np.array_equal(got, ref)
    assert q8.device_status(0) == 1  # B200Q8_ERR_INVALID_ARG, then cleared
    assert q8.device_status(0) == 0


def test_empty_and_dequantize(q8, O, dev):
    k = 96
    table = O.quantize_rows(O.normal(4, 5 * k).reshape(5, k))
    t = torch.from_numpy(table).to(dev)
    empty = q8.get_rows(t, k, torch.zeros(0, dtype=torch.int32, device=dev))
    assert empty.shape == (0, k)
    assert np.array_equal(q8.dequantize_rows(t, k).cpu().numpy(), O.dequantize_rows(table, k))
