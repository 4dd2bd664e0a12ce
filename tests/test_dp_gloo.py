"""The multi-rank host path on CPU with gloo (world size 2): stream
partitioning, barrier + max-over-ranks timing, and failure detection on the
host (a rank that raises before a collective makes the survivor's collective
end with an error after the process-group timeout, instead of hanging)."""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import __graft_entry__ as g

    g.load_package()
    import torch.distributed as dist
    from synthesize_cpp_b200 import dp

    try:
        r, w = dp.init("gloo", timeout_s=10.0 if mode == "fail" else 60.0)
        if mode == "ok":
            first, sizes = dp.partition_streams(512, w, r, 64)
            dp.barrier()
            m = dp.max_over_ranks(float(r + 1) * 1.5)
            q.put(("ok", r, first, sizes, m))
        else:
            if r == 1:
                raise RuntimeError("rank 1 dies before the collective")
            try:
                dp.max_over_ranks(1.0)
                q.put(("no-error", r))
            except Exception as e:  # the survivor must see an error, not hang
                q.put(("error", r, type(e).__name__))
    except RuntimeError as e:
        q.put(("raised", rank, str(e)))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_partition_covers_streams_once():
    sys.path.insert(0, ROOT)
    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import dp

    for world in (1, 2, 3, 4, 8):
        seen = []
        for r in range(world):
            first, sizes = dp.partition_streams(512, world, r, 64)
            assert all(0 < s <= 64 for s in sizes)
            seen.extend(range(first, first + sum(sizes)))
        assert sorted(seen) == list(range(512))
    assert dp.partition_streams(5, 2, 1, 64) == (3, [2])
    with pytest.raises(ValueError):
        dp.partition_streams(10, 2, 2, 4)


def test_two_rank_barrier_and_max():
    out = sorted(_run("ok"), key=lambda t: t[1])
    assert [o[0] for o in out] == ["ok", "ok"]
    assert out[0][2:4] == (0, [64, 64, 64, 64]) and out[1][2:4] == (256, [64, 64, 64, 64])
    assert out[0][4] == out[1][4] == 3.0


def test_dead_rank_is_detected_by_the_survivor():
    out = {o[1]: o for o in _run("fail")}
    assert out[1][0] == "raised"
    assert out[0][0] == "error"
