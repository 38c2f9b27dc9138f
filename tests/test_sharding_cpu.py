"""Row sharding of the linear across ranks (gloo, world size 2, on the CPU).

Each rank quantises and multiplies its own block of rows; the gathered result
must equal the unsharded computation exactly (rows are independent).  The
failure path is exercised on the host: a rank that raises before the gather
makes the other rank's collective fail with an error instead of hanging.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tilegen_b200.sharding import gather_rows, int8_convrot_linear_local, local_rows, shard_bounds


def test_shard_bounds_cover_rows_exactly():
    for m in (0, 1, 7, 8190, 65520):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
    assert shard_bounds(65520, 8, 7) == (57330, 65520)
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, fail_rank, q, overlap=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        torch.manual_seed(0)
        x = torch.randn(m, 512)
        wq = torch.randint(-127, 128, (64, 512), dtype=torch.int8)
        ws = torch.rand(64) * 1e-2
        if rank == fail_rank:
            raise RuntimeError("planted failure before the gather")
        y_local = int8_convrot_linear_local(local_rows(x, world, rank), wq, ws, None, torch.float32)
        ref = int8_convrot_linear_local(x, wq, ws, None, torch.float32)
        if overlap:
            # the gather in flight while the next layer runs on the local rows
            pending = gather_rows(y_local, m, async_op=True)
            w2 = torch.randint(-127, 128, (32, 256), dtype=torch.int8)
            with pending.overlapped():  # gloo: nothing to reserve
                nxt = int8_convrot_linear_local(y_local.repeat(1, 4), w2, torch.rand(32) * 1e-2, None,
                                                torch.float32)
            y = pending.wait()
            ok = bool(torch.equal(y, ref)) and nxt.shape == (y_local.shape[0], 32) and pending.wait() is not None
        else:
            y = gather_rows(y_local, m)
            ok = bool(torch.equal(y, ref))
        q.put((rank, "ok", ok, tuple(y.shape)))
    except Exception as e:  # report, never hang
        q.put((rank, "error", type(e).__name__, str(e)[:80]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, m, fail_rank=-1, overlap=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, fail_rank, q, overlap)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return sorted(q.get(timeout=5) for _ in procs)


@pytest.mark.parametrize("m", [9, 64])
def test_sharded_equals_unsharded_gloo(m):
    res = _run(2, m)
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] for r in res) and all(r[3] == (m, 64) for r in res)


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(2, 16, fail_rank=1)
    assert res[1][1] == "error" and "planted" in res[1][3]
    assert res[0][1] == "error"  # the survivor's collective errors out


def test_async_gather_overlaps_the_next_layer_gloo():
    res = _run(2, 33, overlap=True)
    assert [r[1] for r in res] == ["ok", "ok"], res
    assert all(r[2] for r in res) and all(r[3] == (33, 64) for r in res)


def test_gather_sm_reserves():
    """The SMs the next layer leaves to an in-flight gather (measured on B200)."""
    from tilegen_b200 import sharding

    assert sharding.nccl_gather_reserve(2) == 32 and sharding.nccl_gather_reserve(8) == 64
    assert sharding.nccl_gather_reserve(4) == 64 and sharding.PEER_GATHER_RESERVE == 2
    # A finished (or CPU) gather reserves nothing: the context is a no-op.
    h = sharding.RowGather(None, torch.zeros(4, 2), None, 4, reserve=32)
    with h.overlapped():
        pass
    assert torch.equal(h.wait(), torch.zeros(4, 2))
