"""Row-sharded linear on 2 GPUs with NCCL: each rank runs the kernels on its rows,
gather_rows all-gathers the blocks; the result equals the single-GPU output bit for
bit.  Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, q):
    import datetime

    import torch.distributed as dist

    from tilegen_b200 import _lib
    from tilegen_b200.kernels.int8_convrot import quantize_convrot
    from tilegen_b200.quant import int8_matmul_dequant_chunked, quantize_convrot_weight
    from tilegen_b200.sharding import gather_rows, int8_convrot_linear_local, local_rows
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x = outlier_activations(m, 5120, seed=0, dtype=torch.bfloat16).to(dev)
        wq, ws = quantize_convrot_weight(gaussian_weight(1024, 5120, seed=1, dtype=torch.bfloat16).to(dev), 256)
        y_local = int8_convrot_linear_local(local_rows(x, world, rank), wq, ws, None, torch.bfloat16)
        y = gather_rows(y_local, m)
        xq, xs = quantize_convrot(x, 256, backend="fht")
        ref = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.bfloat16)
        ok = bool(torch.equal(y, ref))
        # In flight: the next layer runs on the SMs NCCL leaves (32 at 2 GPUs).
        pending = gather_rows(y_local, m, async_op=True)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        with pending.overlapped():
            budget = int(_lib.lib().tg_sm_budget())
            z = int8_convrot_linear_local(local_rows(x, world, rank), wq, ws, None, torch.bfloat16)
        y2 = pending.wait()
        ok = (ok and budget == sms - 32 and int(_lib.lib().tg_sm_budget()) == 0 and bool(torch.equal(y2, ref))
              and bool(torch.equal(z, y_local)))
        q.put((rank, ok, tuple(y.shape)))
    except Exception as e:  # report, never hang
        q.put((rank, False, f"{type(e).__name__}: {e}"[:200]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [4096, 8190])
def test_sharded_linear_equals_single_gpu_nccl(m):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    res = sorted(q.get(timeout=10) for _ in procs)
    assert all(r[1] for r in res), res


def _peer_worker(rank, world, port, m, q):
    import datetime

    import torch.distributed as dist

    from tilegen_b200 import ops
    from tilegen_b200.kernels.int8_convrot import quantize_convrot
    from tilegen_b200.quant import int8_matmul_dequant_chunked, quantize_convrot_weight
    from tilegen_b200.sharding import PeerRowGather, local_rows
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    g = None
    try:
        wq, ws = quantize_convrot_weight(gaussian_weight(1024, 5120, seed=1, dtype=torch.bfloat16).to(dev), 256)
        g = PeerRowGather(m, 1024, torch.bfloat16, dev)
        other = torch.randn(4096, 4096, device=dev)
        ok = True
        for step in range(4):  # both buffers, each used twice
            x = outlier_activations(m, 5120, seed=10 + step, dtype=torch.bfloat16).to(dev)
            xq, xs = quantize_convrot(local_rows(x, world, rank), 256, backend="fht")
            ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.bfloat16, out=g.local())
            pending = g.start()
            with pending.overlapped():  # kernels in flight while the copy engines run
                other = other @ other.t() * 1e-4
                nxt = quantize_convrot(local_rows(x, world, rank), 256, backend="fht")
            y = pending.wait()
            ok = ok and bool(torch.equal(nxt[0], xq))
            xq, xs = quantize_convrot(x, 256, backend="fht")
            ref = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.bfloat16)
            ok = ok and bool(torch.equal(y, ref)) and tuple(y.shape) == (m, 1024)
        q.put((rank, ok, m))
    except Exception as e:  # report, never hang
        q.put((rank, False, f"{type(e).__name__}: {e}"[:300]))
    finally:
        if g is not None:
            g.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [4096, 8191])
def test_peer_copy_gather_equals_single_gpu(m):
    """PeerRowGather (copy engines over NVLink, no SMs): four steps alternating its two
    buffers, each step's rows written by the GEMM straight into the mapped buffer, a
    matmul in flight during the copies; every step equals the single-GPU output."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, m, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    res = sorted(q.get(timeout=10) for _ in procs)
    assert all(r[1] for r in res), res


def _peer_one_gpu_worker(rank, world, port, fail_rank, q):
    """Both ranks on cuda:0 with gloo (host-side collectives): the copy-engine gather's
    protocol and buffers without a second GPU.  ``fail_rank`` >= 0 makes that rank's
    buffer allocation fail, and every rank must then raise, none may hang."""
    import datetime

    import torch.distributed as dist

    from tilegen_b200 import _lib
    from tilegen_b200.sharding import PeerRowGather, shard_bounds

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    g = None
    try:
        m, n = 1000, 256
        if rank == fail_rank:
            real = _lib.lib()

            class _Failing:
                def __getattr__(self, name):
                    if name == "tg_peer_alloc":
                        return lambda *a: _lib.TG_ERR_CUDA
                    return getattr(real, name)

            orig = _lib.lib
            _lib.lib = lambda: _Failing()
        try:
            g = PeerRowGather(m, n, torch.bfloat16, dev)
        finally:
            if rank == fail_rank:
                _lib.lib = orig
        ok = True
        for step in range(3):
            full = torch.randn(m, n, generator=torch.Generator().manual_seed(step)).to(torch.bfloat16).to(dev)
            s, e = shard_bounds(m, world, rank)
            g.local().copy_(full[s:e])
            y = g.start().wait()
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(y, full))
        q.put((rank, "ok" if ok else "mismatch"))
    except RuntimeError as e:
        q.put((rank, "raised" if "PeerRowGather" in str(e) else f"other: {e}"[:200]))
    except Exception as e:  # report, never hang
        q.put((rank, f"{type(e).__name__}: {e}"[:200]))
    finally:
        if g is not None:
            g.close()
        dist.destroy_process_group()


def _run_one_gpu(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_one_gpu_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return sorted(q.get(timeout=10) for _ in procs)


def test_peer_gather_protocol_on_one_gpu():
    """Two processes on one GPU: three steps over both buffers equal the full rows."""
    res = _run_one_gpu(-1)
    assert [r[1] for r in res] == ["ok", "ok"], res


def test_peer_gather_setup_failure_raises_on_every_rank():
    """A rank whose buffer allocation fails: both ranks raise (no hang)."""
    res = _run_one_gpu(1)
    assert [r[1] for r in res] == ["raised", "raised"], res
