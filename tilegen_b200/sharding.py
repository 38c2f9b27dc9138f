"""Row (token) sharding of the int8_convrot linear across GPUs.

Every output row depends only on its own input row (the rotation and the
scale are per row, the GEMM contracts over K), so N GPUs each quantise and
multiply a contiguous block of rows against a replicated int8 weight: there is
no collective on the path.  When a caller needs the full ``[M, N]`` output on
every rank, ``gather_rows`` all-gathers the blocks over NCCL (NVLink), as one
collective outside the hot path; with ``async_op=True`` it returns at once and
the caller overlaps the transfer with the next layer's kernels, waiting only
where the gathered output is used.  The rotate+quant and GEMM kernels are
persistent and size their grids for every SM, so run the next layer inside the
handle's ``overlapped()`` context (``ops.sm_budget(sms - reserve)``) while a
gather is in flight, leaving the collective's kernels the SMs they hold (NCCL
2.28's all-gather on B200: about 32 SMs at 2 GPUs, 64 at 8; the copy-engine
gather below: 2); otherwise part of the next layer's grid waits for the
collective to finish::

    g = gather_rows(y_local, M, async_op=True)
    with g.overlapped():
        z_local = next_layer(x_local)
    y = g.wait()

Blocks are ``ceil(M / world)`` rows; the last rank's block may be short or
empty.  ``gather_rows`` pads the short blocks to the common size for the
collective and trims the result.

``PeerRowGather`` is the same gather for a caller that repeats it every step:
each rank writes its rows straight into a buffer that every peer has mapped,
and the peers' blocks are pulled in by the GPU's copy engines over NVLink, so
the transfer uses no SMs and the next layer's kernels keep all of them.
"""
from __future__ import annotations

import contextlib
import ctypes

import torch
import torch.distributed as dist


def shard_bounds(m: int, world: int, rank: int) -> tuple[int, int]:
    """Half-open row range ``[start, end)`` of ``rank``'s block of an ``m``-row input."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    per = -(-m // world)
    start = min(m, rank * per)
    return start, min(m, start + per)


def local_rows(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's block of rows of ``x [M, ...]`` (a view)."""
    s, e = shard_bounds(x.shape[0], world, rank)
    return x[s:e]


def nccl_gather_reserve(world: int) -> int:
    """SMs to leave to NCCL's all-gather while the next layer runs beside it.

    Measured on B200 with NCCL 2.28 (65520 tokens, the next layer ffn_up): at 2
    GPUs 32 (2442 -> 1933 us for gather + next layer), at 8 GPUs 64 (1367 ->
    1045 us; 32 left there was slower than none).  Other sizes take the value of
    the nearer measured one.
    """
    return 32 if world <= 2 else 64


# SMs the copy-engine gather needs while the next layer runs: its one-element
# all-reduce (the ready signal) must find one.
PEER_GATHER_RESERVE = 2


@contextlib.contextmanager
def _reserve_sms(device: torch.device, reserve: int):
    from . import ops

    if device.type != "cuda" or reserve <= 0:
        yield
        return
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    with ops.sm_budget(max(1, sms - reserve)):
        yield


class RowGather:
    """An all-gather of row blocks in flight (``gather_rows(..., async_op=True)``).

    ``wait()`` returns the gathered ``[m_total, N]`` tensor.  On NCCL it only
    makes the caller's current stream wait for the collective (the host does not
    block), so kernels enqueued before ``wait()`` overlap the transfer; enqueue
    them inside ``with handle.overlapped():``, which sizes the persistent kernels'
    grids for the SMs the collective leaves (``nccl_gather_reserve``).
    """

    def __init__(self, work, out: torch.Tensor, parts: list | None, m_total: int, reserve: int = 0):
        self._work, self._out, self._parts, self._m = work, out, parts, m_total
        self.reserve = reserve

    def overlapped(self):
        """Context for the kernels that run while this gather is in flight."""
        dev = self._out.device if self._out is not None else torch.device("cpu")
        return _reserve_sms(dev, self.reserve if self._work is not None else 0)

    def wait(self) -> torch.Tensor:
        if self._work is not None:
            self._work.wait()
            self._work = None
            if self._parts is not None:
                self._out = torch.cat(self._parts, 0)
                self._parts = None
        return self._out[: self._m]


def gather_rows(y_local: torch.Tensor, m_total: int, group=None, async_op: bool = False):
    """All-gather every rank's ``[rows_r, N]`` block into the full ``[m_total, N]``.

    With ``async_op=True`` returns a ``RowGather`` whose ``wait()`` gives the result.
    """
    world = dist.get_world_size(group)
    per = -(-m_total // world)
    n = y_local.shape[1]
    buf = y_local
    if y_local.shape[0] != per:
        buf = torch.zeros((per, n), dtype=y_local.dtype, device=y_local.device)
        buf[: y_local.shape[0]].copy_(y_local)
    buf = buf.contiguous()
    parts = None
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * per, n), dtype=y_local.dtype, device=y_local.device)
        work = dist.all_gather_into_tensor(out, buf, group=group, async_op=async_op)
    else:
        parts = [torch.empty_like(buf) for _ in range(world)]
        work = dist.all_gather(parts, buf, group=group, async_op=async_op)
        out = None if async_op else torch.cat(parts, 0)
    reserve = nccl_gather_reserve(world) if out is not None else 0
    handle = RowGather(work if async_op else None, out, parts if async_op else None, m_total, reserve)
    return handle if async_op else handle.wait()


class _DeviceArray:
    """A raw device buffer seen by torch through ``__cuda_array_interface__`` (no copy)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_INT_VIEW = {1: (torch.int8, "|i1"), 2: (torch.int16, "<i2"), 4: (torch.int32, "<i4")}


class PeerGather:
    """A ``PeerRowGather.start()`` in flight; ``wait()`` orders the caller's current
    stream after the copies and returns the gathered ``[m_total, N]`` tensor.
    Enqueue the kernels that overlap it inside ``with handle.overlapped():``."""

    def __init__(self, events: list, out: torch.Tensor):
        self._events, self._out = events, out
        self.reserve = PEER_GATHER_RESERVE

    def overlapped(self):
        """Context for the kernels that run while these copies are in flight."""
        return _reserve_sms(self._out.device, self.reserve if self._events else 0)

    def wait(self) -> torch.Tensor:
        cur = torch.cuda.current_stream(self._out.device)
        for ev in self._events:
            cur.wait_event(ev)
        self._events = []
        return self._out


class PeerRowGather:
    """Row all-gather by copy engines over NVLink, for one process per GPU on one node.

    Set up once per output shape (``m_total`` rows of ``n`` columns of ``dtype``):
    every rank allocates two buffers of the full ``[world * ceil(m_total / world), n]``
    output and maps its peers' (interprocess handles, exchanged once).  Each step:

    1. write this rank's rows into ``local()`` (e.g. as the GEMM's output);
    2. ``start()``: once every rank has reached its own ``start()`` in stream order
       (a one-element NCCL all-reduce, on a side stream), one copy per peer pulls
       that peer's block from its buffer into this rank's, on separate streams, so
       several copy engines run at once; nothing waits on the host;
    3. ``wait()`` on the returned handle (the caller's current stream waits for the
       copies) gives the full output.  Kernels enqueued between ``start()`` and
       ``wait()`` overlap the transfer; enqueue them inside the handle's
       ``overlapped()`` context (``ops.sm_budget(sms - 2)``) so that the
       one-element all-reduce finds an SM.

    The two buffers alternate between steps, so a step's rows may be written while
    peers may still copy the previous step's.  Call ``wait()`` on one step's gather
    before writing the rows of the step after the next one (in practice: wait on
    each step before starting the next).  Every rank calls ``start()`` the same
    number of times, in the same order as its other collectives.  ``close()`` frees
    the buffers (a barrier, so no peer still reads them); tensors returned earlier
    must not be used after it.
    """

    def __init__(self, m_total: int, n: int, dtype: torch.dtype, device=None, group=None):
        from . import _lib

        self._L = _lib.lib()
        self._check = _lib.check
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n, self.dtype = int(m_total), int(n), dtype
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.per = -(-self.m // self.world)
        esize = torch.empty(0, dtype=dtype).element_size()
        self.row_bytes = self.n * esize
        self.bounds = [shard_bounds(self.m, self.world, r) for r in range(self.world)]
        total = max(1, self.world * self.per * self.row_bytes)
        hb = int(self._L.tg_peer_handle_bytes())
        int_dt, typestr = _INT_VIEW[esize]
        self._own, self._views, handles = [], [], []
        self._peer = [[None] * self.world for _ in range(2)]
        self._closed = True
        # Every rank takes the same collective steps whatever fails locally, and all
        # raise together if any rank failed, so no rank waits in a collective that a
        # failed peer never joins.
        with torch.cuda.device(self.device):
            self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
            err = None
            try:
                for _ in range(2):
                    ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(hb)
                    self._check("tg_peer_alloc", self._L.tg_peer_alloc(total, ctypes.byref(ptr), h))
                    self._own.append(ptr.value)
                    handles.append(h.raw)
                    arr = _DeviceArray(ptr.value, (self.world * self.per, self.n), typestr)
                    self._views.append(torch.as_tensor(arr, device=self.device).view(int_dt).view(dtype))
            except Exception as e:  # reported below, on every rank
                err = e
            self._agree(err, "allocating the gather buffers")
            gathered = [None] * self.world
            dist.all_gather_object(gathered, handles, group=group)
            try:
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    for b in range(2):
                        ptr = ctypes.c_void_p()
                        self._check("tg_peer_open", self._L.tg_peer_open(gathered[r][b], ctypes.byref(ptr)))
                        self._peer[b][r] = ptr.value
            except Exception as e:
                err = e
            self._agree(err, "mapping the peers' buffers")
            self._copy_streams = [torch.cuda.Stream(self.device) for _ in range(max(1, self.world - 1))]
            self._sync_stream = torch.cuda.Stream(self.device)
        self._buf = 0
        self._closed = False

    def _agree(self, err, what: str) -> None:
        """All ranks learn whether any failed at ``what``; on failure each releases what
        it holds and raises."""
        ok = torch.tensor([0.0 if err is not None else 1.0], device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if ok.item() == 1.0:
            return
        for b in range(2):
            for r, ptr in enumerate(self._peer[b]):
                if ptr is not None:
                    self._L.tg_peer_close(ptr)
                    self._peer[b][r] = None
        torch.cuda.synchronize(self.device)
        for ptr in self._own:
            self._L.tg_peer_free(ptr)
        self._own, self._views = [], []
        raise RuntimeError(f"PeerRowGather: {what} failed on "
                           f"{'this rank' if err is not None else 'another rank'}: {err}")

    def local(self) -> torch.Tensor:
        """This rank's rows of the buffer the next ``start()`` gathers (write them first)."""
        s, e = self.bounds[self.rank]
        return self._views[self._buf][s:e]

    def start(self) -> PeerGather:
        b = self._buf
        cur = torch.cuda.current_stream(self.device)
        ready = torch.cuda.Event()
        ready.record(cur)
        self._sync_stream.wait_event(ready)
        with torch.cuda.stream(self._sync_stream):
            dist.all_reduce(self._flag, group=self.group, async_op=True).wait()
        events, j = [], 0
        for r in range(self.world):
            s, e = self.bounds[r]
            if r == self.rank or e <= s:
                continue
            st = self._copy_streams[j]
            j += 1
            st.wait_stream(self._sync_stream)
            off = s * self.row_bytes
            self._check("tg_copy_async", self._L.tg_copy_async(self._own[b] + off, self._peer[b][r] + off,
                                                               (e - s) * self.row_bytes, st.cuda_stream))
            ev = torch.cuda.Event()
            ev.record(st)
            events.append(ev)
        self._buf ^= 1
        return PeerGather(events, self._views[b][: self.m])

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every peer has finished its copies from our buffers
        for b in range(2):
            for r, ptr in enumerate(self._peer[b]):
                if ptr is not None:
                    self._L.tg_peer_close(ptr)
        dist.barrier(group=self.group)
        for ptr in self._own:
            self._L.tg_peer_free(ptr)
        self._views = []


def int8_convrot_linear_local(x_local: torch.Tensor, wq: torch.Tensor, wscale: torch.Tensor,
                              bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                              group_size: int = 256) -> torch.Tensor:
    """One rank's share: rotate+quantise its rows, then the fused INT8 GEMM + dequant."""
    from .kernels.int8_convrot import quantize_convrot
    from .quant.int8_ops import int8_matmul_dequant_chunked

    out_dtype = out_dtype or x_local.dtype
    if x_local.shape[0] == 0:
        return torch.empty((0, wq.shape[0]), dtype=out_dtype, device=x_local.device)
    xq, xs = quantize_convrot(x_local, group_size, backend="fht")
    return int8_matmul_dequant_chunked(xq, xs, wq, wscale, bias, out_dtype)
