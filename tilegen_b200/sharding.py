"""Row (token) sharding of the int8_convrot linear across GPUs.

Every output row depends only on its own input row (the rotation and the
scale are per row, the GEMM contracts over K), so N GPUs each quantise and
multiply a contiguous block of rows against a replicated int8 weight: there is
no collective on the path.  When a caller needs the full ``[M, N]`` output on
every rank, ``gather_rows`` all-gathers the blocks over NCCL (NVLink), as one
collective outside the hot path; with ``async_op=True`` it returns at once and
the caller overlaps the transfer with the next layer's kernels, waiting only
where the gathered output is used.

Blocks are ``ceil(M / world)`` rows; the last rank's block may be short or
empty.  ``gather_rows`` pads the short blocks to the common size for the
collective and trims the result.
"""
from __future__ import annotations

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


class RowGather:
    """An all-gather of row blocks in flight (``gather_rows(..., async_op=True)``).

    ``wait()`` returns the gathered ``[m_total, N]`` tensor.  On NCCL it only
    makes the caller's current stream wait for the collective (the host does not
    block), so kernels enqueued before ``wait()`` overlap the transfer.
    """

    def __init__(self, work, out: torch.Tensor, parts: list | None, m_total: int):
        self._work, self._out, self._parts, self._m = work, out, parts, m_total

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
    handle = RowGather(work if async_op else None, out, parts if async_op else None, m_total)
    return handle if async_op else handle.wait()


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
