"""The int8_convrot linear for activations and outputs in host memory.

``int8_linear_host`` runs the same two kernels as the device path (rotate+quant,
then the INT8 GEMM + dequant; tilegen/comfyui/backend.py:166-244 with
``convrot=True``) on an ``x`` that lives in pinned host memory, and writes the
output to pinned host memory.  The rows go in chunks (growing to
``rows_per_chunk``) over three CUDA streams: chunk i's host->device copy, chunk
i-1's kernels and chunk i-2's device->host copy run at the same time, so a call
costs about the larger of the two PCIe transfers instead of their sum plus the
kernels.  PCIe is full duplex, and the
two copy directions use separate copy engines.

The call is asynchronous like a CUDA op: it returns once everything is
enqueued, and its end is ordered on the caller's current stream (synchronise
that stream before reading ``out`` on the host; do not modify ``x_host``
before then).  Every chunk's result is bit-identical to the device path on
the same rows (the quantiser is per row and the GEMM's rows are independent).
"""
from __future__ import annotations

import torch

from . import ops

_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}


def _copy_streams(idx: int) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
    s = _STREAMS.get(idx)
    if s is None:
        dev = torch.device("cuda", idx)
        s = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
        _STREAMS[idx] = s
    return s


def _chunks(m: int, rows: int):
    """Row ranges: a quarter chunk, a half chunk, then full chunks.  The small
    first chunks start the device->host stream sooner (its copies are the long
    pole); full-size chunks after that keep the per-chunk host overhead low."""
    r0, size = 0, max(1, rows // 4)
    while r0 < m:
        r1 = min(r0 + size, m)
        yield r0, r1
        r0, size = r1, min(rows, size * 2)


def int8_linear_host(x_host: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                     out: torch.Tensor | None = None, *, group_size: int = 256,
                     rows_per_chunk: int = 1024) -> torch.Tensor:
    """``int8_linear(x, weight, weight_scale, bias, out_dtype, convrot=True)`` with ``x`` and
    the result in host memory.

    ``x_host [M, K]`` fp16/bf16 on the CPU (pinned, for the copies to overlap);
    ``weight [N, K]`` int8 and ``weight_scale`` (scalar or ``[N]``) on the CUDA device
    that runs the linear; ``out`` an optional ``[M, N]`` ``out_dtype`` CPU tensor
    (pinned) to write into, else one is allocated (pinned).  Returns ``out``.
    """
    if x_host.is_cuda:
        raise ValueError("int8_linear_host: x_host must be in host memory (use int8_linear for CUDA tensors)")
    if not weight.is_cuda:
        raise ValueError("int8_linear_host: the int8 weight must be on the CUDA device that runs the linear")
    if x_host.ndim != 2 or x_host.shape[1] != weight.shape[1]:
        raise ValueError(f"int8_linear_host: shapes {tuple(x_host.shape)} x {tuple(weight.shape)}^T do not match")
    if x_host.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"int8_linear_host: fp16/bf16 input required, got {x_host.dtype}")
    if rows_per_chunk < 1:
        raise ValueError("int8_linear_host: rows_per_chunk must be positive")
    m, k = x_host.shape
    n = weight.shape[0]
    out_dtype = out_dtype or x_host.dtype
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (m, n) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError(f"int8_linear_host: out must be a contiguous host [{m}, {n}] {out_dtype} tensor")
    if m == 0:
        return out
    x_host = x_host.contiguous()
    dev = weight.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    with torch.cuda.device(idx):
        cur = torch.cuda.current_stream(idx)
        s_in, s_out = _copy_streams(idx)
        # Both copy streams start after whatever the caller enqueued before.
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_in):
            x_dev = torch.empty((m, k), dtype=x_host.dtype, device=dev)
        for r0, r1 in _chunks(m, rows_per_chunk):
            with torch.cuda.stream(s_in):
                x_dev[r0:r1].copy_(x_host[r0:r1], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(s_in)
            cur.wait_event(loaded)
            xq, xs = ops.rotate_quant(x_dev[r0:r1], group_size)
            y = ops.int8_gemm_dequant(xq, xs, weight, weight_scale, bias, out_dtype)
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                out[r0:r1].copy_(y, non_blocking=True)
            y.record_stream(s_out)  # the allocator keeps y until its copy has run
        x_dev.record_stream(cur)
        cur.wait_stream(s_out)
    return out
