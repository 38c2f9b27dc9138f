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

import threading
from collections import OrderedDict

import torch

from . import ops

_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream, torch.cuda.Stream]] = {}


def _streams(idx: int) -> tuple[torch.cuda.Stream, torch.cuda.Stream, torch.cuda.Stream]:
    """Per device: the host->device copy stream, the device->host copy stream and
    the stream graphs are captured on."""
    s = _STREAMS.get(idx)
    if s is None:
        dev = torch.device("cuda", idx)
        s = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
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


def _enqueue(x_host, weight, weight_scale, bias, out_dtype, out, group_size, rows_per_chunk, dev, idx):
    """Enqueue the chunked pipeline; returns the device tensors it uses, which the
    caller keeps until its current stream has joined both copy streams (so none
    of their memory is reused while a copy still reads it)."""
    m, k = x_host.shape
    cur = torch.cuda.current_stream(idx)
    s_in, s_out, _ = _streams(idx)
    # Both copy streams start after whatever the caller enqueued before.
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    x_dev = torch.empty((m, k), dtype=x_host.dtype, device=dev)
    held = [x_dev]
    for r0, r1 in _chunks(m, rows_per_chunk):
        with torch.cuda.stream(s_in):
            x_dev[r0:r1].copy_(x_host[r0:r1], non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(s_in)
        cur.wait_event(loaded)
        xq, xs = ops.rotate_quant(x_dev[r0:r1], group_size)
        y = ops.int8_gemm_dequant(xq, xs, weight, weight_scale, bias, out_dtype)
        held += [xq, xs, y]
        done = torch.cuda.Event()
        done.record(cur)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            out[r0:r1].copy_(y, non_blocking=True)
    cur.wait_stream(s_out)
    return held


_GRAPHS: OrderedDict = OrderedDict()
_GRAPH_CACHE_SIZE = 4
_GRAPH_LOCK = threading.Lock()


def int8_linear_host(x_host: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                     out: torch.Tensor | None = None, *, group_size: int = 256,
                     rows_per_chunk: int = 1024, graph: bool = False) -> torch.Tensor:
    """``int8_linear(x, weight, weight_scale, bias, out_dtype, convrot=True)`` with ``x`` and
    the result in host memory.

    ``x_host [M, K]`` fp16/bf16 on the CPU (pinned, for the copies to overlap);
    ``weight [N, K]`` int8 and ``weight_scale`` (scalar or ``[N]``) on the CUDA device
    that runs the linear; ``out`` an optional ``[M, N]`` ``out_dtype`` CPU tensor
    (pinned) to write into, else one is allocated (pinned).  Returns ``out``.

    ``graph=True`` replays the whole chunked pipeline as one CUDA graph, so a call
    costs one launch on the host instead of a few dozen API calls per chunk: the
    first call with a given set of buffers (x_host, out, weight, scales, bias:
    addresses, shapes and dtypes) runs eagerly and captures the graph, later calls
    with the same buffers replay it (it reads whatever they hold then).  Up to four
    graphs are kept, each holding its device buffers (its split-K scratch
    included, so different graphs may be replayed concurrently; one graph's
    replays must not overlap each other, like any CUDA graph's).
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
    if graph and not x_host.is_contiguous():
        raise ValueError("int8_linear_host: graph=True needs a contiguous x_host (its address is captured)")
    x_host = x_host.contiguous()
    dev = weight.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    args = (x_host, weight, weight_scale, bias, out_dtype, out, group_size, rows_per_chunk, dev, idx)
    with torch.cuda.device(idx):
        if not graph:
            _enqueue(*args)
            return out
        key = (idx, x_host.data_ptr(), tuple(x_host.shape), x_host.dtype, out.data_ptr(), out_dtype,
               weight.data_ptr(), tuple(weight.shape), weight_scale.data_ptr(), weight_scale.numel(),
               weight_scale.dtype, weight_scale.device, None if bias is None else
               (bias.data_ptr(), bias.numel(), bias.dtype, bias.device), group_size, rows_per_chunk)
        with _GRAPH_LOCK:
            entry = _GRAPHS.get(key)
            if entry is not None:
                _GRAPHS.move_to_end(key)
        if entry is not None:
            entry[0].replay()
            return out
        # First call: run it eagerly on the capture stream (one-time launch
        # set-up, and any split-K scratch, which is cached per stream, is made
        # and zeroed outside the capture), then capture the same sequence there.
        # The graph gets a split-K scratch of its own: the capture stream's
        # cached one is dropped from the cache before the eager run and the new
        # one taken out of it after the capture, so graphs replayed at the same
        # time on different streams never share a scratch.
        cur = torch.cuda.current_stream(idx)
        cap = _streams(idx)[2]
        ws_key = (idx, cap.cuda_stream)
        ops._SPLITK_WS.pop(ws_key, None)
        cap.wait_stream(cur)
        with torch.cuda.stream(cap):
            _enqueue(*args)
        cur.wait_stream(cap)
        torch.cuda.synchronize(idx)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            held = _enqueue(*args)
        scratch = ops._SPLITK_WS.pop(ws_key, None)
        if scratch is not None:
            held.append(scratch)  # the graph's kernels use this very buffer, and only this graph
        with _GRAPH_LOCK:
            _GRAPHS[key] = (g, held)
            while len(_GRAPHS) > _GRAPH_CACHE_SIZE:
                _GRAPHS.popitem(last=False)
    return out
