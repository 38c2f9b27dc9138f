"""INT8 GEMM + dequant (API of tilegen/quant/int8_ops.py).

On CUDA tensors ``int8_matmul_dequant_chunked`` is one launch of the fused
tcgen05 GEMM (``tg_int8_gemm_dequant``): the int32 accumulators stay in tensor
memory and the dequantisation runs in the epilogue, so there is no
``[chunk, N]`` temporary and ``max_temp_bytes`` has nothing to bound (it is
accepted for compatibility).  The result is bit-identical to the reference's
``_int_mm`` + ``float()`` + ``mul_`` + ``mul_`` + ``add_`` + ``copy_`` sequence.

CPU tensors take the reference's torch sequence (``torch._int_mm`` per row
chunk), which is what the reference does on any device.
"""
from __future__ import annotations

import torch

from .. import ops


def _int8_matmul_accumulate():
    """The int8 matmul primitive of the torch path (comfy_kitchen's if installed)."""
    try:
        from comfy_kitchen.backends.eager.quantization import _int8_matmul_accumulate as fn
        return fn
    except ImportError:
        return torch._int_mm


def int8_matmul_dequant_chunked(
    xq: torch.Tensor,
    xscale: torch.Tensor,
    wq: torch.Tensor,
    wscale: torch.Tensor,
    bias: torch.Tensor | None,
    out_dtype: torch.dtype,
    max_temp_bytes: int = 256 * 1024 * 1024,
) -> torch.Tensor:
    """``out = float(xq @ wq.T) * xscale[:, None] * wscale[None, :] (+ bias)``.

    Args:
        xq: [M, K] int8 activation.
        xscale: [M] float32 per-row activation scale.
        wq: [N, K] int8 weight.
        wscale: [N] or scalar float32 weight scale.
        bias: optional [N] bias.
        out_dtype: output dtype (fp16/bf16/fp32).
        max_temp_bytes: row-chunk cap of the torch path's int32/fp32 temporaries.
    """
    n = wq.shape[0]
    if wscale.numel() not in (1, n):
        raise ValueError(f"weight scale must be scalar or length {n}, got {tuple(wscale.shape)}")
    if xq.is_cuda:
        return ops.int8_gemm_dequant(xq, xscale, wq, wscale, bias, out_dtype)
    return _torch_chunked(xq, xscale, wq, wscale, bias, out_dtype, max_temp_bytes)


def _torch_chunked(xq, xscale, wq, wscale, bias, out_dtype, max_temp_bytes):
    """The reference's row-chunked torch sequence (int8_ops.py:47-70)."""
    m, n = xq.shape[0], wq.shape[0]
    rows = max(1, min(m, max_temp_bytes // max(1, n * 8)))
    wt = wq.t()
    ws = wscale.to(device=xq.device, dtype=torch.float32).reshape(1, -1)
    mm = _int8_matmul_accumulate()
    out = torch.empty((m, n), device=xq.device, dtype=out_dtype)
    b = None if bias is None else bias.to(device=xq.device, dtype=torch.float32).reshape(1, -1)
    for s in range(0, m, rows):
        e = min(s + rows, m)
        part = mm(xq[s:e], wt).float()
        part.mul_(xscale[s:e].float().reshape(-1, 1))
        part.mul_(ws)
        if b is not None:
            part.add_(b)
        out[s:e].copy_(part)
    return out
