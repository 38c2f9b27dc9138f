"""Offline weight-side ConvRot quantisation (API of tilegen/quant/weight.py).

Rotating W's rows by the group Hadamard and quantising each row (output
channel) with absmax/127 is the same operation as the activation quantiser, so
CUDA fp16/bf16 weights go through the same sm_100a kernel: a 5120 x 13824
weight quantises in well under a millisecond.  fp32 (or CPU) weights take the
reference's torch sequence (weight.py:33-39) in the weight's dtype.  The output
layout is the reference's: int8 [N, K] and fp32 [N].
"""
from __future__ import annotations

import torch

from ..kernels.hadamard import build_hadamard, rotate_by_group
from ..kernels.int8_convrot import NATIVE_GROUP_SIZES
from .. import ops


def quantize_convrot_weight(weight: torch.Tensor, group_size: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate by group Hadamard + per-channel int8 -> ``(wq [N, K] int8, wscale [N] fp32)``."""
    if weight.ndim != 2:
        raise ValueError(f"weight must be 2D [N,K], got {tuple(weight.shape)}")
    n, k = weight.shape
    if k % group_size != 0:
        raise ValueError(f"K={k} must be divisible by group_size={group_size}")
    if (weight.is_cuda and weight.dtype in (torch.float16, torch.bfloat16)
            and group_size in NATIVE_GROUP_SIZES and k % 256 == 0 and k <= ops.rotate_quant_max_k()):
        return ops.rotate_quant(weight, group_size)
    h = build_hadamard(group_size, weight.device, weight.dtype)
    wrot = rotate_by_group(weight, h, group_size)
    wabs = wrot.abs().amax(dim=-1, keepdim=True)
    wscale = (wabs.float() / 127.0).clamp(min=1e-30)
    wq = torch.round(wrot / wscale.to(wrot.dtype)).clamp(-128, 127).to(torch.int8)
    return wq, wscale.reshape(n)
