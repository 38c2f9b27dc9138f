from __future__ import annotations

import torch

from .._activations import apply_input_act


def _int8_matmul_accumulate(a, b):
    return torch._int_mm(a, b)


def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False, convrot_groupsize=256,
                input_act=None):
    """Plain torch int8 linear: optional activation, (ConvRot) row-wise quant, int8 GEMM, dequant."""
    out_dtype = out_dtype or x.dtype
    x = apply_input_act(x, input_act)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if convrot:
        from tilegen_b200.kernels.hadamard import build_hadamard

        g = convrot_groupsize
        h = build_hadamard(g, x2.device, x2.dtype)
        x2 = torch.matmul(x2.reshape(x2.shape[0], -1, g), h).reshape(x2.shape)
    xs = (x2.abs().amax(-1).float() / 127.0).clamp_min(1e-30)
    xq = torch.round(x2 / xs[:, None].to(x2.dtype)).clamp(-128, 127).to(torch.int8)
    acc = _int8_matmul_accumulate(xq, weight.t()).float()
    out = acc * xs[:, None] * weight_scale.float().reshape(1, -1)
    if bias is not None:
        out = out + bias.float()
    return out.to(out_dtype).reshape(*shape[:-1], weight.shape[0])
