"""Rotation-free row-wise INT8 activation quantisation.

The ``else`` branch of the production wrapper (tilegen/comfyui/backend.py:230-232)
as a function, with the input activation of backend.py:201-204 folded in:

    xscale = (x.abs().amax(dim=-1).float() / 127.0).clamp_min(1e-30)
    xq = torch.round(x / xscale[:, None].to(x.dtype)).clamp(-128, 127).to(torch.int8)

On a CUDA fp16/bf16 input whose K is a multiple of 64 (at most
``rotate_quant_max_k()``) it is one pass of the quantiser kernel
(``tg_quantize_act`` with group 1), which evaluates those two lines exactly as
torch does on the GPU; anything else runs the two lines in torch.  The
reference itself reaches this branch only through that wrapper (it has no
public function for it).
"""
from __future__ import annotations

import torch

from .. import ops


def _torch_rowwise(x: torch.Tensor):
    xscale = (x.abs().amax(dim=-1).float() / 127.0).clamp_min(1e-30)
    xq = torch.round(x / xscale[:, None].to(x.dtype)).clamp(-128, 127).to(torch.int8)
    return xq, xscale


def kernel_accepts(x: torch.Tensor, input_act: str | None = None) -> bool:
    """Whether ``quantize_rowwise`` runs ``x`` on the kernel."""
    act_ok = input_act in (None, "none") or input_act in ops.FUSED_ACTS
    return (act_ok and x.is_cuda and x.ndim == 2 and x.dtype in (torch.float16, torch.bfloat16)
            and x.shape[1] % 64 == 0 and 0 < x.shape[1] <= ops.rotate_quant_max_k())


def quantize_rowwise(x: torch.Tensor, input_act: str | None = None):
    """``input_act`` then row-wise symmetric int8 of a 2-D ``x`` -> ``(xq int8, xscale fp32)``."""
    if x.ndim != 2:
        raise ValueError(f"expected 2-D input, got {tuple(x.shape)}")
    if kernel_accepts(x, input_act):
        return ops.quantize_act(x, 1, input_act)
    if input_act not in (None, "none"):
        from comfy_kitchen.backends._activations import apply_input_act

        x = apply_input_act(x, input_act)
    return _torch_rowwise(x)
