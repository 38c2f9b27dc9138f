"""ConvRot activation quantiser (API of tilegen/kernels/int8_convrot.py).

``quantize_convrot_fht`` / ``quantize_convrot_native`` run the prebuilt sm_100a
rotate+quant kernel (``tg_quantize_act``), which replaces the reference's NVRTC
kernel (int8_convrot.py:41-230): the same rotation, row absmax, scale and
rounding, no JIT and no per-K module cache.  Differences, by design:

* bf16 input is read directly instead of being cast to fp16 first
  (int8_convrot.py:204-206), which matches ``_eager_quantize(x.float(), G)``.
* ``quantize_convrot_native`` also serves groups 4, 16 and 64 (the reference
  kernel only does 256); 128 is rejected as in the reference (not a power of
  four).  ``can_use_fht`` keeps the reference's rule (group 256 only), so
  ``quantize_convrot`` sends the other groups to the eager path, in ``x``'s
  dtype, exactly as the reference does.
* the rotation's fp32 sums run in a shorter order than the reference
  kernel's (``ops.ROTATION_ORDERS``): codes can differ by one at rounding ties
  (about 1e-6 of them), within the parity tolerance;
  ``ops.rotate_quant(x, G, order="reference")`` gives the reference kernel's
  bits.
* the ``tilelang`` implementation choice (``TILEGEN_FHT_IMPL``) has no separate
  lowering here; the native kernel serves it.

``quantize_convrot`` keeps the reference's dispatch (int8_convrot.py:271-286):
the FHT kernel when ``can_use_fht`` accepts the input, else the eager torch
path, including the fallback when the kernel raises for a shape (logged).  A
missing native library is not such a failure: it raises.
"""
from __future__ import annotations

import logging
import os

import torch

from .. import ops
from .hadamard import build_hadamard

LOGGER = logging.getLogger("tilegen")

KERNEL_GROUP_SIZE = 256
NATIVE_GROUP_SIZES = (4, 16, 64, 256)


def quantize_convrot_native(x: torch.Tensor, group_size: int = 256):
    """Fused rotate+quant on the prebuilt sm_100a kernel -> ``(xq int8, xscale fp32)``."""
    if group_size not in NATIVE_GROUP_SIZES:
        raise ValueError(f"the radix-4 kernel supports group_size in {NATIVE_GROUP_SIZES}, got {group_size}")
    if x.ndim != 2:
        raise ValueError(f"expected 2-D input, got {tuple(x.shape)}")
    if not x.is_cuda:
        raise ValueError("CUDA tensor required")
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    if x.shape[1] % 256:
        raise ValueError(f"K={x.shape[1]} not divisible by 256")
    return ops.rotate_quant(x, group_size)


_WARNED_IMPL = False


def _impl_choice() -> str:
    return os.environ.get("TILEGEN_FHT_IMPL", "native").strip().lower()


def quantize_convrot_fht(x: torch.Tensor, group_size: int = 256):
    """Apply the radix-4 fused activation quantiser (FHT) to a 2-D tensor."""
    global _WARNED_IMPL
    if _impl_choice() == "tilelang" and not _WARNED_IMPL:
        _WARNED_IMPL = True
        LOGGER.warning("TILEGEN_FHT_IMPL=tilelang: no tilelang lowering on sm_100a; using the native kernel")
    return quantize_convrot_native(x, group_size)


def can_use_fht(x: torch.Tensor, group_size: int, min_k: int = 0) -> bool:
    """Whether the FHT kernel handles ``x`` (``min_k``: smallest K worth it; 0 = any)."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16):
        return False
    if group_size != KERNEL_GROUP_SIZE or x.shape[-1] % 256:
        return False
    if x.shape[-1] < min_k:
        return False
    return x.shape[-1] <= ops.rotate_quant_max_k()


def quantize_convrot(x: torch.Tensor, group_size: int = 256, backend: str = "auto", min_k: int = 0):
    """Quantise ``x`` with ConvRot: FHT kernel when supported, else eager.

    ``backend``: ``"auto"`` (FHT when supported and K >= min_k), ``"fht"`` (FHT
    whenever supported), ``"eager"`` (pure torch).
    """
    backend = backend.strip().lower()
    if backend in ("auto", "fht") and can_use_fht(x, group_size, min_k=min_k if backend == "auto" else 0):
        try:
            return quantize_convrot_fht(x, group_size)
        except Exception:
            LOGGER.exception("FHT failed for shape %s; using eager ConvRot", tuple(x.shape))
    return _eager_quantize(x, group_size)


def _eager_quantize(x: torch.Tensor, group_size: int):
    """Pure-torch ConvRot quantisation in ``x.dtype`` (int8_convrot.py:289-302)."""
    if x.ndim != 2:
        raise ValueError(f"expected 2-D input, got {tuple(x.shape)}")
    m, k = x.shape
    h = build_hadamard(group_size, x.device, x.dtype)
    rot = torch.matmul(x.reshape(m, k // group_size, group_size), h).reshape(m, k)
    scale = (rot.abs().amax(dim=-1).float() / 127.0).clamp_min(1e-30)
    q = torch.round(rot / scale[:, None].to(rot.dtype)).clamp(-128, 127).to(torch.int8)
    return q, scale
