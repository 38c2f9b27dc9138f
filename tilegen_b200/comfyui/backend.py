"""Selective comfy_kitchen ConvRot backend (API of tilegen/comfyui/backend.py).

``install()`` registers a backend named ``tilegen`` ahead of comfy_kitchen's
other backends for ``int8_linear``.  Its call rule ``_fht_applicable`` accepts
only the ConvRot calls the sm_100a kernels serve; anything else falls through
to the next backend.  An accepted call runs ``int8_linear``: the rotate+quant
kernel on the activations (with a ``gelu``/``gelu_tanh`` input activation
applied inside it), then the tcgen05 INT8 GEMM with the dequantisation in its
epilogue.

One decision function, ``kernel_refusal``, says whether the kernel serves an
activation tensor and, if not, why; the registry rule, ``int8_linear`` and the
standalone linear node all ask it, so they cannot disagree.

Environment (the reference's names and meanings, backend.py:39-78):
``TILEGEN_CONVROT_BACKEND`` in {auto, fht, eager, off}; ``TILEGEN_FHT_MIN_K``
(default: 0 on compute capability 10.x and newer, where the kernel is faster
at every K; 5120 on sm_75; 8192 elsewhere); ``TILEGEN_INT8_TEMP_MB`` (accepted;
the fused GEMM needs no temporary); ``TILEGEN_DIAGNOSTICS``.
"""
from __future__ import annotations

import logging
import os
import sys
from collections.abc import Mapping

import torch

from ..quant.int8_ops import int8_matmul_dequant_chunked

LOGGER = logging.getLogger("tilegen.backend")

BACKEND_NAME = "tilegen"
_INSTALLED = False
# (rows, K, dtype, device index) of inputs the kernel raised for: later calls
# of that shape go to the eager path without trying again.
_FAILED_FHT_SHAPES: set[tuple] = set()
_LOGGED_DECISIONS: set[tuple] = set()

_MODES = ("off", "auto", "fht", "eager")
_FALSE_WORDS = ("0", "false", "off", "no")


# ---------------------------------------------------------------- settings
def _mode() -> str:
    """TILEGEN_CONVROT_BACKEND, lower-cased; an unknown value reads as ``auto`` (logged)."""
    raw = os.environ.get("TILEGEN_CONVROT_BACKEND", "auto")
    mode = raw.strip().lower()
    if mode in _MODES:
        return mode
    LOGGER.warning("Unknown TILEGEN_CONVROT_BACKEND=%r; using auto", raw)
    return "auto"


def _default_fht_min_k(device_index: int = 0) -> int:
    """Smallest K at which ``auto`` uses the kernel when TILEGEN_FHT_MIN_K is unset."""
    try:
        major, minor = torch.cuda.get_device_capability(device_index) if torch.cuda.is_available() else (0, 0)
    except (AssertionError, RuntimeError):
        major, minor = 0, 0
    if major >= 10:
        return 0  # Blackwell: the fused kernel beats the eager path at every K
    return 5120 if (major, minor) == (7, 5) else 8192


def _fht_min_k(device_index: int = 0) -> int:
    raw = os.environ.get("TILEGEN_FHT_MIN_K")
    if raw is None:
        return _default_fht_min_k(device_index)
    try:
        return max(0, int(raw))
    except ValueError:
        fallback = _default_fht_min_k(device_index)
        LOGGER.warning("Invalid TILEGEN_FHT_MIN_K=%r; using %d", raw, fallback)
        return fallback


def _diagnostics_enabled() -> bool:
    return os.environ.get("TILEGEN_DIAGNOSTICS", "1").strip().lower() not in _FALSE_WORDS


def _temp_bytes() -> int:
    return max(16, int(os.environ.get("TILEGEN_INT8_TEMP_MB", "256"))) << 20


def _log_decision(decision: str, reason: str, x, weight, group_size: int) -> None:
    """One warning per distinct (decision, reason, shape, dtype, group), if diagnostics are on."""
    if not (_diagnostics_enabled() and isinstance(x, torch.Tensor) and x.ndim >= 2):
        return
    k = x.shape[-1]
    rows = x.numel() // max(1, k)
    n = weight.shape[0] if isinstance(weight, torch.Tensor) and weight.ndim == 2 else "?"
    key = (decision, reason, rows, k, n, x.dtype, group_size)
    if key not in _LOGGED_DECISIONS:
        _LOGGED_DECISIONS.add(key)
        LOGGER.warning("tilegen shape %s: M=%s K=%s N=%s dtype=%s group=%s reason=%s",
                       decision, rows, k, n, x.dtype, group_size, reason)


# ---------------------------------------------------------------- the decision
def kernel_refusal(x: torch.Tensor, group_size: int, mode: str, min_k: int | None = None):
    """``None`` when the rotate+quant kernel serves ``x`` in ``mode``, else
    ``(param, message, log_reason)``: the ValidationResult failure to report and
    the reason to log (``None``: not worth a log line).

    Checks, in order: mode; a CUDA fp16/bf16 tensor of two or more dims; group
    256 and K a multiple of 256 (the reference kernel's rule; other groups take
    the eager path in x's dtype, as in the reference); K at least ``min_k``
    (``auto`` only; default TILEGEN_FHT_MIN_K); K at most the kernel's maximum;
    the shape not one the kernel already failed on.
    """
    from ..kernels.int8_convrot import KERNEL_GROUP_SIZE
    from ..ops import rotate_quant_max_k

    if mode not in ("auto", "fht"):
        return "__tilegen__", f"mode={mode}", f"mode={mode}"
    if not (isinstance(x, torch.Tensor) and x.is_cuda and x.ndim >= 2):
        return "x", "CUDA tensor with at least 2 dims required", None
    if x.dtype not in (torch.float16, torch.bfloat16):
        return "x", "fp16/bf16 input required", None
    k = x.shape[-1]
    if group_size != KERNEL_GROUP_SIZE or k % KERNEL_GROUP_SIZE:
        return "convrot_groupsize", "requires group=256 and K divisible by 256", "unsupported group/K"
    if mode == "auto":
        floor = _fht_min_k(x.device.index or 0) if min_k is None else min_k
        if k < floor:
            return "x", "K below TileGen threshold", f"K below min_k={floor}"
    if k > rotate_quant_max_k():
        return "x", "K above the kernel's maximum", "K above the kernel's maximum"
    if (x.numel() // k, k, x.dtype, x.device.index) in _FAILED_FHT_SHAPES:
        return "x", "FHT previously failed for this shape", "FHT previously failed"
    return None


def _fht_applicable(kwargs: Mapping[str, object]):
    """Registry call rule: accept only the ConvRot calls the kernels serve."""
    from comfy_kitchen.constraints import ValidationResult

    if not kwargs.get("convrot", False):
        return ValidationResult.fail("convrot", "TileGen only handles ConvRot")
    x, weight = kwargs.get("x"), kwargs.get("weight")
    group_size = int(kwargs.get("convrot_groupsize", 256))
    mode = _mode()
    refusal = kernel_refusal(x, group_size, mode, min_k=0 if mode == "fht" else None)
    if refusal is None:
        _log_decision("ACCEPT_FHT", "all constraints passed", x, weight, group_size)
        return ValidationResult.ok()
    param, message, reason = refusal
    if reason is not None:
        _log_decision("KEEP_CUDA", reason, x, weight, group_size)
    return ValidationResult.fail(param, message)


# ---------------------------------------------------------------- the linear
def _unfused_act(x: torch.Tensor, act: str | None) -> torch.Tensor:
    """comfy_kitchen's ``apply_input_act`` (the reference applies it as its own op)."""
    if act is None:
        return x
    from comfy_kitchen.backends._activations import apply_input_act

    return apply_input_act(x, act)


def quantise_activations(x2d: torch.Tensor, group_size: int, act: str | None, mode: str):
    """``(xq, xscale)`` of ``act(x2d)``: on the kernel when ``kernel_refusal`` allows
    it (the activation fused into the quantiser when it is one of
    ``ops.FUSED_ACTS``), else -- or when the kernel raises, which is remembered
    for the shape -- the eager torch rotation in ``x2d``'s dtype."""
    from ..kernels.int8_convrot import _eager_quantize, quantize_convrot_fht
    from ..ops import FUSED_ACTS, quantize_act

    if kernel_refusal(x2d, group_size, mode, min_k=0 if mode == "fht" else None) is None:
        try:
            if act is None:
                return quantize_convrot_fht(x2d, group_size)
            if act in FUSED_ACTS:
                return quantize_act(x2d, group_size, act)
            return quantize_convrot_fht(_unfused_act(x2d, act), group_size)
        except Exception:
            _FAILED_FHT_SHAPES.add((x2d.shape[0], x2d.shape[1], x2d.dtype, x2d.device.index))
            LOGGER.exception("FHT failed for M=%d K=%d; using eager ConvRot", x2d.shape[0], x2d.shape[1])
    return _eager_quantize(_unfused_act(x2d, act), group_size)


def int8_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
    convrot: bool = False,
    convrot_groupsize: int = 256,
    input_act: str | None = None,
) -> torch.Tensor:
    """Backend-compatible replacement for comfy_kitchen's ``int8_linear``.

    Non-ConvRot layouts, and every call in ``eager`` mode, are comfy_kitchen's
    own eager ``int8_linear``.  ConvRot calls: ``act(x)`` rotated and quantised
    row-wise (``quantise_activations``), then the INT8 GEMM with the
    dequantisation fused, the output reshaped to ``x``'s leading dims.
    """
    k = x.shape[-1]
    if k != weight.shape[-1]:
        raise ValueError(f"input and weight inner dimensions differ: {k} != {weight.shape[-1]}")
    out_dtype = out_dtype or x.dtype
    mode = _mode()
    if not convrot or mode == "eager":
        from comfy_kitchen.backends.eager.quantization import int8_linear as kitchen_eager

        return kitchen_eager(x, weight, weight_scale, bias=bias, out_dtype=out_dtype, convrot=convrot,
                             convrot_groupsize=convrot_groupsize, input_act=input_act)
    if k % convrot_groupsize:
        raise ValueError(f"ConvRot group size {convrot_groupsize} does not divide K={k}")
    act = None if input_act in (None, "none") else input_act
    lead = x.shape[:-1]
    xq, xscale = quantise_activations(x.reshape(-1, k).contiguous(), convrot_groupsize, act, mode)
    wq = weight.to(device=x.device, dtype=torch.int8)
    y = int8_matmul_dequant_chunked(xq, xscale, wq, weight_scale, bias, out_dtype, max_temp_bytes=_temp_bytes())
    return y.reshape(*lead, wq.shape[0])


# ---------------------------------------------------------------- registration
def install() -> bool:
    """Register the selective backend ahead of the others.  False (nothing
    registered) when the mode is ``off`` or comfy_kitchen is unavailable."""
    global _INSTALLED
    if _INSTALLED:
        return True
    mode = _mode()
    if mode == "off":
        return False
    try:
        from comfy_kitchen.constraints import FunctionConstraints
        from comfy_kitchen.registry import registry

        eager = registry.get_constraints("eager", "int8_linear")
        if eager is None:
            raise RuntimeError("comfy_kitchen eager int8_linear constraints are unavailable")
        # The eager backend's parameter and device constraints, plus our rule.
        ours = FunctionConstraints(params=eager.params, default_devices=eager.default_devices,
                                   min_compute_capability=eager.min_compute_capability,
                                   call_rules=tuple(getattr(eager, "call_rules", ())) + (_fht_applicable,))
        registry.register(BACKEND_NAME, sys.modules[__name__], {"int8_linear": ours})
        registry.set_priority([BACKEND_NAME] + [b for b in registry._priority if b != BACKEND_NAME])
    except Exception:
        LOGGER.exception("tilegen: could not register the ConvRot backend")
        return False
    _INSTALLED = True
    dev = torch.cuda.current_device() if torch.cuda.is_available() else 0
    LOGGER.warning("tilegen selective FHT dispatch enabled: mode=%s FHT min K=%s temp=%s MiB priority=%s",
                   mode, 0 if mode == "fht" else _fht_min_k(dev), os.environ.get("TILEGEN_INT8_TEMP_MB", "256"),
                   registry._priority)
    return True
