"""Standalone ComfyUI nodes for INT8 ConvRot (API of tilegen/comfyui/nodes.py).

Typical wiring::

    weight (fp16) -> QuantizeConvRotWeight -> (wq, wscale)
    activation (fp16) -> Int8ConvRotLinear(wq, wscale) -> output (fp16)

Class names, ``INPUT_TYPES``, return types and categories are the ComfyUI
workflow format of the reference's nodes.  The linear node asks the same
decision function as the selective backend (``backend.kernel_refusal``) whether
the rotate+quant kernel serves its input.
"""
from __future__ import annotations

import logging
import os

import torch

from ..kernels.hadamard import build_hadamard
from ..quant.int8_ops import int8_matmul_dequant_chunked
from ..quant.weight import quantize_convrot_weight
from . import backend

LOGGER = logging.getLogger("tilegen.nodes")

_GROUP_INPUT = ("INT", {"default": 256, "min": 4, "max": 1024, "step": 4})


class TileGenConvRotModelConfig:
    """MODEL passthrough that writes the TILEGEN_* runtime variables from a workflow."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "model": ("MODEL",),
                "backend": (["auto", "fht", "off"], {"default": "auto"}),
                "fht_min_k": ("INT", {"default": 8192, "min": 0, "max": 32768, "step": 256}),
                "fht_impl": (["native", "tilelang"], {"default": "native"}),
                "int8_temp_mb": ("INT", {"default": 1024, "min": 16, "max": 8192, "step": 16}),
                "diagnostics": ("BOOLEAN", {"default": True}),
            }
        }

    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "configure"
    CATEGORY = "model/optimization/tilegen"

    def configure(self, model, backend, fht_min_k, fht_impl, int8_temp_mb, diagnostics):
        settings = {
            "TILEGEN_CONVROT_BACKEND": backend,
            "TILEGEN_FHT_MIN_K": str(max(0, int(fht_min_k))),
            "TILEGEN_FHT_IMPL": fht_impl,
            "TILEGEN_INT8_TEMP_MB": str(max(16, int(int8_temp_mb))),
            "TILEGEN_DIAGNOSTICS": "1" if diagnostics else "0",
        }
        os.environ.update(settings)
        LOGGER.warning("tilegen workflow config: backend=%s min_k=%s impl=%s temp=%sMiB diagnostics=%s",
                       backend, fht_min_k, fht_impl, int8_temp_mb, diagnostics)
        return (model,)


def _resolve_device(choice: str) -> str:
    cuda = torch.cuda.is_available()
    if choice == "auto":
        return "cuda" if cuda else "cpu"
    if choice == "cuda" and not cuda:
        raise RuntimeError("CUDA was requested but torch.cuda.is_available() is false")
    return choice


class ConvRotTestTensors:
    """Seeded (x, weight) tensors that make a standalone ConvRot test branch runnable."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "rows": ("INT", {"default": 32, "min": 1, "max": 4096, "step": 1}),
                "in_features": ("INT", {"default": 5120, "min": 4, "max": 32768, "step": 4}),
                "out_features": ("INT", {"default": 256, "min": 1, "max": 32768, "step": 1}),
                "group_size": _GROUP_INPUT,
                "seed": ("INT", {"default": 20260726, "min": 0, "max": 0x7FFFFFFFFFFFFFFF}),
                "dtype": (["float16", "bfloat16"], {"default": "float16"}),
                "device": (["auto", "cuda", "cpu"], {"default": "auto"}),
            },
        }

    RETURN_TYPES = ("TENSOR", "TENSOR")
    RETURN_NAMES = ("x", "weight")
    FUNCTION = "create"
    CATEGORY = "quantization/convrot/testing"

    def create(self, rows, in_features, out_features, group_size, seed, dtype, device):
        if in_features % group_size:
            raise ValueError(f"in_features={in_features} must be divisible by group_size={group_size}")
        build_hadamard(group_size, "cpu", torch.float32)  # raises for a group that is not a power of four
        dev = _resolve_device(device)
        dt = {"float16": torch.float16, "bfloat16": torch.bfloat16}[dtype]
        gen = torch.Generator(device=dev).manual_seed(int(seed))
        # x first, then the weight, from one generator (N(0,1) and N(0, 0.02)).
        x = torch.randn((rows, in_features), generator=gen, device=dev, dtype=dt)
        w = torch.randn((out_features, in_features), generator=gen, device=dev, dtype=dt) * 0.02
        return (x, w)


class QuantizeConvRotWeight:
    """Offline weight quantisation: group-Hadamard rotation + per-channel int8."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"weight": ("TENSOR",), "group_size": _GROUP_INPUT}}

    RETURN_TYPES = ("TENSOR", "TENSOR")
    RETURN_NAMES = ("weight_quantized", "weight_scale")
    FUNCTION = "quantize"
    CATEGORY = "quantization/convrot"

    def quantize(self, weight: torch.Tensor, group_size: int):
        return quantize_convrot_weight(weight, group_size)


class Int8ConvRotLinear:
    """INT8 ConvRot linear: rotate+quant of the activations, then the INT8 GEMM + dequant.

    The mode is TILEGEN_CONVROT_BACKEND when set, else the node's ``backend``
    input.  The node's ``auto`` threshold is TILEGEN_FHT_MIN_K, else 8192 (5120
    on sm_75) on pre-Blackwell GPUs and 0 on Blackwell, as the backend's.
    """

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "x": ("TENSOR",),
                "weight_quantized": ("TENSOR",),
                "weight_scale": ("TENSOR",),
                "group_size": _GROUP_INPUT,
            },
            "optional": {"bias": ("TENSOR",), "backend": (["auto", "fht", "eager"], {"default": "auto"})},
        }

    RETURN_TYPES = ("TENSOR",)
    RETURN_NAMES = ("output",)
    FUNCTION = "forward"
    CATEGORY = "quantization/convrot"

    def forward(self, x, weight_quantized, weight_scale, group_size, bias=None, backend="auto"):
        k = x.shape[-1]
        if k % group_size:
            raise ValueError(f"K={k} must be divisible by group_size={group_size}")
        mode = os.environ.get("TILEGEN_CONVROT_BACKEND", backend).strip().lower()
        xq, xscale = _node_quantise(x.reshape(-1, k).contiguous(), group_size, mode)
        wq = weight_quantized.to(device=x.device, dtype=torch.int8)
        y = int8_matmul_dequant_chunked(xq, xscale, wq, weight_scale, bias, x.dtype)
        return (y.reshape(*x.shape[:-1], wq.shape[0]),)


def _node_quantise(x2d: torch.Tensor, group_size: int, mode: str):
    # "eager" (or anything but auto/fht) makes kernel_refusal decline, so the
    # eager rotation runs, as in the reference node.
    return backend.quantise_activations(x2d, group_size, None, mode if mode in ("auto", "fht") else "eager")
