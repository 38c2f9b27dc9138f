"""Standalone ComfyUI nodes for INT8 ConvRot (API of tilegen/comfyui/nodes.py).

Typical wiring::

    weight (fp16) -> QuantizeConvRotWeight -> (wq, wscale)
    activation (fp16) -> Int8ConvRotLinear(wq, wscale) -> output (fp16)
"""
from __future__ import annotations

import logging
import os

import torch

from ..kernels.hadamard import build_hadamard
from ..kernels.int8_convrot import _eager_quantize, can_use_fht, quantize_convrot_fht
from ..quant.int8_ops import int8_matmul_dequant_chunked
from ..quant.weight import quantize_convrot_weight

LOGGER = logging.getLogger("tilegen.nodes")


class TileGenConvRotModelConfig:
    """MODEL passthrough that sets the TILEGEN_* runtime variables from a workflow."""

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
        os.environ["TILEGEN_CONVROT_BACKEND"] = backend
        os.environ["TILEGEN_FHT_MIN_K"] = str(max(0, int(fht_min_k)))
        os.environ["TILEGEN_FHT_IMPL"] = fht_impl
        os.environ["TILEGEN_INT8_TEMP_MB"] = str(max(16, int(int8_temp_mb)))
        os.environ["TILEGEN_DIAGNOSTICS"] = "1" if diagnostics else "0"
        LOGGER.warning("tilegen workflow config: backend=%s min_k=%s impl=%s temp=%sMiB diagnostics=%s",
                       backend, fht_min_k, fht_impl, int8_temp_mb, diagnostics)
        return (model,)


class ConvRotTestTensors:
    """Deterministic (x, weight) tensors for a standalone ConvRot test graph."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "rows": ("INT", {"default": 32, "min": 1, "max": 4096, "step": 1}),
                "in_features": ("INT", {"default": 5120, "min": 4, "max": 32768, "step": 4}),
                "out_features": ("INT", {"default": 256, "min": 1, "max": 32768, "step": 1}),
                "group_size": ("INT", {"default": 256, "min": 4, "max": 1024, "step": 4}),
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
        if in_features % group_size != 0:
            raise ValueError(f"in_features={in_features} must be divisible by group_size={group_size}")
        build_hadamard(group_size, "cpu", torch.float32)  # validates the group size
        dev = ("cuda" if torch.cuda.is_available() else "cpu") if device == "auto" else device
        if dev == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("CUDA was requested but torch.cuda.is_available() is false")
        dt = torch.float16 if dtype == "float16" else torch.bfloat16
        g = torch.Generator(device=dev)
        g.manual_seed(int(seed))
        x = torch.randn((rows, in_features), generator=g, device=dev, dtype=dt)
        w = torch.randn((out_features, in_features), generator=g, device=dev, dtype=dt) * 0.02
        return (x, w)


class QuantizeConvRotWeight:
    """Offline weight quantisation: group-Hadamard rotation + per-channel int8."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"weight": ("TENSOR",),
                             "group_size": ("INT", {"default": 256, "min": 4, "max": 1024, "step": 4})}}

    RETURN_TYPES = ("TENSOR", "TENSOR")
    RETURN_NAMES = ("weight_quantized", "weight_scale")
    FUNCTION = "quantize"
    CATEGORY = "quantization/convrot"

    def quantize(self, weight: torch.Tensor, group_size: int):
        return quantize_convrot_weight(weight, group_size)


class Int8ConvRotLinear:
    """INT8 ConvRot linear: fused rotate+quant -> fused INT8 GEMM + dequant."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "x": ("TENSOR",),
                "weight_quantized": ("TENSOR",),
                "weight_scale": ("TENSOR",),
                "group_size": ("INT", {"default": 256, "min": 4, "max": 1024, "step": 4}),
            },
            "optional": {"bias": ("TENSOR",), "backend": (["auto", "fht", "eager"], {"default": "auto"})},
        }

    RETURN_TYPES = ("TENSOR",)
    RETURN_NAMES = ("output",)
    FUNCTION = "forward"
    CATEGORY = "quantization/convrot"

    def forward(self, x, weight_quantized, weight_scale, group_size, bias=None, backend="auto"):
        shape = tuple(x.shape)
        x2d = x.reshape(-1, x.shape[-1]).contiguous()
        k = x2d.shape[1]
        n = weight_quantized.shape[0]
        if k % group_size != 0:
            raise ValueError(f"K={k} must be divisible by group_size={group_size}")
        # The environment variable overrides the node input (nodes.py:180).
        mode = os.environ.get("TILEGEN_CONVROT_BACKEND", backend).strip().lower()
        if mode in {"auto", "fht"} and self._can_use_fht(x2d, group_size, mode):
            try:
                xq, xscale = quantize_convrot_fht(x2d, group_size)
            except Exception as e:  # pragma: no cover
                print(f"[Int8ConvRotLinear] FHT failed, using eager: {e}")
                xq, xscale = _eager_quantize(x2d, group_size)
        else:
            xq, xscale = _eager_quantize(x2d, group_size)
        wq = weight_quantized.to(device=x.device, dtype=torch.int8)
        out = int8_matmul_dequant_chunked(xq, xscale, wq, weight_scale, bias, x.dtype)
        return (out.reshape(*shape[:-1], n),)

    @staticmethod
    def _can_use_fht(x: torch.Tensor, group_size: int, mode: str) -> bool:
        min_k = 0
        if mode == "auto":
            from .backend import _fht_min_k

            min_k = _fht_min_k(x.device.index or 0) if x.is_cuda else 0
        return can_use_fht(x, group_size, min_k=min_k)
