"""ComfyUI integration (API of tilegen/comfyui).

Node mappings for the standalone ConvRot nodes, and the selective
comfy_kitchen backend, registered at import unless
``TILEGEN_CONVROT_BACKEND=off`` (a no-op returning False without comfy_kitchen).
"""
from __future__ import annotations

import logging
import os

LOGGER = logging.getLogger("tilegen")

NODE_CLASS_MAPPINGS: dict = {}
NODE_DISPLAY_NAME_MAPPINGS: dict = {}

try:
    from .nodes import ConvRotTestTensors, Int8ConvRotLinear, QuantizeConvRotWeight, TileGenConvRotModelConfig

    NODE_CLASS_MAPPINGS = {
        "ConvRotTestTensors": ConvRotTestTensors,
        "QuantizeConvRotWeight": QuantizeConvRotWeight,
        "Int8ConvRotLinear": Int8ConvRotLinear,
        "TileGenConvRotModelConfig": TileGenConvRotModelConfig,
    }
    NODE_DISPLAY_NAME_MAPPINGS = {
        "ConvRotTestTensors": "ConvRot Test Tensors",
        "QuantizeConvRotWeight": "Quantize ConvRot Weight (INT8)",
        "Int8ConvRotLinear": "INT8 ConvRot Linear (tilegen)",
        "TileGenConvRotModelConfig": "TileGen ConvRot Runtime (MODEL passthrough)",
    }
except Exception:  # pragma: no cover - an import error must not break ComfyUI
    LOGGER.exception("tilegen: nodes failed to import")

_BACKEND_INSTALLED = False
try:
    from . import backend as _backend

    if os.environ.get("TILEGEN_CONVROT_BACKEND", "auto").strip().lower() != "off":
        _BACKEND_INSTALLED = _backend.install()
except Exception:  # pragma: no cover
    LOGGER.exception("tilegen: backend registration failed")

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
