"""ComfyUI custom-node entry point (copy or link this folder into ComfyUI/custom_nodes/tilegen)."""

from tilegen.comfyui import NODE_CLASS_MAPPINGS, NODE_DISPLAY_NAME_MAPPINGS

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
