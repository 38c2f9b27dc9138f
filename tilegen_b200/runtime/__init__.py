"""Runtime helpers (API of tilegen/runtime): library presence and device probing."""
from .device import probe, usable_shared_bytes
from .nvrtc import bootstrap, ensure_nvrtc, ensure_nvrtc_12, require_nvrtc

__all__ = ["ensure_nvrtc", "ensure_nvrtc_12", "require_nvrtc", "bootstrap", "probe", "usable_shared_bytes"]
