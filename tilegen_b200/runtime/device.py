"""Device capability probe (API of tilegen/runtime/device.py).

The reference used these limits to size its per-K NVRTC kernel; here they are
informational (the prebuilt kernels size themselves), kept for callers that
gate on ``usable_shared_bytes``.
"""
from __future__ import annotations

import functools

_FALLBACK = {
    "sm": (7, 5),
    "shared_per_block": 49152,
    "shared_per_block_optin": 65536,
    "shared_per_sm": 65536,
    "sm_count": 1,
    "name": "unknown",
}


@functools.lru_cache(maxsize=8)
def probe(device_index: int = 0) -> dict:
    """Shared-memory and SM limits of ``device_index`` (cached); a conservative
    fallback when no CUDA device is visible."""
    try:
        import torch

        if not torch.cuda.is_available():
            return dict(_FALLBACK)
        p = torch.cuda.get_device_properties(device_index)
        return {
            "sm": (int(p.major), int(p.minor)),
            "shared_per_block": int(p.shared_memory_per_block),
            "shared_per_block_optin": int(p.shared_memory_per_block_optin),
            "shared_per_sm": int(p.shared_memory_per_multiprocessor),
            "sm_count": int(p.multi_processor_count),
            "name": "cuda:%d" % device_index,
        }
    except Exception:
        return dict(_FALLBACK)


def usable_shared_bytes(device_index: int = 0, headroom: int = 1024) -> int:
    """Opt-in dynamic shared memory per block minus ``headroom``."""
    return max(0, probe(device_index)["shared_per_block_optin"] - headroom)
