"""NVRTC bootstrap entry points (API of tilegen/runtime/nvrtc.py).

The reference JIT-compiled its kernel with NVRTC at first use.  This build ships
the kernels precompiled for sm_100a in ``libtilegen_b200.so``, so there is
nothing to bootstrap: these functions only confirm that the library loads.
"""
from __future__ import annotations


def ensure_nvrtc(min_version=(11, 0)) -> bool:
    """True when the prebuilt kernel library loads (no NVRTC is needed)."""
    try:
        from .. import _lib

        _lib.lib()
        return True
    except Exception:
        return False


def require_nvrtc(min_version=(11, 0)) -> None:
    """Raise if the prebuilt kernel library cannot be loaded."""
    from .. import _lib

    _lib.lib()


def bootstrap() -> dict:
    from .. import _lib

    return {"library": _lib.LIB_PATH, "loaded": ensure_nvrtc(), "jit": False}


ensure_nvrtc_12 = ensure_nvrtc
