"""CPU oracle for the int8_convrot path (test infrastructure, never the product).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
use this package, and only as the checker / the timed CPU baseline.  It wraps
``liboracle.so`` (``convrot_oracle.c``, a plain-C restatement of
tilegen/kernels/int8_convrot.py:47-104, tilegen/quant/int8_ops.py:22-70 and
tilegen/comfyui/backend.py:230-232; see that file's header for the per-step
citations).

Parity is pinned: ``tests/test_oracle.py`` checks this oracle against the
fixtures in ``tests/golden/``, which the reference's own eager functions
produced (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
_DTYPE_CODES = {"float32": DT_F32, "float16": DT_F16, "bfloat16": DT_BF16}

_lib = None


def build(force: bool = False) -> str:
    """Compile ``liboracle.so`` with the committed Makefile (gcc, OpenMP)."""
    src = os.path.join(HERE, "convrot_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-s", "-B" if force else "liboracle.so"],
                       check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        i64, p = ctypes.c_int64, ctypes.c_void_p
        L.oracle_rotate_quant.argtypes = [p, ctypes.c_int, i64, i64, ctypes.c_int, p, p]
        L.oracle_rotate_quant.restype = ctypes.c_int
        L.oracle_rotate_quant_short.argtypes = [p, ctypes.c_int, i64, i64, ctypes.c_int, p, p]
        L.oracle_rotate_quant_short.restype = ctypes.c_int
        L.oracle_rowwise_quant.argtypes = [p, ctypes.c_int, i64, i64, p, p]
        L.oracle_rowwise_quant.restype = ctypes.c_int
        L.oracle_int8_gemm_dequant.argtypes = [p, p, p, p, i64, p, i64, i64, i64, ctypes.c_int, p]
        L.oracle_int8_gemm_dequant.restype = ctypes.c_int
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_set_num_threads.argtypes = [ctypes.c_int]
        L.oracle_ln_mod.argtypes = [p, ctypes.c_int, i64, i64, ctypes.c_float, p, p, i64, p]
        L.oracle_ln_mod.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def rotate_quant(x: np.ndarray, dtype: str, group: int = 256, order: str = "reference"):
    """Rotate+quantize rows of ``x``.

    ``x`` is float32 for ``dtype="float32"``; for ``"float16"``/``"bfloat16"`` it
    holds the raw 16-bit patterns (uint16/int16).  ``order="reference"`` is the
    reference kernel's butterfly order (pinned to the golden vectors);
    ``"short"`` restates the CUDA kernel's default order.  Returns
    ``(q int8[M,K], scale f32[M])``.
    """
    x = np.ascontiguousarray(x)
    m, k = x.shape
    q = np.empty((m, k), np.int8)
    s = np.empty((m,), np.float32)
    if order not in ("reference", "short"):
        raise ValueError(f"unknown butterfly order {order!r}")
    fn = lib().oracle_rotate_quant if order == "reference" else lib().oracle_rotate_quant_short
    rc = fn(_ptr(x), _DTYPE_CODES[dtype], m, k, group, _ptr(q), _ptr(s))
    if rc != 0:
        raise ValueError(f"oracle_rotate_quant rejected M={m} K={k} group={group}")
    return q, s


def ln_mod(x: np.ndarray, dtype: str, eps: float, scale: np.ndarray, shift: np.ndarray, mod_rows: int):
    """``LayerNorm(x) * (1 + scale[v]) + shift[v]`` per row (``v = row // mod_rows``) in
    the CUDA prologue's arithmetic; all arrays hold raw fp16/bf16 patterns.  Returns
    the ``[M, K]`` patterns of the modulated rows."""
    x = np.ascontiguousarray(x).view(np.uint16)
    scale = np.ascontiguousarray(scale).view(np.uint16)
    shift = np.ascontiguousarray(shift).view(np.uint16)
    m, k = x.shape
    if scale.shape != shift.shape or scale.shape[1] != k or scale.shape[0] < -(-m // mod_rows):
        raise ValueError("modulation vectors must be [ceil(M / mod_rows), K]")
    y = np.empty((m, k), np.uint16)
    rc = lib().oracle_ln_mod(_ptr(x), _DTYPE_CODES[dtype], m, k, float(eps), _ptr(scale), _ptr(shift),
                             int(mod_rows), _ptr(y))
    if rc != 0:
        raise ValueError(f"oracle_ln_mod rejected M={m} K={k} dtype={dtype}")
    return y


def rowwise_quant(x: np.ndarray, dtype: str):
    """Rotation-free row-wise int8 of ``x`` (raw fp16/bf16 patterns) -> ``(q, scale)``."""
    x = np.ascontiguousarray(x)
    m, k = x.shape
    q = np.empty((m, k), np.int8)
    s = np.empty((m,), np.float32)
    rc = lib().oracle_rowwise_quant(_ptr(x), _DTYPE_CODES[dtype], m, k, _ptr(q), _ptr(s))
    if rc != 0:
        raise ValueError(f"oracle_rowwise_quant rejected M={m} K={k} dtype={dtype}")
    return q, s


def int8_gemm_dequant(xq, xscale, wq, wscale, bias, out_dtype: str):
    """``((float(xq @ wq.T) * xscale[:,None]) * wscale[None,:]) + bias`` -> out dtype.

    Returns float32 for ``"float32"``, else the raw uint16 patterns of fp16/bf16.
    """
    xq = np.ascontiguousarray(xq, np.int8)
    wq = np.ascontiguousarray(wq, np.int8)
    xs = np.ascontiguousarray(xscale, np.float32).reshape(-1)
    ws = np.ascontiguousarray(wscale, np.float32).reshape(-1)
    m, k = xq.shape
    n = wq.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, np.float32).reshape(-1)
    out = np.empty((m, n), np.float32 if out_dtype == "float32" else np.uint16)
    rc = lib().oracle_int8_gemm_dequant(_ptr(xq), _ptr(xs), _ptr(wq), _ptr(ws), ws.size,
                                        None if b is None else _ptr(b), m, n, k,
                                        _DTYPE_CODES[out_dtype], _ptr(out))
    if rc != 0:
        raise ValueError("oracle_int8_gemm_dequant rejected its arguments")
    return out


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))
