"""Loader for the prebuilt sm_100a library ``libtilegen_b200.so`` (the C ABI in
``include/tilegen_b200.h``).

There is no fallback: if the library is missing or fails to load, every op
raises.  ``build()`` compiles it in-tree with nvcc (``-gencode
arch=compute_100a,code=sm_100a``); the built file travels with the repository.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
HEADER = os.path.join(REPO_DIR, "include", "tilegen_b200.h")
LIB_PATH = os.path.join(PKG_DIR, "libtilegen_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]

TG_OK = 0
TG_ERR_INVALID_ARG = 1
TG_ERR_UNSUPPORTED = 2
TG_ERR_MISALIGNED = 3
TG_ERR_CUDA = 4
TG_ERR_DEVICE_TIMEOUT = 5

TG_DT_F32, TG_DT_F16, TG_DT_BF16 = 0, 1, 2
TG_ACT_NONE, TG_ACT_GELU_TANH, TG_ACT_GELU = 0, 1, 2
TG_QUANT_REFERENCE_ORDER = 0x100  # OR'ed into tg_quantize_act's act: the reference butterfly order

_lock = threading.Lock()
_lib = None


class TileGenError(RuntimeError):
    """A tilegen_b200 C-ABI call returned a non-OK status."""

    def __init__(self, func: str, status: int, msg: str):
        super().__init__(f"{func} failed: {msg} (status {status})")
        self.status = status


def _sources():
    return [os.path.join(CSRC_DIR, f) for f in sorted(os.listdir(CSRC_DIR))
            if f.endswith((".cu", ".cuh"))] + [HEADER]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libtilegen_b200.so`` for sm_100a if it is missing or stale."""
    srcs = _sources()
    if not force and os.path.exists(LIB_PATH):
        if os.path.getmtime(LIB_PATH) >= max(os.path.getmtime(s) for s in srcs):
            return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", LIB_PATH, os.path.join(CSRC_DIR, "capi.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB_PATH


def declared_functions() -> list[str]:
    """Names of the functions ``include/tilegen_b200.h`` declares."""
    with open(HEADER) as f:
        text = f.read()
    return re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(tg_\w+)\s*\(", text, re.M)


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once).  Raises if it cannot be loaded."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(tilegen_b200 has no CPU or eager fallback)")
        L = ctypes.CDLL(LIB_PATH)
        i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        L.tg_version.restype = i32
        L.tg_status_string.argtypes = [i32]
        L.tg_status_string.restype = ctypes.c_char_p
        L.tg_rotate_quant.argtypes = [p, i32, i64, i64, i32, p, p, p]
        L.tg_rotate_quant.restype = i32
        L.tg_rotate_quant_max_k.restype = i64
        L.tg_quantize_act.argtypes = [p, i32, i64, i64, i32, i32, p, p, p]
        L.tg_quantize_act.restype = i32
        L.tg_quantize_ln_mod.argtypes = [p, i32, i64, i64, i32, ctypes.c_float, p, p, i64, p, p, p]
        L.tg_quantize_ln_mod.restype = i32
        L.tg_int8_gemm_dequant.argtypes = [p, p, p, p, i64, p, i32, i64, i64, i64, i32, p, p]
        L.tg_int8_gemm_dequant.restype = i32
        L.tg_gemm_config.argtypes = [i64, i64, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        L.tg_gemm_config.restype = i32
        L.tg_set_gemm_config.argtypes = [i32, i32]
        L.tg_set_gemm_config.restype = i32
        L.tg_device_status.argtypes = [i32, ctypes.POINTER(ctypes.c_uint32), i32]
        L.tg_device_status.restype = i32
        L.tg_int8_gemm_dequant_splitk.argtypes = [p, p, p, p, i64, p, i32, i64, i64, i64, i32, p, p,
                                                  ctypes.c_size_t, p]
        L.tg_int8_gemm_dequant_splitk.restype = i32
        L.tg_int8_gemm_dequant_splitk_workspace.argtypes = [i64, i64]
        L.tg_int8_gemm_dequant_splitk_workspace.restype = ctypes.c_size_t
        L.tg_int8_gemm_dequant_splitk_max_m.restype = i64
        L.tg_int8_gemm_dequant_splitk_config.argtypes = [i64, i64, i64, i32, i32, ctypes.POINTER(i32),
                                                         ctypes.POINTER(i32)]
        L.tg_int8_gemm_dequant_splitk_config.restype = i32
        L.tg_int8_gemv_dequant.argtypes = [p, p, p, p, i64, p, i32, i64, i64, i64, i32, p, p]
        L.tg_int8_gemv_dequant.restype = i32
        L.tg_int8_gemv_dequant_config.argtypes = [i64, i64, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        L.tg_int8_gemv_dequant_config.restype = i32
        L.tg_peer_handle_bytes.restype = ctypes.c_size_t
        L.tg_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(p), p]
        L.tg_peer_alloc.restype = i32
        L.tg_peer_free.argtypes = [p]
        L.tg_peer_free.restype = i32
        L.tg_peer_open.argtypes = [p, ctypes.POINTER(p)]
        L.tg_peer_open.restype = i32
        L.tg_peer_close.argtypes = [p]
        L.tg_peer_close.restype = i32
        L.tg_copy_async.argtypes = [p, p, ctypes.c_size_t, p]
        L.tg_copy_async.restype = i32
        L.tg_set_sm_budget.argtypes = [i32]
        L.tg_set_sm_budget.restype = i32
        L.tg_sm_budget.restype = i32
        _lib = L
    return _lib


def check(func: str, status: int) -> None:
    if status != TG_OK:
        msg = lib().tg_status_string(status).decode()
        if status in (TG_ERR_INVALID_ARG, TG_ERR_UNSUPPORTED, TG_ERR_MISALIGNED):
            raise ValueError(f"{func}: {msg} (status {status})")
        raise TileGenError(func, status, msg)


def splitk_config(m: int, n: int, k: int, out_dtype_code: int = TG_DT_F16, has_bias: bool = False) -> tuple[int, int]:
    """(slices, cluster flag) of the small-M kernel for an m x n x k problem on the current device."""
    sl, cl = ctypes.c_int(0), ctypes.c_int(0)
    check("tg_int8_gemm_dequant_splitk_config",
          lib().tg_int8_gemm_dequant_splitk_config(int(m), int(n), int(k), int(out_dtype_code), int(has_bias),
                                                   ctypes.byref(sl), ctypes.byref(cl)))
    return sl.value, cl.value


def gemv_config(n: int, k: int) -> tuple[int, int]:
    """(K parts per 4-row group, CTAs) of the few-row GEMV for an n x k weight on the current device."""
    parts, ctas = ctypes.c_int(0), ctypes.c_int(0)
    check("tg_int8_gemv_dequant_config",
          lib().tg_int8_gemv_dequant_config(int(n), int(k), ctypes.byref(parts), ctypes.byref(ctas)))
    return parts.value, ctas.value


def gemm_config(m: int, n: int) -> tuple[int, int]:
    """(tile width, pair flag) the GEMM uses for an m x n problem on the current device."""
    bn, pair = ctypes.c_int(0), ctypes.c_int(0)
    check("tg_gemm_config", lib().tg_gemm_config(int(m), int(n), ctypes.byref(bn), ctypes.byref(pair)))
    return bn.value, pair.value


def set_gemm_config(bn: int = 0, pair: int = -1) -> None:
    """Force the GEMM tile shape (bn 0 / pair -1 restore the automatic choice)."""
    check("tg_set_gemm_config", lib().tg_set_gemm_config(int(bn), int(pair)))


def device_status(device: int, clear: bool = True) -> int:
    """Device status word (0 = healthy); synchronises ``device``."""
    bits = ctypes.c_uint32(0)
    st = lib().tg_device_status(int(device), ctypes.byref(bits), int(clear))
    if st not in (TG_OK, TG_ERR_DEVICE_TIMEOUT):
        check("tg_device_status", st)
    return int(bits.value)
