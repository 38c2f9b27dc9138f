"""Torch-facing wrappers over the C ABI, plus their ``torch.library`` custom ops.

``rotate_quant``, ``quantize_act`` and ``int8_gemm_dequant`` allocate their outputs with torch's
caching allocator and enqueue the sm_100a kernels on the current stream of the
input's device.  They never fall back to another implementation: an input the
kernels do not handle raises ``ValueError``, a CUDA failure raises
``TileGenError``.  ``int8_gemm_dequant`` with one to ``GEMV_MAX_M`` rows runs the
few-row GEMV on the CUDA cores; with up to ``SPLITK_MAX_M`` rows (see
``splitk_route``) the split-K kernel and a cached, self-clearing scratch per
(device, stream); otherwise the tiled tcgen05 kernel.

The same functions are registered as ``torch.ops.tilegen.rotate_quant``,
``torch.ops.tilegen.quantize_act``, ``torch.ops.tilegen.quantize_ln_mod`` and
``torch.ops.tilegen.int8_gemm_dequant``
(with fake implementations, so they trace under ``torch.compile``/``torch.export``
as opaque ops).
"""
from __future__ import annotations

import contextlib

import torch

from . import _lib

_DTYPE_CODE = {
    torch.float32: _lib.TG_DT_F32,
    torch.float16: _lib.TG_DT_F16,
    torch.bfloat16: _lib.TG_DT_BF16,
}
_SUPPORTED_GROUPS = (4, 16, 64, 256)
# input_act names (tilegen/comfyui/backend.py:174) the quantiser applies itself.
FUSED_ACTS = {"gelu_tanh": _lib.TG_ACT_GELU_TANH, "gelu": _lib.TG_ACT_GELU}
# Butterfly orders of the rotation.  "short" (the default): per radix-4
# butterfly S = (a0 + a2) + (a1 + a3) and each output S - 2*a_i in one fma, and
# the codes' rint(v * inv) in one fma for rows without inf/NaN -- codes differ
# from the reference kernel's by one at rounding ties (about 1e-6 of them on
# DiT-like activations; the parity tolerance allows 1e-3), scales by a few
# ulps.  "reference": the reference kernel's left-to-right sums
# (tilegen/kernels/int8_convrot.py:74-77), bit-identical to it.
ROTATION_ORDERS = {"short": 0, "reference": _lib.TG_QUANT_REFERENCE_ORDER}


def _order_flag(fn: str, order: str) -> int:
    if order not in ROTATION_ORDERS:
        raise ValueError(f"{fn}: order must be one of {sorted(ROTATION_ORDERS)}, got {order!r}")
    return ROTATION_ORDERS[order]


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _call(func: str, dev: torch.device, *args) -> None:
    L = _lib.lib()
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(idx).cuda_stream
    if idx != torch.cuda.current_device():
        with torch.cuda.device(idx):
            st = getattr(L, func)(*args, stream)
    else:
        st = getattr(L, func)(*args, stream)
    _lib.check(func, st)


def rotate_quant_max_k() -> int:
    return int(_lib.lib().tg_rotate_quant_max_k())


def rotate_quant(x: torch.Tensor, group: int = 256, order: str = "short"):
    """Group-Hadamard rotation + row-wise int8 quantisation of ``x [M, K]``.

    Returns ``(q int8 [M, K], scale fp32 [M])``.  ``x`` must be a CUDA fp16/bf16
    tensor, ``group`` one of 4/16/64/256 and ``K`` a multiple of 256 (at most
    ``rotate_quant_max_k()``).  ``order``: a key of ``ROTATION_ORDERS``.
    """
    flag = _order_flag("rotate_quant", order)
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("rotate_quant: CUDA tensor required")
    if x.ndim != 2:
        raise ValueError(f"rotate_quant: expected 2-D input, got {tuple(x.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"rotate_quant: fp16/bf16 input required, got {x.dtype}")
    if group not in _SUPPORTED_GROUPS:
        raise ValueError(f"rotate_quant: group must be one of {_SUPPORTED_GROUPS}, got {group}")
    m, k = x.shape
    if k % 256:
        raise ValueError(f"rotate_quant: K={k} must be a multiple of 256")
    x = _aligned(x)
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    if m:
        _call("tg_quantize_act", x.device, x.data_ptr(), _DTYPE_CODE[x.dtype], m, k, int(group),
              _lib.TG_ACT_NONE | flag, q.data_ptr(), s.data_ptr())
    return q, s


def quantize_act(x: torch.Tensor, group: int = 256, act: str | None = None, order: str = "short"):
    """``act`` applied to ``x [M, K]``, then rotate+quantise (``group`` 4..256) or,
    with ``group=1``, the rotation-free row-wise quantisation of
    tilegen/comfyui/backend.py:230-232.  One pass over ``x`` (``tg_quantize_act``).

    ``act``: None/``"none"``, or a name in ``FUSED_ACTS``; the activation is what
    torch's ``F.gelu`` (``approximate="tanh"`` for ``gelu_tanh``) stores for an
    fp16/bf16 tensor.  Returns ``(q int8 [M, K], scale fp32 [M])``.  ``K`` must be
    a multiple of 256 (of 64 for ``group=1``).  ``order``: a key of
    ``ROTATION_ORDERS`` (the row-wise form has no rotation).
    """
    flag = _order_flag("quantize_act", order)
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("quantize_act: CUDA tensor required")
    if x.ndim != 2:
        raise ValueError(f"quantize_act: expected 2-D input, got {tuple(x.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"quantize_act: fp16/bf16 input required, got {x.dtype}")
    if group != 1 and group not in _SUPPORTED_GROUPS:
        raise ValueError(f"quantize_act: group must be 1 or one of {_SUPPORTED_GROUPS}, got {group}")
    if act in (None, "none"):
        code = _lib.TG_ACT_NONE
    elif act in FUSED_ACTS:
        code = FUSED_ACTS[act]
    else:
        raise ValueError(f"quantize_act: activation {act!r} is not one of {sorted(FUSED_ACTS)}")
    m, k = x.shape
    if k % (64 if group == 1 else 256):
        raise ValueError(f"quantize_act: K={k} must be a multiple of {64 if group == 1 else 256}")
    x = _aligned(x)
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    if m:
        _call("tg_quantize_act", x.device, x.data_ptr(), _DTYPE_CODE[x.dtype], m, k, int(group), code | flag,
              q.data_ptr(), s.data_ptr())
    return q, s


def quantize_ln_mod(x: torch.Tensor, group: int, scale: torch.Tensor, shift: torch.Tensor, eps: float = 1e-6,
                    rows_per_vector: int | None = None):
    """The DiT block's normalisation in front of a projection, fused into the
    quantiser (``tg_quantize_ln_mod``): ``y = LayerNorm(x) * (1 + scale) + shift``
    (LayerNorm without affine, ``eps``), then rotate+quantise ``y`` with ``group``
    (4..256, the short butterfly order), in one pass over ``x`` -- the modulated
    activations are never written to memory.

    ``x``: ``[..., K]`` fp16/bf16 CUDA, flattened to ``[M, K]`` rows.  ``scale`` and
    ``shift``: ``[K]`` (one vector) or ``[S, ..., K]`` (``S`` vectors, e.g. a DiT's
    per-sample ``[B, 1, K]``), converted to ``x``'s dtype; row ``r`` uses vector
    ``r // rows_per_vector`` (default ``M // S``, which must divide evenly).  Each
    of the normalised row, the product and the sum is rounded to ``x``'s dtype as
    torch's separate ops store them; the mean and variance are fp32 sums in a
    fixed order, so codes match ``F.layer_norm`` + the two ops + ``rotate_quant``
    within the parity tolerance, not bit for bit.  Returns ``(q int8 [M, K],
    scale fp32 [M])``.
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("quantize_ln_mod: CUDA tensor required")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"quantize_ln_mod: fp16/bf16 input required, got {x.dtype}")
    if group not in _SUPPORTED_GROUPS:
        raise ValueError(f"quantize_ln_mod: group must be one of {_SUPPORTED_GROUPS}, got {group}")
    k = x.shape[-1]
    if k % 256:
        raise ValueError(f"quantize_ln_mod: K={k} must be a multiple of 256")
    x2 = _aligned(x.reshape(-1, k))
    m = x2.shape[0]
    vecs = []
    for name, t in (("scale", scale), ("shift", shift)):
        if not isinstance(t, torch.Tensor) or t.shape[-1] != k:
            raise ValueError(f"quantize_ln_mod: {name} must be a tensor whose last dimension is K={k}")
        vecs.append(_aligned(t.to(device=x.device, dtype=x.dtype).reshape(-1, k)))
    sc, sh = vecs
    if sc.shape != sh.shape:
        raise ValueError(f"quantize_ln_mod: scale {tuple(scale.shape)} and shift {tuple(shift.shape)} differ")
    nvec = sc.shape[0]
    if rows_per_vector is None:
        if m % nvec:
            raise ValueError(f"quantize_ln_mod: {m} rows do not split evenly over {nvec} modulation vectors")
        rows_per_vector = max(1, m // nvec)
    rows_per_vector = int(rows_per_vector)
    if rows_per_vector < 1 or nvec < -(-m // rows_per_vector):
        raise ValueError(f"quantize_ln_mod: {nvec} vectors cannot cover {m} rows at {rows_per_vector} a vector")
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    if m:
        _call("tg_quantize_ln_mod", x.device, x2.data_ptr(), _DTYPE_CODE[x.dtype], m, k, int(group), float(eps),
              sc.data_ptr(), sh.data_ptr(), rows_per_vector, q.data_ptr(), s.data_ptr())
    return q, s


def int8_gemm_dequant(xq: torch.Tensor, xscale: torch.Tensor, wq: torch.Tensor, wscale: torch.Tensor,
                      bias: torch.Tensor | None, out_dtype: torch.dtype, out: torch.Tensor | None = None) -> torch.Tensor:
    """``((float(xq @ wq.T) * xscale[:, None]) * wscale[None, :]) + bias`` as ``out_dtype``.

    ``xq [M, K]`` and ``wq [N, K]`` int8 on the same CUDA device; ``xscale [M]``;
    ``wscale`` scalar or ``[N]``; ``bias [N]`` fp32/fp16/bf16 or None.  ``out``: an
    optional contiguous ``[M, N]`` ``out_dtype`` tensor on that device (16-byte
    aligned) to write into, e.g. this rank's rows of a ``PeerRowGather`` buffer.
    """
    if not (xq.is_cuda and wq.is_cuda):
        raise ValueError("int8_gemm_dequant: CUDA tensors required")
    if xq.dtype != torch.int8 or wq.dtype != torch.int8:
        raise ValueError("int8_gemm_dequant: int8 operands required")
    if xq.ndim != 2 or wq.ndim != 2 or xq.shape[1] != wq.shape[1]:
        raise ValueError(f"int8_gemm_dequant: shapes {tuple(xq.shape)} x {tuple(wq.shape)}^T do not match")
    if out_dtype not in _DTYPE_CODE:
        raise ValueError(f"int8_gemm_dequant: unsupported out_dtype {out_dtype}")
    dev = xq.device
    m, k = xq.shape
    n = wq.shape[0]
    xq = _aligned(xq)
    wq = _aligned(wq.to(dev))
    xs = xscale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if xs.numel() != m:
        raise ValueError(f"int8_gemm_dequant: xscale has {xs.numel()} elements, expected {m}")
    ws = wscale.to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
    if ws.numel() not in (1, n):
        raise ValueError(f"weight scale must be scalar or length {n}, got {tuple(wscale.shape)}")
    b_ptr, b_code = None, _lib.TG_DT_F32
    if bias is not None:
        b = bias.to(device=dev).reshape(-1)
        if b.dtype not in _DTYPE_CODE:
            b = b.float()
        b = b.contiguous()
        if b.numel() != n:
            raise ValueError(f"int8_gemm_dequant: bias has {b.numel()} elements, expected {n}")
        bias = b
        b_ptr, b_code = b.data_ptr(), _DTYPE_CODE[b.dtype]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=dev)
    elif (tuple(out.shape) != (m, n) or out.dtype != out_dtype or out.device != dev or not out.is_contiguous()
          or out.data_ptr() % 16):
        raise ValueError(f"int8_gemm_dequant: out must be a contiguous 16-byte aligned [{m}, {n}] {out_dtype} "
                         f"tensor on {dev}")
    if m and gemv_route(m, n, k):
        _call("tg_int8_gemv_dequant", dev, xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(),
              ws.numel(), b_ptr, b_code, m, n, k, _DTYPE_CODE[out_dtype], out.data_ptr())
    elif m and splitk_route(m, n, k):
        work = _splitk_workspace(dev, m, n)
        _call("tg_int8_gemm_dequant_splitk", dev, xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(),
              ws.numel(), b_ptr, b_code, m, n, k, _DTYPE_CODE[out_dtype], out.data_ptr(), work.data_ptr(),
              work.numel())
    elif m:
        _call("tg_int8_gemm_dequant", dev, xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(),
              ws.numel(), b_ptr, b_code, m, n, k, _DTYPE_CODE[out_dtype], out.data_ptr())
    return out


@contextlib.contextmanager
def sm_budget(sms: int):
    """Within the block, the persistent kernels (rotate+quant, the tiled GEMM) size their
    grids for at most ``sms`` SMs (``tg_set_sm_budget``; process-wide, restored on
    exit).  Use it for kernels that run while a collective is in flight on another
    stream, leaving that collective the SMs it occupies, so both proceed at once."""
    L = _lib.lib()
    old = int(L.tg_sm_budget())
    _lib.check("tg_set_sm_budget", L.tg_set_sm_budget(int(sms)))
    try:
        yield
    finally:
        L.tg_set_sm_budget(old)


# Largest M int8_gemm_dequant sends to the few-row GEMV (tg_int8_gemv_dequant,
# at most 4); 0 sends none there.
GEMV_MAX_M = 4


def gemv_route(m: int, n: int, k: int) -> bool:
    """Whether an m x n x k product goes to the few-row GEMV (at most GEMV_MAX_M rows).

    Measured on B200 at the DiT shapes against the split-K kernel, whole linears
    (quantiser + GEMM) replayed from a CUDA graph with L2 flushed before each:
    the GEMV is faster at M <= 2 everywhere (M = 1: qkv 16.0 vs 21.3 us, o_proj
    9.2 vs 11.0, ffn_up 15.4 vs 20.8, ffn_down 15.9 vs 18.9) and at M <= 4 for
    K < 8192; at K = 13824 with 3-4 rows the two are even, and split-K stays.
    """
    return 0 < m <= min(GEMV_MAX_M, 4 if k < 8192 else 2)


# Largest M int8_gemm_dequant sends to the split-K kernel
# (tg_int8_gemm_dequant_splitk); 0 sends every M to the tiled kernel.
SPLITK_MAX_M = 128


def splitk_route(m: int, n: int, k: int) -> bool:
    """Whether an m x n x k product goes to the split-K kernel (at most SPLITK_MAX_M rows).

    Measured on B200 at the DiT shapes against the tiled kernel (whose M <= 128
    tiles give only N/128 CTAs), whole linears replayed from a CUDA graph with
    L2 flushed before each (cold weights, as in a model): split-K is faster for
    M <= 24 everywhere, and up to 128 rows when N <= 8192 or K >= 8192.
    """
    if not 0 < m <= SPLITK_MAX_M:
        return False
    return m <= 24 or n <= 8192 or k >= 8192


# Split-K scratch, one per (device, stream): zero-filled when created and left
# zero by every call, so it is reused as is; it only grows.
_SPLITK_WS: dict[tuple[int, int], torch.Tensor] = {}


def _splitk_workspace(dev: torch.device, m: int, n: int) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    need = int(_lib.lib().tg_int8_gemm_dequant_splitk_workspace(m, n))
    ws = _SPLITK_WS.get(key)
    if ws is None or ws.numel() < need:
        # The caching allocator returns 512-byte aligned blocks (256 needed).
        ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _SPLITK_WS[key] = ws
    return ws


# ---------------------------------------------------------------- custom ops
@torch.library.custom_op("tilegen::rotate_quant", mutates_args=())
def _rotate_quant_op(x: torch.Tensor, group: int) -> tuple[torch.Tensor, torch.Tensor]:
    return rotate_quant(x, group)


@_rotate_quant_op.register_fake
def _(x, group):
    return x.new_empty(x.shape, dtype=torch.int8), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("tilegen::quantize_act", mutates_args=())
def _quantize_act_op(x: torch.Tensor, group: int, act: str | None) -> tuple[torch.Tensor, torch.Tensor]:
    return quantize_act(x, group, act)


@_quantize_act_op.register_fake
def _(x, group, act):
    return x.new_empty(x.shape, dtype=torch.int8), x.new_empty((x.shape[0],), dtype=torch.float32)


@torch.library.custom_op("tilegen::quantize_ln_mod", mutates_args=())
def _quantize_ln_mod_op(x: torch.Tensor, group: int, scale: torch.Tensor, shift: torch.Tensor,
                        eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    return quantize_ln_mod(x, group, scale, shift, eps)


@_quantize_ln_mod_op.register_fake
def _(x, group, scale, shift, eps):
    m = x.numel() // x.shape[-1]
    return x.new_empty((m, x.shape[-1]), dtype=torch.int8), x.new_empty((m,), dtype=torch.float32)


@torch.library.custom_op("tilegen::int8_gemm_dequant", mutates_args=())
def _int8_gemm_dequant_op(xq: torch.Tensor, xscale: torch.Tensor, wq: torch.Tensor, wscale: torch.Tensor,
                          bias: torch.Tensor | None, out_dtype: torch.dtype) -> torch.Tensor:
    return int8_gemm_dequant(xq, xscale, wq, wscale, bias, out_dtype)


@_int8_gemm_dequant_op.register_fake
def _(xq, xscale, wq, wscale, bias, out_dtype):
    return xq.new_empty((xq.shape[0], wq.shape[0]), dtype=out_dtype)
