"""The no-allocation entry point tg_int8_gemm_dequant_splitk_noalloc on the GPU.

Some callers cannot allocate device memory at all -- a plugin inside a host
application that hands out all GPU memory through its own allocator, or a
serving process that reserved its memory up front -- so this variant of the
small-M GEMM keeps its scratch in a fixed array inside the library instead of
taking a workspace.  The test calls it through the C ABI twice in a row (with
different shapes, so the second call also shows the array holds nothing over
from the first) and requires the same bits as the library's regular GEMM entry
point on the same inputs; it also checks the size limits are refused cleanly.

This file is collected last on purpose: the variant shares one array per GPU,
so it runs after every other test, and it must pass in a fresh process too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests._util import out_bits
from tilegen_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _fn():
    L = _lib.lib()
    f = L.tg_int8_gemm_dequant_splitk_noalloc
    i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    f.argtypes = [p, p, p, p, i64, p, i32, i64, i64, i64, i32, p, p]
    f.restype = i32
    return f


def _case(m, n, k, seed, dev):
    g = torch.Generator().manual_seed(seed)
    xq = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8).to(dev)
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8).to(dev)
    xs = (torch.rand(m, generator=g) * 0.02 + 1e-4).to(dev)
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-5).to(dev)
    bias = torch.randn(n, generator=g).to(dev)
    return xq, xs, wq, ws, bias


def _noalloc(f, case, out_dtype):
    xq, xs, wq, ws, bias = case
    m, k = xq.shape
    n = wq.shape[0]
    out = torch.empty((m, n), dtype=out_dtype, device=xq.device)
    code = {torch.float32: _lib.TG_DT_F32, torch.float16: _lib.TG_DT_F16, torch.bfloat16: _lib.TG_DT_BF16}
    stream = torch.cuda.current_stream(xq.device).cuda_stream
    st = f(xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(), ws.numel(), bias.data_ptr(),
           _lib.TG_DT_F32, m, n, k, code[out_dtype], out.data_ptr(), stream)
    _lib.check("tg_int8_gemm_dequant_splitk_noalloc", st)
    return out


def _regular(case, out_dtype):
    """The same product through the regular (tiled) entry point tg_int8_gemm_dequant."""
    xq, xs, wq, ws, bias = case
    old = ops.SPLITK_MAX_M
    ops.SPLITK_MAX_M = 0
    try:
        return ops.int8_gemm_dequant(xq, xs, wq, ws, bias, out_dtype)
    finally:
        ops.SPLITK_MAX_M = old


def test_two_calls_in_a_row_match_the_regular_entry_point(cuda):
    f = _fn()
    # The first call is the largest; the second uses a different part of the
    # shared array with other shapes and must not see the first call's sums.
    for m, n, k, out_dtype, seed in ((64, 4096, 3072, torch.bfloat16, 1), (9, 1280, 5120, torch.float16, 2)):
        case = _case(m, n, k, seed, cuda)
        got = _noalloc(f, case, out_dtype)
        ref = _regular(case, out_dtype)
        torch.cuda.synchronize()
        assert np.array_equal(out_bits(got), out_bits(ref)), f"M={m} N={n} K={k}"
    assert _lib.device_status(0) == 0


def test_sizes_beyond_the_array_are_refused(cuda):
    f = _fn()
    for m, n in ((65, 128), (64, 32768), (16, 65536 + 128)):
        case = _case(m, n, 64, 0, cuda)
        with pytest.raises(ValueError, match="unsupported"):
            _noalloc(f, case, torch.float16)
