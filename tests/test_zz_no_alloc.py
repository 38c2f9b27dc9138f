"""The no-allocation entry point tg_int8_gemm_dequant_splitk_noalloc on the GPU.

Some callers cannot allocate device memory at all -- a plugin inside a host
application that hands out all GPU memory through its own allocator, or a
serving process that reserved its memory up front -- so this variant of the
small-M GEMM keeps its scratch in a fixed array inside the library instead of
taking a workspace.  The test calls it through the C ABI on shapes whose K is
split more ways than a cluster holds, so the partial sums really go through the
library's array: twice in a row on one shape, then on a smaller one that reuses
the start of the array, each time requiring the same bits as the library's
regular GEMM entry point and as the oracle; it also checks that the size limits
are refused cleanly.

This file is collected last on purpose: the variant shares one array per GPU,
so it runs after every other test, and it must pass in a fresh process too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from tests._util import DT_NAME, out_bits
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


_CODE = {torch.float32: _lib.TG_DT_F32, torch.float16: _lib.TG_DT_F16, torch.bfloat16: _lib.TG_DT_BF16}


def _oracle(case, out_dtype):
    xq, xs, wq, ws, bias = (t.cpu() for t in case)
    return oracle.int8_gemm_dequant(xq.numpy(), xs.numpy(), wq.numpy(), ws.numpy(), bias.numpy(),
                                    DT_NAME[out_dtype])


def test_two_calls_in_a_row_match_the_regular_entry_point(cuda):
    f = _fn()
    # K split 10 and 20 ways (more than a cluster's 8): the partial sums go
    # through the shared array.  The first shape covers the larger part of it;
    # the second reuses its start.  Outputs must be bit-identical to the
    # regular entry point and to the oracle, on both calls of the first shape.
    shapes = ((64, 3072, 5120, torch.bfloat16, 1), (64, 3072, 5120, torch.bfloat16, 1),
              (9, 1280, 5120, torch.float16, 2))
    for m, n, k, out_dtype, seed in shapes:
        slices, cluster = _lib.splitk_config(m, n, k, _CODE[out_dtype], True)
        assert cluster == 0 and slices > 8, (m, n, k, slices, cluster)
        case = _case(m, n, k, seed, cuda)
        got = _noalloc(f, case, out_dtype)
        ref = _regular(case, out_dtype)
        torch.cuda.synchronize()
        assert np.array_equal(out_bits(got), out_bits(ref)), f"M={m} N={n} K={k}"
        assert np.array_equal(out_bits(got), _oracle(case, out_dtype)), f"M={m} N={n} K={k} vs oracle"
    assert _lib.device_status(0) == 0


def test_sizes_beyond_the_array_are_refused(cuda):
    f = _fn()
    for m, n in ((65, 128), (64, 32768), (16, 65536 + 128)):
        case = _case(m, n, 64, 0, cuda)
        with pytest.raises(ValueError, match="unsupported"):
            _noalloc(f, case, torch.float16)
