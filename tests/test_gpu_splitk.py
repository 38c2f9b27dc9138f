"""Parity of the small-M split-K INT8 GEMM (tg_int8_gemm_dequant_splitk) on the GPU.

With M <= 128 rows the weight is streamed by (N/128 column tiles) x (K slices)
CTAs whose exact int32 partial sums meet in a scratch accumulator; the last
slice of a tile dequantises.  Integer addition makes the sums order-independent,
so the output must be bit-identical to the tiled kernel, to the oracle, and to
the reference's torch sequence (tilegen/quant/int8_ops.py:22-70, torch._int_mm
is exact), for every M from 1 to 128, ragged N and K, all output dtypes, bias
and scale variants, and repeated calls on one scratch.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests._util import DT_NAME, out_bits
from tilegen_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed, scalar_ws=False, bias_dtype=None, dev="cpu"):
    g = torch.Generator().manual_seed(seed)
    xq = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
    xs = torch.rand(m, generator=g) * 0.02 + 1e-4
    ws = torch.rand(1 if scalar_ws else n, generator=g) * 0.01 + 1e-5
    bias = None if bias_dtype is None else torch.randn(n, generator=g).to(bias_dtype)
    return xq, xs, wq, ws, bias


def _bits(y):
    b = out_bits(y)
    return b.view(np.uint32) if b.dtype == np.float32 else b


def _run(case, out_dtype, dev, max_m):
    """int8_gemm_dequant with every M <= max_m on the split-K kernel (0: the tiled kernel)."""
    xq, xs, wq, ws, bias = case
    route, gemv = ops.splitk_route, ops.gemv_route
    ops.splitk_route = lambda m, n, k: 0 < m <= max_m
    ops.gemv_route = lambda m, n, k: False
    try:
        y = ops.int8_gemm_dequant(xq.to(dev), xs.to(dev), wq.to(dev), ws.to(dev),
                                  None if bias is None else bias.to(dev), out_dtype)
        torch.cuda.synchronize()
    finally:
        ops.splitk_route, ops.gemv_route = route, gemv
    return y


@pytest.fixture(autouse=True)
def _healthy_device(cuda):
    yield
    assert _lib.device_status(0) == 0, "a bounded wait expired during the test"


# (n, k, cluster): 1536 x 2048 splits K 16 ways (partials reduced through the
# workspace); 5120 x 2048 splits it 6 ways (one cluster per column tile,
# reduced in shared memory).
FORMS = [(1536, 2048, 0), (5120, 2048, 1)]


@pytest.mark.parametrize("n,k,cluster", FORMS)
@pytest.mark.parametrize("m", [1, 2, 7, 16, 17, 31, 32, 33, 48, 63, 64, 65, 96, 100, 127, 128])
def test_rows_bit_exact_vs_tiled_kernel(cuda, m, n, k, cluster):
    assert _lib.splitk_config(m, n, k)[1] == cluster
    case = _case(m, n, k, seed=m)
    a = _run(case, torch.float16, cuda, 128)
    b = _run(case, torch.float16, cuda, 0)
    assert np.array_equal(_bits(a), _bits(b))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bias_dtype", [None, torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("scalar_ws", [False, True])
@pytest.mark.parametrize("n,cluster", [(640, 0), (4096, 1)])
def test_against_oracle(cuda, out_dtype, bias_dtype, scalar_ws, n, cluster):
    m, k = 24, 1152
    code = {torch.float32: _lib.TG_DT_F32, torch.float16: _lib.TG_DT_F16, torch.bfloat16: _lib.TG_DT_BF16}[out_dtype]
    assert _lib.splitk_config(m, n, k, code, bias_dtype is not None)[1] == cluster
    case = _case(m, n, k, seed=3, scalar_ws=scalar_ws, bias_dtype=bias_dtype)
    y = _run(case, out_dtype, cuda, 128)
    xq, xs, wq, ws, bias = case
    ref = oracle.int8_gemm_dequant(xq.numpy(), xs.numpy(), wq.numpy(), ws.numpy(),
                                   None if bias is None else bias.float().numpy(), DT_NAME[out_dtype])
    got = out_bits(y)
    if got.dtype == np.float32:
        got, ref = got.view(np.uint32), ref.view(np.uint32)
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} outputs differ, first at {bad[:3].tolist()}"


@pytest.mark.parametrize("n,k", [(8, 16), (136, 144), (1000, 4112), (4000, 1040), (5120, 13824), (15360, 5120)])
def test_ragged_and_dit_shapes(cuda, n, k):
    if n >= 4000:  # these reduce in shared memory (4000 x 1040: ragged N and K in that form)
        assert all(_lib.splitk_config(m, n, k)[1] == 1 for m in (1, 64, 128))
    for m in (1, 64, 128):
        case = _case(m, n, k, seed=n + k + m)
        a = _run(case, torch.bfloat16, cuda, 128)
        xq, xs, wq, ws, _ = case
        # int8 products summed in float64 are exact (|sum| < 2^53); .float()
        # then rounds once, as float(int32) does.
        acc = (xq.to(cuda).double() @ wq.to(cuda).double().t()).float()
        ref = acc * xs.to(cuda)[:, None] * ws.to(cuda)[None, :]
        assert np.array_equal(_bits(a), _bits(ref.to(torch.bfloat16)))


def test_scratch_is_left_zero_and_reused(cuda):
    outs, refs = [], []
    for i in range(5):
        case = _case(40, 2048, 3072, seed=100 + i, bias_dtype=torch.float32)
        outs.append(_run(case, torch.float16, cuda, 128))
        refs.append(_run(case, torch.float16, cuda, 0))
    for a, b in zip(outs, refs):
        assert np.array_equal(_bits(a), _bits(b))
    key = (0, torch.cuda.current_stream(0).cuda_stream)
    assert int(ops._SPLITK_WS[key].count_nonzero()) == 0, "split-K scratch not returned to zero"
