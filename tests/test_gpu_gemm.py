"""Parity of the tcgen05 INT8 GEMM + fused dequant (tg_int8_gemm_dequant) on the GPU.

The reference (tilegen/quant/int8_ops.py:22-70) computes an exact int32 GEMM and
then fp32 `.float()`, `* xscale`, `* wscale`, `+ bias`, `copy_` to the output
dtype; the kernel performs the same operations with the same roundings, so the
output must be bit-identical: against the reference's own outputs
(tests/golden/gemm.npz), against the oracle, and at full DiT sizes against the
same torch sequence run on the GPU (torch._int_mm is exact).
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
from tests._util import DT_NAME, out_bits
from tests.conftest import GOLDEN
from tilegen_b200 import _lib, ops
from tilegen_b200.quant.int8_ops import int8_matmul_dequant_chunked

pytestmark = pytest.mark.gpu

DTS = [torch.float32, torch.float16, torch.bfloat16]


def _rand_case(m, n, k, seed, scalar_ws=False, bias_dtype=None):
    g = torch.Generator().manual_seed(seed)
    xq = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
    xs = torch.rand(m, generator=g) * 0.02 + 1e-4
    ws = torch.rand(1 if scalar_ws else n, generator=g) * 0.01 + 1e-5
    bias = None if bias_dtype is None else torch.randn(n, generator=g).to(bias_dtype)
    return xq, xs, wq, ws, bias


def _check_vs_oracle(case, out_dtype, dev):
    xq, xs, wq, ws, bias = case
    y = ops.int8_gemm_dequant(xq.to(dev), xs.to(dev), wq.to(dev), ws.to(dev),
                              None if bias is None else bias.to(dev), out_dtype)
    torch.cuda.synchronize()
    ref = oracle.int8_gemm_dequant(xq.numpy(), xs.numpy(), wq.numpy(), ws.numpy(),
                                   None if bias is None else bias.float().numpy(), DT_NAME[out_dtype])
    got = out_bits(y)
    if got.dtype == np.float32:
        got, ref = got.view(np.uint32), ref.view(np.uint32)
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} outputs differ, first at {bad[:3].tolist()}"


def test_reference_golden_outputs_bit_exact(cuda):
    d = np.load(os.path.join(GOLDEN, "gemm.npz"))
    for name in "abcd":
        m, n, k, od, has_bias, scalar = (int(v) for v in d[f"{name}_meta"])
        out_dtype = DTS[od]
        xq = torch.from_numpy(d[f"{name}_xq"]).to(cuda)
        wq = torch.from_numpy(d[f"{name}_wq"]).to(cuda)
        xs = torch.from_numpy(d[f"{name}_xscale"]).to(cuda)
        ws = torch.from_numpy(d[f"{name}_wscale"]).to(cuda)
        if scalar:
            ws = ws.reshape(())
        bias = torch.from_numpy(d[f"{name}_bias"]).to(cuda) if has_bias else None
        y = int8_matmul_dequant_chunked(xq, xs, wq, ws, bias, out_dtype)
        assert np.array_equal(out_bits(y), d[f"{name}_y"]), name


@pytest.mark.parametrize("out_dtype", DTS)
@pytest.mark.parametrize("mnk", [(1, 256, 256), (128, 256, 128), (130, 264, 1024), (257, 520, 5120),
                                 (33, 72, 400), (200, 1024, 13824)])
def test_bit_exact_vs_oracle(cuda, out_dtype, mnk):
    m, n, k = mnk
    _check_vs_oracle(_rand_case(m, n, k, seed=m * 7 + n), out_dtype, cuda)


@pytest.mark.parametrize("bias_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_bias_dtypes_and_scalar_wscale(cuda, bias_dtype):
    _check_vs_oracle(_rand_case(70, 136, 512, seed=5, bias_dtype=bias_dtype), torch.float16, cuda)
    _check_vs_oracle(_rand_case(70, 136, 512, seed=6, scalar_ws=True, bias_dtype=bias_dtype), torch.bfloat16, cuda)


def _torch_reference(xq, xs, wq, ws, bias, out_dtype):
    """The reference's torch sequence (int8_ops.py:60-68) on the GPU, unchunked."""
    part = torch._int_mm(xq, wq.t()).float()
    part.mul_(xs.float().reshape(-1, 1))
    part.mul_(ws.float().reshape(1, -1))
    if bias is not None:
        part.add_(bias.float().reshape(1, -1))
    return part.to(out_dtype)


@pytest.mark.parametrize("shape", [("qkv", 4096, 15360, 5120), ("o", 4096, 5120, 5120),
                                   ("ffn_up", 4096, 13824, 5120), ("ffn_down", 4096, 5120, 13824),
                                   ("ragged", 8190, 5120, 5120)])
def test_full_size_bit_exact_vs_torch_sequence(cuda, shape):
    _, m, n, k = shape
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    xq = torch.randint(-128, 128, (m, k), generator=g, device=cuda, dtype=torch.int8)
    wq = torch.randint(-128, 128, (n, k), generator=g, device=cuda, dtype=torch.int8)
    xs = torch.rand(m, generator=g, device=cuda) * 1e-3
    ws = torch.rand(n, generator=g, device=cuda) * 1e-3
    bias = torch.randn(n, generator=g, device=cuda, dtype=torch.float16)
    for out_dtype, b in ((torch.float16, None), (torch.bfloat16, bias)):
        y = ops.int8_gemm_dequant(xq, xs, wq, ws, b, out_dtype)
        ref = _torch_reference(xq, xs, wq, ws, b, out_dtype)
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16)), (shape, out_dtype)


@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("bn", [256, 224, 192, 160, 128])
def test_every_tile_shape_bit_exact(cuda, bn, pair):
    _lib.set_gemm_config(bn, pair)
    try:
        for out_dtype in DTS:
            _check_vs_oracle(_rand_case(300, 600, 1024, seed=bn, bias_dtype=torch.bfloat16), out_dtype, cuda)
        _check_vs_oracle(_rand_case(1, 72, 256, seed=3), torch.float16, cuda)        # one row
        _check_vs_oracle(_rand_case(513, 264, 5120, seed=4), torch.bfloat16, cuda)   # ragged M and N
    finally:
        _lib.set_gemm_config(0, -1)


def test_tile_shape_choice_for_dit_shapes(cuda):
    for n in (15360, 5120, 13824):
        bn, pair = _lib.gemm_config(4096, n)
        assert pair == 1 and bn in (256, 224, 192, 160, 128)
    assert _lib.gemm_config(64, 5120)[1] == 0


def test_empty_and_rejected(cuda):
    xq = torch.zeros(0, 256, dtype=torch.int8, device=cuda)
    wq = torch.zeros(64, 256, dtype=torch.int8, device=cuda)
    y = ops.int8_gemm_dequant(xq, torch.zeros(0, device=cuda), wq, torch.ones(64, device=cuda), None, torch.float16)
    assert y.shape == (0, 64)
    with pytest.raises(ValueError):  # K not a multiple of 16
        ops.int8_gemm_dequant(torch.zeros(4, 24, dtype=torch.int8, device=cuda), torch.ones(4, device=cuda),
                              torch.zeros(8, 24, dtype=torch.int8, device=cuda), torch.ones(8, device=cuda),
                              None, torch.float16)
    with pytest.raises(ValueError):  # bad weight-scale length
        ops.int8_gemm_dequant(torch.zeros(4, 32, dtype=torch.int8, device=cuda), torch.ones(4, device=cuda),
                              torch.zeros(8, 32, dtype=torch.int8, device=cuda), torch.ones(3, device=cuda),
                              None, torch.float16)


def test_custom_op_and_status(cuda):
    xq, xs, wq, ws, bias = _rand_case(40, 64, 256, seed=11, bias_dtype=torch.float32)
    a = torch.ops.tilegen.int8_gemm_dequant(xq.to(cuda), xs.to(cuda), wq.to(cuda), ws.to(cuda),
                                            bias.to(cuda), torch.float16)
    b = ops.int8_gemm_dequant(xq.to(cuda), xs.to(cuda), wq.to(cuda), ws.to(cuda), bias.to(cuda), torch.float16)
    assert torch.equal(a, b)
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("m,n,k", [(9000, 1000, 1024), (65520, 512, 256)])
def test_large_m_spans_several_tile_groups(cuda, m, n, k):
    # More than 16 pair m-tiles: the tile order walks groups of 16 m-tiles; every
    # tile must still be computed once.  Exact reference: int8 products summed in
    # float64 (|sum| < 2^53), one rounding to fp32, then the fp32 epilogue.
    g = torch.Generator().manual_seed(m + n)
    xq = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8).to(cuda)
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8).to(cuda)
    xs = (torch.rand(m, generator=g) * 0.02 + 1e-4).to(cuda)
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-5).to(cuda)
    y = ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.float16)
    acc = (xq.double() @ wq.double().t()).float()
    ref = (acc * xs[:, None] * ws[None, :]).to(torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
