"""Parity of the quantiser's fused input activation and rotation-free branch
(tg_quantize_act) on the GPU.

* Fused ``input_act`` (tilegen/comfyui/backend.py:201-204): the reference
  applies the activation as its own op on the fp16/bf16 tensor and then
  quantises.  The fused kernel must give the same codes and scales bit for bit
  as that composition run here: torch's ``F.gelu`` on the GPU, then the
  rotate+quant kernel, and the oracle on the activated tensor.
* Rotation-free branch (backend.py:230-232): bit-identical to torch's own
  evaluation of those two lines on the GPU (scales NaN exactly where torch's
  are), and to the oracle that restates them.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from tests._util import DT_NAME, raw16
from tests.conftest import GOLDEN
from tilegen_b200 import ops
from tilegen_b200.quant.rowwise import _torch_rowwise, quantize_rowwise
from tilegen_b200.synthetic import outlier_activations

pytestmark = pytest.mark.gpu

ACTS = {
    "gelu_tanh": lambda x: F.gelu(x, approximate="tanh"),
    "gelu": lambda x: F.gelu(x),
}


def _same_scales(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.cpu(), b.cpu()
    nan_a, nan_b = torch.isnan(a), torch.isnan(b)
    return torch.equal(nan_a, nan_b) and torch.equal(a[~nan_a].view(torch.int32), b[~nan_b].view(torch.int32))


def _assert_same(q, s, rq, rs, what: str):
    q, rq = q.cpu(), rq.cpu()
    bad = (q != rq).nonzero()
    assert bad.numel() == 0, f"{what}: {bad.shape[0]} codes differ, first at {bad[:3].tolist()}"
    assert _same_scales(s, rs), f"{what}: scales differ"


@pytest.mark.parametrize("act", sorted(ACTS))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("group", [4, 64, 256])
def test_fused_act_equals_act_then_quantise(cuda, act, dtype, group):
    for m, k in ((1, 256), (67, 5120), (9, 13824)):
        x = outlier_activations(m, k, seed=m + k + group, dtype=dtype).to(cuda)
        q, s = ops.quantize_act(x, group, act)
        xa = ACTS[act](x)
        rq, rs = ops.rotate_quant(xa, group)
        torch.cuda.synchronize()
        _assert_same(q, s, rq, rs, f"{act} {dtype} G={group} M={m} K={k}")
        oq, os_ = oracle.rotate_quant(raw16(xa), DT_NAME[dtype], group, order="short")
        assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)


@pytest.mark.parametrize("act", sorted(ACTS))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_act_over_the_activation_range(cuda, act, dtype):
    """Every fp16 / bf16 value once (the tanh/erf branches, overflow, NaN and inf included)."""
    bits = (torch.arange(0, 1 << 16, dtype=torch.int32) - 32768).to(torch.int16)
    x = bits.view(dtype).reshape(256, 256).to(cuda)
    q, s = ops.quantize_act(x, 1, act)
    rq, rs = _torch_rowwise(ACTS[act](x))
    torch.cuda.synchronize()
    _assert_same(q, s, rq, rs, f"{act} all fp16 values")
    # the activation values themselves, through the rotation-free identity on
    # single-element rows: the scale of a row [a] is |a| * fp32(1/127) (or 1e-30)
    xb = bits.view(dtype).reshape(-1, 1)
    xb = torch.cat([xb, torch.zeros(xb.shape[0], 63, dtype=dtype)], 1).to(cuda)
    _, s1 = ops.quantize_act(xb, 1, act)
    _, rs1 = _torch_rowwise(ACTS[act](xb))
    torch.cuda.synchronize()
    assert _same_scales(s1, rs1), f"{act}: activation values differ from torch's"


def _special_rows(k: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    x = outlier_activations(12, k, seed=seed, dtype=dtype)
    x[0].zero_()                                                     # 0/0 codes
    x[1] = x[1].float().mul(1e-8).to(dtype)                          # fp16 divisor underflows
    x[2] = x[2].float().mul(1e-7).to(dtype)                          # fp16 divisor subnormal
    x[3] = x[3].float().mul(2000.0).clamp(-60000, 60000).to(dtype)  # near fp16 max
    x[4, 5] = float("nan")                                           # NaN scale, all codes 0
    x[5, 7] = float("inf")                                           # inf scale
    x[6, 9] = -float("inf")
    # absmax values where fp32 a/127 and a * fp32(1/127) differ (the scale
    # must follow torch's CUDA evaluation, the reciprocal product)
    r = torch.tensor(1.0) / torch.tensor(127.0)
    cand = torch.arange(1, 200, 0.25, dtype=torch.float32).to(dtype).float().unique()
    split = cand[cand / torch.tensor(127.0) != cand * r]
    for i, row in enumerate(range(7, 12)):
        x[row] = x[row].float().mul(0.01).to(dtype)
        x[row, (13 * i) % k] = split[(7 * i) % split.numel()].to(dtype)
    return x


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("k", [64, 320, 5120, 13824])
def test_rowwise_equals_torch_on_gpu(cuda, dtype, k):
    x = _special_rows(k, dtype, seed=k).to(cuda)
    q, s = ops.quantize_act(x, 1, None)
    rq, rs = _torch_rowwise(x)
    torch.cuda.synchronize()
    _assert_same(q, s, rq, rs, f"rowwise {dtype} K={k}")
    oq, os_ = oracle.rowwise_quant(raw16(x), DT_NAME[dtype])
    assert np.array_equal(q.cpu().numpy(), oq)
    assert _same_scales(s, torch.from_numpy(os_))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rowwise_exhaustive(cuda, dtype):
    """Every (value, row absmax) pair of the dtype: for each finite absmax a, one
    row holds the non-negative values up to a and one holds +a and the
    negative values down to -a (K = 32768, zero padded).  This covers every
    divisor the row-wise branch can see and every value it divides, on both the
    fast quotient path and the underflowed-divisor path."""
    k = 32768
    top = 0x7BFF if dtype == torch.float16 else 0x7F7F  # largest finite bit pattern
    idx = torch.arange(k, device=cuda, dtype=torch.int32)[None, :]
    checked = 0
    for a0 in range(0, top + 1, 2048):
        a = torch.arange(a0, min(a0 + 2048, top + 1), device=cuda, dtype=torch.int32)[:, None]
        pos = torch.where(idx <= a, idx, 0)
        neg = torch.where((idx >= 1) & (idx <= a), idx - 32768, 0)  # sign bit set, as int16
        neg[:, :1] = a
        x = torch.stack([pos, neg], 1).reshape(-1, k).to(torch.int16).view(dtype)
        q, s = ops.quantize_act(x, 1, None)
        rq, rs = _torch_rowwise(x)
        bad = (q != rq).nonzero()
        assert bad.numel() == 0, f"{bad.shape[0]} codes differ from torch, first rows {bad[:3].tolist()}"
        assert torch.equal(s.view(torch.int32), rs.view(torch.int32)), f"scales differ near absmax bits {a0}"
        checked += x.shape[0]
    assert checked == 2 * (top + 1)


@pytest.mark.parametrize("act", sorted(ACTS))
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rowwise_with_act_equals_torch(cuda, act, dtype):
    for m, k in ((1, 64), (33, 5120), (130, 13824)):
        x = outlier_activations(m, k, seed=m + k, dtype=dtype).to(cuda)
        q, s = ops.quantize_act(x, 1, act)
        rq, rs = _torch_rowwise(ACTS[act](x))
        torch.cuda.synchronize()
        _assert_same(q, s, rq, rs, f"rowwise {act} {dtype} M={m} K={k}")


@pytest.mark.parametrize("m", [1, 2, 63, 65, 1000, 4097])
def test_rowwise_ragged_rows(cuda, m):
    x = outlier_activations(m, 5120, seed=m, dtype=torch.bfloat16).to(cuda)
    q, s = ops.quantize_act(x, 1, None)
    rq, rs = _torch_rowwise(x)
    torch.cuda.synchronize()
    _assert_same(q, s, rq, rs, f"rowwise M={m}")


def test_rowwise_golden_fixtures(cuda):
    """The reference's own two lines, run by torch on the CPU: same codes; the
    scales differ from the CPU's division by at most one ulp (CUDA multiplies)."""
    d = np.load(os.path.join(GOLDEN, "rowwise.npz"))
    for name in sorted({f.split("_")[0] for f in d.files}):
        m, k, dt = (int(v) for v in d[f"{name}_meta"])
        dtype = torch.float16 if dt == 1 else torch.bfloat16
        x = torch.from_numpy(d[f"{name}_x"].view(np.int16)).view(dtype).to(cuda)
        q, s = ops.quantize_act(x, 1, None)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), d[f"{name}_q"]), name
        ulps = np.abs(s.cpu().numpy().view(np.int32).astype(np.int64) - d[f"{name}_scale"].view(np.int32))
        assert ulps.max() <= 1, name


def test_quantize_rowwise_dispatch(cuda):
    x = outlier_activations(40, 320, seed=3, dtype=torch.float16).to(cuda)
    q, s = quantize_rowwise(x)
    rq, rs = _torch_rowwise(x)
    _assert_same(q, s, rq, rs, "quantize_rowwise kernel")
    # K not a multiple of 64: the torch lines run instead (same definition)
    x = outlier_activations(40, 100, seed=4, dtype=torch.float16).to(cuda)
    q, s = quantize_rowwise(x)
    rq, rs = _torch_rowwise(x)
    _assert_same(q, s, rq, rs, "quantize_rowwise torch")


@pytest.mark.parametrize("act", ["gelu_tanh", "gelu"])
def test_int8_linear_input_act_equals_reference_composition(cuda, fake_kitchen, act):
    """backend.int8_linear(..., input_act=act): the reference applies
    comfy_kitchen's apply_input_act (the test double: torch F.gelu), then the
    FHT quantiser and the GEMM; the fused path must give the same output bits."""
    from comfy_kitchen.backends._activations import apply_input_act

    from tilegen.comfyui import backend
    from tilegen.kernels.int8_convrot import quantize_convrot_fht
    from tilegen.quant.int8_ops import int8_matmul_dequant_chunked
    from tilegen.quant.weight import quantize_convrot_weight

    x = outlier_activations(2 * 77, 13824, seed=5, dtype=torch.bfloat16).reshape(2, 77, 13824).to(cuda)
    w = torch.randn(640, 13824, generator=torch.Generator().manual_seed(6)).mul(0.02).to(cuda)
    wq, ws = quantize_convrot_weight(w.to(torch.bfloat16), 256)
    bias = torch.randn(640, generator=torch.Generator().manual_seed(7)).to(cuda)
    y = backend.int8_linear(x, wq, ws, bias=bias, out_dtype=torch.bfloat16, convrot=True,
                            convrot_groupsize=256, input_act=act)
    xa = apply_input_act(x, act).reshape(-1, 13824)
    xq, xs = quantize_convrot_fht(xa, 256)
    ref = int8_matmul_dequant_chunked(xq, xs, wq, ws, bias, torch.bfloat16).reshape(2, 77, 640)
    torch.cuda.synchronize()
    assert y.shape == ref.shape
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_registry_rule_on_cuda_inputs(cuda, fake_kitchen, monkeypatch):
    """The selective backend's call rule (the reference's rule order, backend.py:129-163):
    group 256 only, K >= TILEGEN_FHT_MIN_K in auto mode (0 in fht mode), K within the
    kernel's maximum, shapes that failed before refused; everything else accepted."""
    from tilegen_b200 import ops
    from tilegen_b200.comfyui import backend

    def rule(x, group=256):
        return backend._fht_applicable({"x": x, "weight": torch.zeros(8, x.shape[-1], dtype=torch.int8),
                                        "convrot": True, "convrot_groupsize": group})

    x = torch.zeros(4, 5120, dtype=torch.float16, device=cuda)
    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "auto")
    monkeypatch.delenv("TILEGEN_FHT_MIN_K", raising=False)
    assert rule(x).success                                         # Blackwell: min K 0
    assert rule(x, 64).failed_param == "convrot_groupsize"       # other groups: eager, in x's dtype
    assert rule(x.float()).failed_param == "x"                    # fp32: not a kernel input
    monkeypatch.setenv("TILEGEN_FHT_MIN_K", "8192")
    assert rule(x).failed_param == "x"                            # auto: below the threshold
    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "fht")
    assert rule(x).success                                        # fht: no threshold
    big = torch.zeros(1, ops.rotate_quant_max_k() + 256, dtype=torch.float16, device=cuda)
    assert rule(big).failed_param == "x"
    monkeypatch.setattr(backend, "_FAILED_FHT_SHAPES", {(4, 5120, torch.float16, cuda.index or 0)})
    assert rule(x).failed_param == "x"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rowwise_and_fused_act_at_the_dit_block_size(cuda, dtype):
    """65520 rows (the DiT block's 2 x 32760 tokens on one GPU), K=5120: each
    persistent CTA turns its ring hundreds of times.  Row-wise: bit-identical to
    torch's evaluation on the GPU and to the oracle; fused gelu_tanh + rotation:
    bit-identical to torch's GELU followed by the quantiser."""
    x = outlier_activations(65520, 5120, seed=31, dtype=dtype, device=cuda)
    q, s = ops.quantize_act(x, 1, None)
    rq, rs = _torch_rowwise(x)
    torch.cuda.synchronize()
    _assert_same(q, s, rq, rs, "row-wise at 65520 rows")
    oq, os_ = oracle.rowwise_quant(raw16(x), DT_NAME[dtype])
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)
    fq, fs = ops.quantize_act(x, 256, "gelu_tanh")
    uq, us = ops.rotate_quant(F.gelu(x, approximate="tanh"), 256)
    torch.cuda.synchronize()
    _assert_same(fq, fs, uq, us, "fused gelu_tanh at 65520 rows")
