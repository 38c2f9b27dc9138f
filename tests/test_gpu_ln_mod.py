"""Parity of the quantiser with the fused LayerNorm + modulation prologue
(tg_quantize_ln_mod, ops.quantize_ln_mod) on the GPU.

The kernel's arithmetic is restated by the oracle: oracle.ln_mod (the modulated
rows, in x's dtype) followed by the short-order rotate+quant
(oracle_rotate_quant_short) -- codes and scales must be bit-identical.  Against
torch's own composition, F.layer_norm(x, (K,), eps) * (1 + scale) + shift then
the quantiser, the row statistics are summed in another order, so the parity
tolerance applies: codes equal except +-1 on at most 0.1 % of the elements,
scales within 1e-3 relative.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from tests._util import DT_NAME, raw16
from tilegen_b200 import _lib, ops
from tilegen_b200.synthetic import dit_modulation, residual_stream

pytestmark = pytest.mark.gpu

CODE_TOL_FRAC = 1e-3   # parity tolerance: +-1 on <= 0.1 % of codes
SCALE_TOL_REL = 1e-3   # parity tolerance: scales within 1e-3 relative


@pytest.fixture(autouse=True)
def _healthy_device(cuda):
    yield
    assert _lib.device_status(0) == 0


def _oracle(x, scale, shift, eps, rows, group):
    y = oracle.ln_mod(raw16(x), DT_NAME[x.dtype], eps, raw16(scale), raw16(shift), rows)
    return oracle.rotate_quant(y, DT_NAME[x.dtype], group, order="short")


def _check_exact(x, scale, shift, eps, rows, group, dev):
    q, s = ops.quantize_ln_mod(x.to(dev), group, scale.to(dev), shift.to(dev), eps, rows)
    torch.cuda.synchronize()
    rq, rs = _oracle(x, scale, shift, eps, rows, group)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    bad = np.argwhere(q != rq)
    assert bad.size == 0, f"{len(bad)} codes differ, first at {bad[:3].tolist()}"
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32)), "scales differ"
    return q, s


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("k", [256, 1536, 5120, 13824])
def test_bit_exact_vs_oracle(cuda, k, dtype):
    for m, rows in ((1, 1), (3, 1), (66, 33), (130, 130)):
        x = residual_stream(m, k, seed=k + m, dtype=dtype)
        scale, shift = dit_modulation(-(-m // rows), k, seed=m, dtype=dtype)
        _check_exact(x, scale, shift, 1e-6, rows, 256, cuda)


@pytest.mark.parametrize("group", [4, 16, 64])
def test_other_groups(cuda, group):
    x = residual_stream(70, 3072, seed=group, dtype=torch.bfloat16)
    scale, shift = dit_modulation(2, 3072, seed=1, dtype=torch.bfloat16)
    _check_exact(x, scale, shift, 1e-5, 35, group, cuda)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dit_block_size_vs_oracle_and_torch(cuda, dtype):
    """4096 tokens of two samples at K=5120 (the qkv / ffn_up input): bit-identical to
    the oracle, and within the parity tolerance of torch's LayerNorm + modulation
    followed by the quantiser."""
    m, k = 4096, 5120
    x = residual_stream(m, k, seed=7, dtype=dtype)
    scale, shift = dit_modulation(2, k, seed=8, dtype=dtype)
    q, s = _check_exact(x, scale, shift, 1e-6, m // 2, 256, cuda)
    xd, sc, sh = x.to(cuda), scale.to(cuda), shift.to(cuda)
    vec = torch.arange(m, device=cuda) // (m // 2)
    y = F.layer_norm(xd, (k,), eps=1e-6) * (1 + sc[vec]) + sh[vec]
    tq, ts = ops.rotate_quant(y, 256)
    diff = np.abs(q.astype(np.int32) - tq.cpu().numpy().astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() <= CODE_TOL_FRAC
    assert (np.abs(s - ts.cpu().numpy()) / ts.cpu().numpy()).max() <= SCALE_TOL_REL


def test_many_rows_and_per_row_vectors(cuda):
    """65520 rows (many ring turns per CTA) with one modulation vector per 4095 rows."""
    m, k = 65520, 5120
    x = residual_stream(m, k, seed=11, dtype=torch.float16, device=cuda).cpu()
    scale, shift = dit_modulation(16, k, seed=12, dtype=torch.float16)
    _check_exact(x, scale, shift, 1e-6, 4095, 256, cuda)


def test_special_rows(cuda):
    k = 1536
    x = residual_stream(6, k, seed=5, dtype=torch.float32)
    x[0] = 0.0                        # zero row: LN gives 0, y = shift
    x[1] = -3.25                      # constant row
    x[2, 9] = float("inf")            # inf: the row's statistics and outputs are NaN
    x[3, 100] = float("nan")
    x[4] *= 1e-4                      # tiny values (fp16 subnormals in places)
    scale, shift = dit_modulation(1, k, seed=6, dtype=torch.float32)
    for dt in (torch.float16, torch.bfloat16):
        _check_exact(x.to(dt), scale.to(dt), shift.to(dt), 1e-6, 6, 256, cuda)


def test_shapes_and_broadcast_vectors(cuda):
    """[B, L, K] activations with [B, 1, K] vectors (a DiT's per-sample modulation),
    and one [K] vector for every row."""
    b, l, k = 3, 40, 1024
    x = residual_stream(b * l, k, seed=9, dtype=torch.float16)
    scale, shift = dit_modulation(b, k, seed=10, dtype=torch.float16)
    q3, s3 = ops.quantize_ln_mod(x.view(b, l, k).to(cuda), 256, scale.view(b, 1, k).to(cuda),
                                 shift.view(b, 1, k).to(cuda))
    rq, rs = _oracle(x, scale, shift, 1e-6, l, 256)
    assert np.array_equal(q3.cpu().numpy(), rq) and np.array_equal(s3.cpu().numpy(), rs)
    q1, s1 = ops.quantize_ln_mod(x.to(cuda), 256, scale[0].to(cuda), shift[0].to(cuda))
    rq, rs = _oracle(x, scale[:1], shift[:1], 1e-6, b * l, 256)
    assert np.array_equal(q1.cpu().numpy(), rq) and np.array_equal(s1.cpu().numpy(), rs)


def test_empty_and_rejects(cuda):
    k = 512
    sc, sh = dit_modulation(1, k, dtype=torch.float16, device=cuda)
    q, s = ops.quantize_ln_mod(torch.empty(0, k, dtype=torch.float16, device=cuda), 256, sc, sh)
    assert q.shape == (0, k) and s.shape == (0,)
    x = torch.zeros(4, k, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.quantize_ln_mod(x, 1, sc, sh)                       # row-wise group
    with pytest.raises(ValueError):
        ops.quantize_ln_mod(x, 256, sc, sh, eps=-1.0)
    with pytest.raises(ValueError):
        ops.quantize_ln_mod(x, 256, torch.zeros(3, k, dtype=torch.float16, device=cuda), sh)
    with pytest.raises(ValueError):
        ops.quantize_ln_mod(x, 256, sc, sh, rows_per_vector=2)   # 2 vectors needed, 1 given
    with pytest.raises(ValueError):
        ops.quantize_ln_mod(x.float(), 256, sc, sh)


def test_linear_with_fused_norm_matches_unfused(cuda):
    """A projection fed by the fused quantiser is within 1e-3 (relative Frobenius) of
    the same projection fed by torch's LayerNorm + modulation and the quantiser:
    the few codes that differ by one move the output by far less than the int8
    quantisation itself."""
    from tilegen_b200.synthetic import gaussian_weight

    m, k, n = 512, 5120, 1024
    x = residual_stream(m, k, seed=21, dtype=torch.bfloat16, device=cuda)
    scale, shift = dit_modulation(1, k, seed=22, dtype=torch.bfloat16, device=cuda)
    wq, ws = ops.rotate_quant(gaussian_weight(n, k, seed=23, dtype=torch.bfloat16, device=cuda), 256)
    xq, xs = ops.quantize_ln_mod(x, 256, scale, shift)
    y = ops.int8_gemm_dequant(xq, xs, wq, ws, None, torch.bfloat16)
    ref = F.layer_norm(x, (k,), eps=1e-6) * (1 + scale) + shift
    rq, rs = ops.rotate_quant(ref, 256)
    y_ref = ops.int8_gemm_dequant(rq, rs, wq, ws, None, torch.bfloat16)
    rel = float((y.float() - y_ref.float()).norm() / y_ref.float().norm())
    assert rel < 1e-3, rel


def test_fused_linear_in_graph_matches_eager(cuda):
    """The fused quantiser and the GEMM after it (its programmatic dependent),
    captured in a CUDA graph and replayed: identical to the eager calls."""
    from tilegen_b200.synthetic import gaussian_weight

    m, k, n = 256, 5120, 640
    x = residual_stream(m, k, seed=31, dtype=torch.float16, device=cuda)
    scale, shift = dit_modulation(2, k, seed=32, dtype=torch.float16, device=cuda)
    wq, ws = ops.rotate_quant(gaussian_weight(n, k, seed=33, dtype=torch.float16, device=cuda), 256)

    def linear():
        return ops.int8_gemm_dequant(*ops.quantize_ln_mod(x, 256, scale, shift), wq, ws, None, torch.float16)

    eager = linear()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        linear()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = linear()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)


def test_custom_op_matches(cuda):
    x = residual_stream(64, 3072, seed=41, dtype=torch.bfloat16, device=cuda)
    sc, sh = dit_modulation(1, 3072, seed=42, dtype=torch.bfloat16, device=cuda)
    a = torch.ops.tilegen.quantize_ln_mod(x, 256, sc, sh, 1e-6)
    b = ops.quantize_ln_mod(x, 256, sc, sh, 1e-6)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
