"""End-to-end int8_convrot linear on the GPU through the reference-facing API.

Mirrors the reference's own smoke tests (tests/test_smoke.py:41-91) and adds the
parity targets: the dequantised output within 1e-2 relative Frobenius error
of the reference int8_convrot output (the fp32 CPU workload, x [256, 5120] and
W [5120, 5120]: tests/golden/cpu_workload_256x5120.npz), and codes/scales
within tolerance of the reference eager path at the DiT sizes.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
import tilegen  # the drop-in alias package
from tests._util import raw16, rel_fro
from tests.conftest import GOLDEN
from tilegen.kernels.hadamard import build_hadamard, rotate_by_group
from tilegen.kernels.int8_convrot import _eager_quantize, can_use_fht, quantize_convrot, quantize_convrot_fht
from tilegen.quant.int8_ops import int8_matmul_dequant_chunked
from tilegen.quant.weight import quantize_convrot_weight
from tilegen_b200.synthetic import DIT_SHAPES, dit_activations, gaussian_weight, outlier_activations

pytestmark = pytest.mark.gpu
G = 256
DT = torch.float16


def test_hadamard_is_normalized_and_orthogonal(cuda):
    h = build_hadamard(256, cuda, DT)
    eye = torch.matmul(h, h.t())
    assert rel_fro(eye.cpu(), torch.eye(256, dtype=DT)) < 1e-2


def test_rotate_by_group_preserves_norm(cuda):
    x = torch.randn(8, 5120, device=cuda, dtype=DT) * 0.1
    xr = rotate_by_group(x, build_hadamard(G, cuda, DT), G)
    assert rel_fro(x.float().norm(dim=-1).cpu(), xr.float().norm(dim=-1).cpu()) < 1e-2


def test_weight_quant_shape_and_dtype(cuda):
    w = torch.randn(5120, 5120, device=cuda, dtype=DT) * 0.1
    wq, wscale = quantize_convrot_weight(w, G)
    assert wq.shape == w.shape and wq.dtype == torch.int8
    assert wscale.shape == (5120,) and wscale.dtype == torch.float32


def test_weight_quant_kernel_path_bit_exact_full_qkv_weight(cuda):
    """quantize_convrot_weight on a CUDA bf16 [15360, 5120] weight (the qkv projection) runs
    the rotate+quant kernel: bit-identical to the oracle's restatement of the kernel's order,
    and within the parity tolerance of the reference order (weight.py:14-39)."""
    w = gaussian_weight(15360, 5120, seed=3, dtype=torch.bfloat16, device=cuda)
    wq, ws = quantize_convrot_weight(w, G)
    wq, ws = wq.cpu().numpy(), ws.cpu().numpy()
    rq, rs = oracle.rotate_quant(raw16(w), "bfloat16", G, order="short")
    assert np.array_equal(wq, rq) and np.array_equal(ws.view(np.uint32), rs.view(np.uint32))
    eq, es = oracle.rotate_quant(raw16(w), "bfloat16", G, order="reference")
    d = np.abs(wq.astype(np.int32) - eq.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() <= 1e-3 and (np.abs(ws - es) / es).max() <= 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_weight_quant_kernel_path_vs_reference_outputs(cuda, dtype):
    """The reference's quantize_convrot_weight outputs on fp16/bf16-valued weights
    (tests/golden/weight16.npz) against the kernel path: codes +-1 on <= 0.1 %, scales 1e-3 rel."""
    d = np.load(os.path.join(GOLDEN, "weight16.npz"))
    name = "f16" if dtype == torch.float16 else "bf16"
    w = torch.from_numpy(d[f"{name}_w"].view(np.int16)).view(dtype).to(cuda)
    wq, ws = quantize_convrot_weight(w, G)
    dq = np.abs(wq.cpu().numpy().astype(np.int32) - d[f"{name}_wq"].astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3
    assert (np.abs(ws.cpu().numpy() - d[f"{name}_wscale"]) / d[f"{name}_wscale"]).max() <= 1e-3


def test_weight_quant_fp32_path_vs_reference_outputs(cuda):
    """fp32 weights take the reference's own torch sequence (tests/golden/weight.npz)."""
    d = np.load(os.path.join(GOLDEN, "weight.npz"))
    wq, ws = quantize_convrot_weight(torch.from_numpy(d["w"]).to(cuda), G)
    dq = np.abs(wq.cpu().numpy().astype(np.int32) - d["wq"].astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3
    assert (np.abs(ws.cpu().numpy() - d["wscale"]) / d["wscale"]).max() <= 1e-3


def _torch_gemm_sequence(xq, xs, wq, ws, out_dtype):
    """The reference's GEMM + dequant (int8_ops.py:60-68) as torch runs it on the GPU, unchunked."""
    part = torch._int_mm(xq, wq.t()).float()
    part.mul_(xs.float().reshape(-1, 1))
    part.mul_(ws.float().reshape(1, -1))
    return part.to(out_dtype)


@pytest.mark.parametrize("name,k,n", DIT_SHAPES)
def test_dit_block_linear_8190_rows_bf16(cuda, name, k, n):
    """The DiT-block workload at 8 GPUs: 65520 tokens / 8 = 8190 bf16 rows per GPU (not a
    multiple of 128), each projection through the reference-facing calls.
    * activation and weight codes/scales: bit-identical to the oracle (kernel order) and
      within tolerance of the reference order;
    * output: bit-identical to the reference's torch GEMM sequence on the same codes, and
      to the oracle's GEMM + dequant on the first and last (ragged-tile) rows;
    * output within 1e-2 relative Frobenius of the reference int8_convrot output (the
      reference order's codes through the same exact GEMM)."""
    m = 8190
    x = dit_activations(name, m, seed=5, dtype=torch.bfloat16, device=cuda)
    w = gaussian_weight(n, k, seed=6, dtype=torch.bfloat16, device=cuda)
    xq, xs = quantize_convrot(x, G, backend="fht")
    wq, ws = quantize_convrot_weight(w, G)
    y = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.bfloat16)
    torch.cuda.synchronize()
    xr = raw16(x)
    oq, os_ = oracle.rotate_quant(xr, "bfloat16", G, order="short")
    assert np.array_equal(xq.cpu().numpy(), oq) and np.array_equal(xs.cpu().numpy().view(np.uint32), os_.view(np.uint32))
    ow, ows = oracle.rotate_quant(raw16(w), "bfloat16", G, order="short")
    assert np.array_equal(wq.cpu().numpy(), ow) and np.array_equal(ws.cpu().numpy(), ows)
    ref = _torch_gemm_sequence(xq, xs, wq, ws, torch.bfloat16)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    rows = np.r_[0:4, m - 6:m]
    oy = oracle.int8_gemm_dequant(oq[rows], os_[rows], ow, ows, None, "bfloat16")
    assert np.array_equal(raw16(y[torch.from_numpy(rows).to(cuda)]), oy)
    eq, es = oracle.rotate_quant(xr, "bfloat16", G, order="reference")
    dq = np.abs(oq.astype(np.int32) - eq.astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3 and (np.abs(os_ - es) / es).max() <= 1e-3
    y_ref = _torch_gemm_sequence(torch.from_numpy(eq).to(cuda), torch.from_numpy(es).to(cuda), wq, ws, torch.float32)
    assert rel_fro(y.float().cpu(), y_ref.cpu()) <= 1e-2


def test_fht_vs_eager_numerics(cuda):
    """The reference's own check (test_smoke.py:62-68) against its fp16 eager path."""
    x = torch.randn(2048, 5120, device=cuda, dtype=DT) * 0.1
    xq_fht, xs_fht = quantize_convrot_fht(x, G)
    xq_eager, xs_eager = _eager_quantize(x, G)
    assert (xq_fht.int() - xq_eager.int()).abs().max().item() <= 1
    assert (xs_fht - xs_eager).abs().max().item() < 1e-4


def test_can_use_fht_thresholds(cuda):
    x_cuda = torch.randn(8, 5120, device=cuda, dtype=DT)
    assert can_use_fht(x_cuda, 256, min_k=0) is True
    assert can_use_fht(x_cuda.cpu(), 256) is False
    assert can_use_fht(x_cuda, 128, min_k=0) is False
    assert can_use_fht(x_cuda, 256, min_k=99999) is False
    # the reference's rule: other groups go to the eager path (in x's dtype)
    assert can_use_fht(x_cuda, 64, min_k=0) is False
    xq, xs = quantize_convrot(x_cuda, 64)
    eq, es = _eager_quantize(x_cuda, 64)
    assert torch.equal(xq, eq) and torch.equal(xs, es)


def test_end_to_end_linear_vs_dense(cuda):
    """test_smoke.py:80-91: int8 ConvRot linear vs F.linear, rel-Frobenius < 5e-2."""
    m, k, n = 1024, 5120, 5120
    x = torch.randn(m, k, device=cuda, dtype=DT) * 0.1
    w = torch.randn(n, k, device=cuda, dtype=DT) * 0.1
    bias = torch.randn(n, device=cuda, dtype=DT)
    wq, wscale = quantize_convrot_weight(w, G)
    xq, xscale = quantize_convrot_fht(x, G)
    out = int8_matmul_dequant_chunked(xq, xscale, wq, wscale, bias, DT)
    ref = torch.nn.functional.linear(x, w, bias)
    assert rel_fro(out.cpu(), ref.cpu()) < 5e-2


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cpu_workload_vs_reference_output(cuda, dtype):
    """The CPU reference workload (x [256,5120] with outliers, W [5120,5120]) run through
    the kernels in fp16/bf16: output within 1e-2 relative Frobenius of the reference's
    fp32 int8_convrot output (tests/golden/cpu_workload_256x5120.npz)."""
    g = np.load(os.path.join(GOLDEN, "cpu_workload_256x5120.npz"))
    x = outlier_activations(256, 5120, seed=0, dtype=torch.float32)
    w = gaussian_weight(5120, 5120, seed=0)
    xq, xs = quantize_convrot(x.to(cuda, dtype), G, backend="fht")
    wq, ws = quantize_convrot_weight(w.to(cuda, dtype), G)
    y = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.float32).cpu()
    y_ref_head = torch.from_numpy(g["y_head"])
    assert rel_fro(y[:8], y_ref_head) < 1e-2
    assert abs(float(y.norm()) / float(g["y_norm"]) - 1.0) < 1e-2
    # weight scales of the bf16/fp16-cast weight vs the reference's fp32 weight quant
    assert np.abs(ws.cpu().numpy() / g["wscale"] - 1).max() < 1e-2


def test_cpu_workload_fp32_path_matches_reference_bitwise_in_gemm(cuda):
    """fp32 activations take the eager rotation (as in the reference), the GEMM is
    the fused kernel: with the reference's own codes and scales the output is
    bit-identical to the reference's head rows."""
    g = np.load(os.path.join(GOLDEN, "cpu_workload_256x5120.npz"))
    xq = torch.from_numpy(g["xq_head"]).to(cuda)
    xs = torch.from_numpy(g["xscale"][:8]).to(cuda)
    w = gaussian_weight(5120, 5120, seed=0)
    from tilegen_b200.kernels.hadamard import build_hadamard as bh

    wrot = rotate_by_group(w, bh(G, "cpu", torch.float32), G)
    ws = torch.from_numpy(g["wscale"])
    wq = torch.round(wrot / ws[:, None]).clamp(-128, 127).to(torch.int8)
    y = int8_matmul_dequant_chunked(xq, xs, wq.to(cuda), ws.to(cuda), None, torch.float32).cpu()
    assert rel_fro(y, torch.from_numpy(g["y_head"])) < 1e-5


@pytest.mark.parametrize("name,k,n", DIT_SHAPES)
def test_dit_shapes_codes_and_output_within_tolerance(cuda, name, k, n):
    """Codes +-1 on <= 0.1 %, scales <= 1e-3 rel vs the eager rotation in fp32; output
    rel-Frobenius <= 1e-2 vs dequant(int8 GEMM) of the eager codes."""
    m = 1024
    x = dit_activations(name, m, seed=1, dtype=torch.bfloat16).to(cuda)
    w = gaussian_weight(n, k, seed=2, dtype=torch.bfloat16).to(cuda)
    xq, xs = quantize_convrot_fht(x, G)
    eq, es = _eager_quantize(x.float(), G)
    d = (xq.int() - eq.int()).abs()
    assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 1e-3
    assert ((xs - es).abs() / es).max().item() <= 1e-3
    wq, ws = quantize_convrot_weight(w, G)
    y = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.bfloat16)
    y_ref = int8_matmul_dequant_chunked(eq, es, wq, ws, None, torch.float32)
    assert rel_fro(y.float().cpu(), y_ref.cpu()) <= 1e-2


def test_alias_package_is_the_same_code():
    import tilegen_b200.kernels.int8_convrot as mine

    assert tilegen.kernels.int8_convrot is mine
