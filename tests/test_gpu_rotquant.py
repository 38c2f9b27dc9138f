"""Parity of the sm_100a rotate+quant kernel (tg_quantize_act) on the GPU.

The kernel has two butterfly orders.  "reference": the oracle's
oracle_rotate_quant restates the reference kernel's arithmetic
(tilegen/kernels/int8_convrot.py:47-104), so codes and scales must be
bit-identical.  "short" (the default): the oracle's oracle_rotate_quant_short
restates the kernel's arithmetic, bit-identical again; against the reference
order (and the golden fixtures, which pin the reference's eager path
_eager_quantize(x.float(), G), int8_convrot.py:289-302) the parity tolerance
applies: codes equal except +-1 on at most 0.1 % of the elements, scales
within 1e-3 relative.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
from tests._util import DT_NAME, oracle_input
from tests.conftest import GOLDEN
from tilegen_b200 import _lib, ops
from tilegen_b200.synthetic import dit_activations, outlier_activations

pytestmark = pytest.mark.gpu

CODE_TOL_FRAC = 1e-3   # parity tolerance: +-1 on <= 0.1 % of codes
SCALE_TOL_REL = 1e-3   # parity tolerance: scales within 1e-3 relative


ORDERS = ["short", "reference"]


def _run_and_check(x_cpu: torch.Tensor, group: int, dev, order: str = "short"):
    q, s = ops.rotate_quant(x_cpu.to(dev), group, order=order)
    torch.cuda.synchronize()
    rq, rs = oracle.rotate_quant(oracle_input(x_cpu), DT_NAME[x_cpu.dtype], group, order=order)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    bad = np.argwhere(q != rq)
    assert bad.size == 0, f"{len(bad)} codes differ, first at {bad[:3].tolist()}"
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32)), "scales differ"
    return q, s


def _within_tolerance(q, s, rq, rs):
    """The parity tolerance: codes +-1 on at most 0.1 % of elements, scales 1e-3 relative."""
    diff = np.abs(q.astype(np.int32) - rq.astype(np.int32))
    assert diff.max(initial=0) <= 1 and (diff > 0).mean() <= CODE_TOL_FRAC
    assert (np.abs(s - rs) / np.maximum(rs, np.float32(1e-30))).max(initial=0) <= SCALE_TOL_REL


@pytest.mark.parametrize("order", ORDERS)
@pytest.mark.parametrize("k", [256, 1536, 3072, 5120, 13824, 32768])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bit_exact_vs_oracle_k_sweep(cuda, k, dtype, order):
    for m in (1, 3, 66):
        x = outlier_activations(m, k, seed=k + m, dtype=dtype)
        _run_and_check(x, 256, cuda, order)


@pytest.mark.parametrize("order", ORDERS)
@pytest.mark.parametrize("group", [4, 16, 64, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bit_exact_vs_oracle_groups(cuda, group, dtype, order):
    for m, k in ((5, 1536), (130, 3072), (7, 5120)):
        x = outlier_activations(m, k, seed=group + m, dtype=dtype)
        _run_and_check(x, group, cuda, order)


@pytest.mark.parametrize("order", ORDERS)
@pytest.mark.parametrize("m", [1, 2, 63, 64, 65, 1000, 4097])
def test_ragged_row_counts(cuda, m, order):
    x = outlier_activations(m, 5120, seed=m, dtype=torch.float16)
    _run_and_check(x, 256, cuda, order)


@pytest.mark.parametrize("order", ORDERS)
def test_full_size_qkv_input(cuda, order):
    """M=4096, K=5120 fp16 with 1 % outlier channels x30 (the qkv_proj activations)."""
    x = dit_activations("qkv_proj", 4096, seed=0, dtype=torch.float16)
    _run_and_check(x, 256, cuda, order)


@pytest.mark.parametrize("order", ORDERS)
def test_full_size_ffn_down_input_bf16(cuda, order):
    """M=4096, K=13824 bf16 GELU activations with 0.5 % outlier channels x50."""
    x = dit_activations("ffn_down", 4096, seed=0, dtype=torch.bfloat16)
    _run_and_check(x, 256, cuda, order)


@pytest.mark.parametrize("m", [65520, 65536])
@pytest.mark.parametrize("k", [5120, 13824])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dit_block_and_sweep_sizes(cuda, m, k, dtype):
    """The DiT block's 2 x 32760 tokens on one GPU and the quantiser sweep's largest M.

    At these sizes each persistent CTA runs hundreds of batches through its
    TMA ring (the mbarrier phase flips every ring turn).  Default order:
    bit-identical to the oracle's restatement of it, and within the parity
    tolerance of the reference order.
    """
    x = outlier_activations(m, k, seed=m + k, dtype=dtype, device=cuda).cpu()  # generated on the GPU: faster
    q, s = _run_and_check(x, 256, cuda, "short")
    rq, rs = oracle.rotate_quant(oracle_input(x), DT_NAME[dtype], 256, order="reference")
    _within_tolerance(q, s, rq, rs)


def test_orders_agree_within_tolerance(cuda):
    """Short order vs reference order on the GPU, at the qkv activations' size."""
    x = dit_activations("qkv_proj", 4096, seed=1, dtype=torch.float16).to(cuda)
    q, s = ops.rotate_quant(x, 256, order="short")
    rq, rs = ops.rotate_quant(x, 256, order="reference")
    _within_tolerance(q.cpu().numpy(), s.cpu().numpy(), rq.cpu().numpy(), rs.cpu().numpy())


@pytest.mark.parametrize("order", ORDERS)
def test_nan_and_inf_rows_each_order(cuda, order):
    """Rows with NaN or inf take the clamped code form in the short order too."""
    k = 5120
    x = outlier_activations(6, k, seed=11, dtype=torch.float32)
    x[0, 300] = float("nan")
    x[1, 7] = float("inf")
    x[2, 9] = float("-inf")
    x[3, 1000] = float("nan")
    x[3, 4000] = float("inf")
    x[4, :] = float("nan")
    for dt in (torch.float16, torch.bfloat16):
        _run_and_check(x.to(dt), 256, cuda, order)
        _run_and_check(x.to(dt), 64, cuda, order)


def test_special_values(cuda):
    k = 1536
    x = outlier_activations(8, k, seed=9, dtype=torch.float32)
    x[0] = 0.0                       # all-zero row: scale clamps to 1e-30, codes 0
    x[1] *= 1e-6                     # tiny values (fp16 subnormals)
    x[2] = x[2].sign() * 65504.0     # fp16 max magnitude everywhere
    x[3, 17] = float("nan")          # NaN is skipped by the absmax and coded -128
    x[4, 5] = float("inf")           # inf row: scale inf, the inf element NaN -> -128
    x[5, :256] = -0.0
    for order in ORDERS:
        for dt in (torch.float16, torch.bfloat16):
            q, s = _run_and_check(x.to(dt), 256, cuda, order)
        assert (q[0] == 0).all() and s[0] == np.float32(1e-30)


@pytest.mark.parametrize("order", ORDERS)
def test_bf16_large_magnitudes(cuda, order):
    x = outlier_activations(4, 3072, seed=5, dtype=torch.float32) * 1e30
    _run_and_check(x.to(torch.bfloat16), 256, cuda, order)


def test_against_reference_golden_vectors(cuda):
    """The reference eager path's outputs (tests/golden/quant.npz) within the parity tolerance (codes +-1 on <= 0.1 %, scales 1e-3 relative)."""
    d = np.load(os.path.join(GOLDEN, "quant.npz"))
    names = sorted({f.split("_")[0] for f in d.files})
    checked = 0
    for n in names:
        m, k, g, dt = (int(v) for v in d[f"{n}_meta"])
        if dt == 0:
            continue  # fp32 inputs: the kernel reads fp16/bf16
        raw = torch.from_numpy(d[f"{n}_x"].view(np.int16))
        x = raw.view(torch.float16 if dt == 1 else torch.bfloat16)
        q, s = ops.rotate_quant(x.to(cuda), g)
        q, s = q.cpu().numpy().astype(np.int32), s.cpu().numpy()
        rq, rs = d[f"{n}_q"].astype(np.int32), d[f"{n}_scale"]
        diff = np.abs(q - rq)
        assert diff.max() <= 1 and (diff > 0).mean() <= CODE_TOL_FRAC, n
        assert (np.abs(s - rs) / rs).max() <= SCALE_TOL_REL, n
        checked += 1
    assert checked >= 4


def test_deterministic_and_idempotent_inputs(cuda):
    x = outlier_activations(300, 5120, seed=3, dtype=torch.float16).to(cuda)
    x_before = x.clone()
    a = ops.rotate_quant(x, 256)
    b = ops.rotate_quant(x, 256)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert torch.equal(x, x_before)  # input untouched


def test_unaligned_and_strided_inputs(cuda):
    base = outlier_activations(17, 5120 + 8, seed=4, dtype=torch.float16).to(cuda)
    x = base[:, 8:]  # non-contiguous and 16-byte misaligned rows
    q, s = ops.rotate_quant(x, 256)
    rq, rs = oracle.rotate_quant(oracle_input(x.cpu()), "float16", 256, order="short")
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_empty_input(cuda):
    q, s = ops.rotate_quant(torch.empty(0, 5120, dtype=torch.float16, device=cuda), 256)
    assert q.shape == (0, 5120) and s.shape == (0,)


def test_rejects_unsupported(cuda):
    x = torch.zeros(4, 5120, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        ops.rotate_quant(x, 128)          # not a power of four (reference rejects it too)
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros(4, 320, dtype=torch.float16, device=cuda), 64)
    with pytest.raises(ValueError):
        ops.rotate_quant(x.float(), 256)  # fp32 is not a kernel input dtype
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros(2, ops.rotate_quant_max_k() + 256, dtype=torch.float16, device=cuda), 256)
    with pytest.raises(ValueError):
        ops.rotate_quant(x, 256, order="sylvester")


def test_custom_op_matches(cuda):
    x = outlier_activations(64, 3072, seed=8, dtype=torch.bfloat16).to(cuda)
    a = torch.ops.tilegen.rotate_quant(x, 256)
    b = ops.rotate_quant(x, 256)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_device_status_clean(cuda):
    assert _lib.device_status(0) == 0
