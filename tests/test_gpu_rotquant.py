"""Parity of the sm_100a rotate+quant kernel (tg_rotate_quant) on the GPU.

The oracle (oracle/convrot_oracle.c) restates the reference kernel's arithmetic
(tilegen/kernels/int8_convrot.py:47-104), so codes and scales must be
bit-identical.  The golden fixtures pin the reference's eager path
(_eager_quantize(x.float(), G), int8_convrot.py:289-302); against it the
parity tolerance applies: codes equal except +-1 on at most 0.1 % of the
elements, scales within 1e-3 relative.
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


def _run_and_check(x_cpu: torch.Tensor, group: int, dev):
    q, s = ops.rotate_quant(x_cpu.to(dev), group)
    torch.cuda.synchronize()
    rq, rs = oracle.rotate_quant(oracle_input(x_cpu), DT_NAME[x_cpu.dtype], group)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    bad = np.argwhere(q != rq)
    assert bad.size == 0, f"{len(bad)} codes differ, first at {bad[:3].tolist()}"
    assert np.array_equal(s.view(np.uint32), rs.view(np.uint32)), "scales differ"
    return q, s


@pytest.mark.parametrize("k", [256, 1536, 3072, 5120, 13824, 32768])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bit_exact_vs_oracle_k_sweep(cuda, k, dtype):
    for m in (1, 3, 66):
        x = outlier_activations(m, k, seed=k + m, dtype=dtype)
        _run_and_check(x, 256, cuda)


@pytest.mark.parametrize("group", [4, 16, 64, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bit_exact_vs_oracle_groups(cuda, group, dtype):
    for m, k in ((5, 1536), (130, 3072), (7, 5120)):
        x = outlier_activations(m, k, seed=group + m, dtype=dtype)
        _run_and_check(x, group, cuda)


@pytest.mark.parametrize("m", [1, 2, 63, 64, 65, 1000, 4097])
def test_ragged_row_counts(cuda, m):
    x = outlier_activations(m, 5120, seed=m, dtype=torch.float16)
    _run_and_check(x, 256, cuda)


def test_full_size_qkv_input(cuda):
    """M=4096, K=5120 fp16 with 1 % outlier channels x30 (the qkv_proj activations)."""
    x = dit_activations("qkv_proj", 4096, seed=0, dtype=torch.float16)
    _run_and_check(x, 256, cuda)


def test_full_size_ffn_down_input_bf16(cuda):
    """M=4096, K=13824 bf16 GELU activations with 0.5 % outlier channels x50."""
    x = dit_activations("ffn_down", 4096, seed=0, dtype=torch.bfloat16)
    _run_and_check(x, 256, cuda)


def test_special_values(cuda):
    k = 1536
    x = outlier_activations(8, k, seed=9, dtype=torch.float32)
    x[0] = 0.0                       # all-zero row: scale clamps to 1e-30, codes 0
    x[1] *= 1e-6                     # tiny values (fp16 subnormals)
    x[2] = x[2].sign() * 65504.0     # fp16 max magnitude everywhere
    x[3, 17] = float("nan")          # NaN is skipped by the absmax and coded -128
    x[4, 5] = float("inf")           # inf row: scale inf, the inf element NaN -> -128
    x[5, :256] = -0.0
    for dt in (torch.float16, torch.bfloat16):
        q, s = _run_and_check(x.to(dt), 256, cuda)
    assert (q[0] == 0).all() and s[0] == np.float32(1e-30)


def test_bf16_large_magnitudes(cuda):
    x = outlier_activations(4, 3072, seed=5, dtype=torch.float32) * 1e30
    _run_and_check(x.to(torch.bfloat16), 256, cuda)


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
    rq, rs = oracle.rotate_quant(oracle_input(x.cpu()), "float16", 256)
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


def test_custom_op_matches(cuda):
    x = outlier_activations(64, 3072, seed=8, dtype=torch.bfloat16).to(cuda)
    a = torch.ops.tilegen.rotate_quant(x, 256)
    b = ops.rotate_quant(x, 256)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_device_status_clean(cuda):
    assert _lib.device_status(0) == 0
