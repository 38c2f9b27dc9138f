"""The oracle's restatement of the fused LayerNorm + modulation prologue
(oracle_ln_mod) against torch's own composition on the CPU:
F.layer_norm(x, (K,), eps) * (1 + scale) + shift in x's dtype.  The mean and
variance are summed in different orders (torch: Welford), so the two may differ
by one unit in the last place of x's dtype on a few elements; everything else is
the same sequence of roundings.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from tests._util import DT_NAME, raw16
from tilegen_b200.synthetic import dit_modulation, residual_stream


def _torch_ln_mod(x, scale, shift, eps, rows):
    vec = torch.arange(x.shape[0]) // rows
    return F.layer_norm(x, (x.shape[1],), eps=eps) * (1 + scale[vec]) + shift[vec]


def _ulps(a: np.ndarray, b: np.ndarray, dtype) -> np.ndarray:
    """Distance in units in the last place between two arrays of fp16/bf16 patterns."""
    def key(u):
        v = u.astype(np.int32)
        return np.where(v & 0x8000, 0x8000 - v, v)   # monotone in the represented value
    return np.abs(key(a) - key(b))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("k,rows", [(256, 1), (1536, 3), (5120, 8)])
def test_oracle_ln_mod_matches_torch_within_one_ulp(dtype, k, rows):
    m = 24
    x = residual_stream(m, k, seed=k, dtype=dtype)
    scale, shift = dit_modulation(-(-m // rows), k, seed=k + 1, dtype=dtype)
    y = oracle.ln_mod(raw16(x), DT_NAME[dtype], 1e-6, raw16(scale), raw16(shift), rows)
    ref = raw16(_torch_ln_mod(x, scale, shift, 1e-6, rows))
    d = _ulps(y, ref, dtype)
    assert d.max() <= 2 and (d > 0).mean() <= 0.01, (d.max(), (d > 0).mean())


def test_oracle_ln_mod_special_rows():
    k = 512
    x = residual_stream(4, k, seed=3, dtype=torch.float16)
    x[0] = 1.5                       # constant row: variance 0, LN gives 0, y = shift
    x[1, 7] = float("inf")           # inf: the row's mean is inf, its outputs NaN
    scale, shift = dit_modulation(1, k, seed=4, dtype=torch.float16)
    y = oracle.ln_mod(raw16(x), "float16", 1e-6, raw16(scale), raw16(shift), 4)
    yt = torch.from_numpy(y.view(np.int16)).view(torch.float16)
    assert torch.equal(yt[0], (torch.zeros(k, dtype=torch.float16) * (1 + scale[0]) + shift[0]))
    assert torch.isnan(yt[1]).all()
    with pytest.raises(ValueError):
        oracle.ln_mod(raw16(x), "float16", 1e-6, raw16(scale), raw16(shift), 3)   # 2 vectors needed, 1 given
