"""The CPU oracle against the reference's own outputs (tests/golden/*.npz).

This pins the oracle before it is trusted as the checker: its rotate+quant must
reproduce the reference eager path's codes and scales (they agree exactly on
every fixture case; the parity tolerance is the bound asserted), and its
GEMM + dequant must reproduce int8_matmul_dequant_chunked bit for bit.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import GOLDEN

DT_NAMES = ["float32", "float16", "bfloat16"]


def _quant_cases():
    d = np.load(os.path.join(GOLDEN, "quant.npz"))
    return d, sorted({f.split("_")[0] for f in d.files})


def test_rotate_quant_matches_reference_eager():
    d, names = _quant_cases()
    assert len(names) == 7
    for n in names:
        m, k, g, dt = (int(v) for v in d[f"{n}_meta"])
        q, s = oracle.rotate_quant(d[f"{n}_x"], DT_NAMES[dt], g)
        rq, rs = d[f"{n}_q"], d[f"{n}_scale"]
        diff = np.abs(q.astype(np.int32) - rq.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() <= 1e-3, n
        assert (np.abs(s - rs) / rs).max() <= 1e-6, n
        # on these fixtures the agreement is exact
        assert np.array_equal(q, rq), n


@pytest.mark.parametrize("order", ["reference", "short"])
def test_both_orders_within_tolerance_of_reference_eager(order):
    """Both butterfly orders against the reference eager path: codes +-1 on <= 0.1 %,
    scales 1e-3 relative (the parity tolerance; observed: identical codes)."""
    d, names = _quant_cases()
    for n in names:
        m, k, g, dt = (int(v) for v in d[f"{n}_meta"])
        q, s = oracle.rotate_quant(d[f"{n}_x"], DT_NAMES[dt], g, order=order)
        diff = np.abs(q.astype(np.int32) - d[f"{n}_q"].astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() <= 1e-3, n
        assert (np.abs(s - d[f"{n}_scale"]) / d[f"{n}_scale"]).max() <= 1e-3, n


def test_short_order_vs_reference_order_on_dit_activations():
    """The kernel's default order against the reference kernel's order on 256 x 13824
    GELU activations and 256 x 5120 outlier activations: within tolerance."""
    from tests._util import raw16
    from tilegen_b200.synthetic import dit_activations

    for name, dt in (("ffn_down", torch.bfloat16), ("qkv_proj", torch.float16)):
        x = raw16(dit_activations(name, 256, seed=3, dtype=dt))
        dn = "bfloat16" if dt == torch.bfloat16 else "float16"
        q, s = oracle.rotate_quant(x, dn, 256, order="short")
        rq, rs = oracle.rotate_quant(x, dn, 256, order="reference")
        diff = np.abs(q.astype(np.int32) - rq.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() <= 1e-3
        assert (np.abs(s - rs) / rs).max() <= 1e-3


def test_short_order_planted_mistake_is_caught():
    """The short order's outputs come out digit-reversed (output 3 - i at input i);
    a copy that forgets the reversal (planted here, in numpy) gives other codes."""
    x = np.random.default_rng(1).standard_normal((4, 256)).astype(np.float32)
    q, s = oracle.rotate_quant(x, "float32", 256, order="short")
    y = x.copy()
    for st in range(4):
        st_s = 1 << (2 * st)
        for b in range(64):
            base = (b // st_s) * 4 * st_s + b % st_s
            a = [y[:, base + i * st_s].copy() for i in range(4)]
            tot = (a[0] + a[2]) + (a[1] + a[3])
            for i in range(4):
                y[:, base + i * st_s] = tot - np.float32(2) * a[i]  # planted: should be a[3 - i]
    inv = (np.float32(1) / (s * np.float32(16))).astype(np.float32)
    bad = np.clip(np.rint((y * inv[:, None]).astype(np.float32)), -128, 127).astype(np.int8)
    assert (bad != q).mean() > 0.5


def test_weight16_fixture_both_orders():
    """fp16/bf16-valued weights quantised by the reference in fp32 (tests/golden/weight16.npz):
    both orders within the parity tolerance."""
    d = np.load(os.path.join(GOLDEN, "weight16.npz"))
    for name, dt in (("f16", "float16"), ("bf16", "bfloat16")):
        for order in ("reference", "short"):
            q, s = oracle.rotate_quant(d[f"{name}_w"], dt, 256, order=order)
            diff = np.abs(q.astype(np.int32) - d[f"{name}_wq"].astype(np.int32))
            assert diff.max() <= 1 and (diff > 0).mean() <= 1e-3, (name, order)
            assert (np.abs(s - d[f"{name}_wscale"]) / d[f"{name}_wscale"]).max() <= 1e-3, (name, order)


def test_weight_quant_matches_reference():
    d = np.load(os.path.join(GOLDEN, "weight.npz"))
    q, s = oracle.rotate_quant(d["w"], "float32", 256)
    assert np.array_equal(q, d["wq"])
    assert (np.abs(s - d["wscale"]) / d["wscale"]).max() <= 1e-6


def test_gemm_dequant_bit_exact_vs_reference():
    d = np.load(os.path.join(GOLDEN, "gemm.npz"))
    for n in "abcd":
        m, nn, k, od, has_bias, scalar = (int(v) for v in d[f"{n}_meta"])
        y = oracle.int8_gemm_dequant(d[f"{n}_xq"], d[f"{n}_xscale"], d[f"{n}_wq"], d[f"{n}_wscale"],
                                     d[f"{n}_bias"] if has_bias else None, DT_NAMES[od])
        assert np.array_equal(y.view(np.uint8), d[f"{n}_y"].view(np.uint8)), n


def test_cpu_workload_end_to_end():
    """The CPU reference workload: same seeded inputs, scales and head outputs."""
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    g = np.load(os.path.join(GOLDEN, "cpu_workload_256x5120.npz"))
    x = outlier_activations(256, 5120, seed=0, dtype=torch.float32)
    w = gaussian_weight(5120, 5120, seed=0)
    sha = lambda t: hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    assert sha(x) == str(g["x_sha"]) and sha(w) == str(g["w_sha"]), "seeded inputs changed"
    xq, xs = oracle.rotate_quant(x.numpy(), "float32", 256)
    wq, ws = oracle.rotate_quant(w.numpy(), "float32", 256)
    assert (np.abs(xs - g["xscale"]) / g["xscale"]).max() <= 1e-5
    assert (np.abs(ws - g["wscale"]) / g["wscale"]).max() <= 1e-5
    dq = np.abs(xq[:8].astype(int) - g["xq_head"].astype(int))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3
    y = oracle.int8_gemm_dequant(xq[:8], xs[:8], wq, ws, None, "float32")
    rel = np.linalg.norm(y - g["y_head"]) / np.linalg.norm(g["y_head"])
    assert rel <= 1e-2
    assert float(g["rel_vs_dense"]) < 2e-2


def test_planted_mistake_is_caught():
    """A wrong butterfly sign (planted in a Python copy of the oracle's math) changes the codes."""
    x = np.random.default_rng(0).standard_normal((2, 256)).astype(np.float32)
    q, _ = oracle.rotate_quant(x, "float32", 256)
    y = x.copy().reshape(2, 256)
    for st in range(4):
        s = 1 << (2 * st)
        for b in range(64):
            base = (b // s) * 4 * s + b % s
            a0, a1, a2, a3 = (y[:, base + i * s].copy() for i in range(4))
            y[:, base], y[:, base + s] = a0 + a1 + a2 - a3, a0 + a1 - a2 + a3
            y[:, base + 2 * s], y[:, base + 3 * s] = a0 - a1 + a2 + a3, a0 + a1 + a2 + a3  # planted: -a0 -> +a0
    scale = np.maximum(np.abs(y).max(1) / 2032, 1e-30)
    bad = np.clip(np.rint(y / (16 * scale[:, None])), -128, 127).astype(np.int8)
    assert not np.array_equal(bad, q)


def test_rejects_bad_groups():
    with pytest.raises(ValueError):
        oracle.rotate_quant(np.zeros((1, 256), np.float32), "float32", 128)
    with pytest.raises(ValueError):
        oracle.rotate_quant(np.zeros((1, 320), np.float32), "float32", 256)


def _rowwise_cases():
    d = np.load(os.path.join(GOLDEN, "rowwise.npz"))
    for name in sorted({k.split("_")[0] for k in d.files}):
        m, k, dt = (int(v) for v in d[f"{name}_meta"])
        yield name, d[f"{name}_x"], ("float16" if dt == 1 else "bfloat16"), d[f"{name}_q"], d[f"{name}_scale"]


def test_rowwise_matches_reference_lines():
    """oracle_rowwise_quant vs backend.py:231-232 run by torch on the CPU.

    Codes are identical.  Scales are identical except where torch's CPU kernel
    and its CUDA kernel evaluate `amax.float() / 127.0` differently: the CPU
    divides, CUDA multiplies by fp32(1/127), and the oracle restates the CUDA
    evaluation (the product's device).  The fixtures plant absmax values where
    the two differ; there the fixture must equal the division and the oracle
    the reciprocal product, one ulp apart.
    """
    r = np.float32(1) / np.float32(127)
    split_rows = 0
    for name, x, dt, gq, gs in _rowwise_cases():
        q, s = oracle.rowwise_quant(x, dt)
        assert np.array_equal(q, gq), name
        xf = torch.from_numpy(x.view(np.int16)).view(torch.float16 if dt == "float16" else torch.bfloat16)
        amax = xf.float().abs().amax(dim=1).numpy()
        div = np.maximum(amax / np.float32(127), np.float32(1e-30))
        mul = np.maximum(amax * r, np.float32(1e-30))
        assert np.array_equal(gs.view(np.uint32), div.view(np.uint32)), name
        assert np.array_equal(s.view(np.uint32), mul.view(np.uint32)), name
        split_rows += int(np.sum(div != mul))
    assert split_rows >= 6  # the planted rows really separate the two evaluations


def test_rowwise_planted_mistake_is_caught():
    """A code off by one in the oracle's output would fail the fixture comparison."""
    name, x, dt, gq, _ = next(_rowwise_cases())
    q, _ = oracle.rowwise_quant(x, dt)
    q[0, 0] = np.int8(q[0, 0] + (1 if q[0, 0] < 127 else -1))
    assert not np.array_equal(q, gq)
