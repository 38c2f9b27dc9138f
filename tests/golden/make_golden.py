"""Generate the golden fixtures in this folder from the reference implementation.

Run from the repository root in a container that has the reference sources,
passing the reference checkout's root (required):

    python tests/golden/make_golden.py <reference root> [--only rowwise|weight16]

It imports the reference's own pure-torch functions (they run on the CPU) and
records their outputs on small seeded inputs:

* ``quant.npz``   - ``tilegen.kernels.int8_convrot._eager_quantize(x.float(), G)``
  (int8_convrot.py:289-302) for fp32/fp16/bf16 inputs, several K and G, plus rows
  with zeros, tiny and huge values.
* ``weight.npz``  - ``tilegen.quant.weight.quantize_convrot_weight(W, 256)``
  (weight.py:14-39) on fp32 weights.
* ``weight16.npz`` - the same on fp32 weights whose values are exactly fp16
  (``f16_*``) or bf16 (``bf16_*``) numbers, so that the GPU kernel, which reads
  the 16-bit tensor, sees the reference's inputs exactly.  ``--only weight16``
  writes just this file.
* ``gemm.npz``    - ``tilegen.quant.int8_ops.int8_matmul_dequant_chunked``
  (int8_ops.py:22-70) through CPU ``torch._int_mm``: fp16/bf16/fp32 outputs,
  with and without bias, per-channel and scalar weight scales, small chunk caps.
* ``rowwise.npz`` - the rotation-free branch of the production wrapper
  (tilegen/comfyui/backend.py:230-232), executed from the reference file's own
  two lines (the reference has no function for it) on fp16/bf16 inputs, with
  an all-zero row, a row whose fp16 divisor underflows and near-max values.
  ``--only rowwise`` writes just this file.
* ``cpu_workload_256x5120.npz`` - the CPU reference workload end to end: x fp32 [256, 5120]
  N(0,1) with 1 % outlier channels x30, W fp32 [5120, 5120] N(0, 0.02), seed 0;
  Y = dequant(int8 GEMM).  Stored: input checksums, both scale vectors, the
  first rows of the codes and of Y, and Y's Frobenius norm.

The fixtures are committed; the tests never read the reference at run time.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _u16(t: torch.Tensor) -> np.ndarray:
    """fp16/bf16 tensor -> its raw 16-bit patterns (numpy has no bf16)."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _split_absmax(dtype: torch.dtype, m: int) -> torch.Tensor:
    """m values of ``dtype`` in [1, 256) whose fp32 a/127 and a*fp32(1/127) differ."""
    bits = torch.arange(0, 0x7c00 if dtype == torch.float16 else 0x7f80, dtype=torch.int32)
    vals = bits.to(torch.int16).view(dtype).float()
    vals = vals[(vals >= 1) & (vals < 256)]
    r = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(127.0, dtype=torch.float32)
    split = vals[vals / torch.tensor(127.0) != vals * r]
    idx = torch.linspace(0, split.numel() - 1, m).long()
    return split[idx]


def rowwise(ref_root: str) -> None:
    """Run backend.py:231-232 (the row-wise branch's two statements) on seeded inputs."""
    sys.path.append(REPO)
    from tilegen_b200.synthetic import outlier_activations

    with open(os.path.join(ref_root, "tilegen", "comfyui", "backend.py")) as f:
        lines = f.read().splitlines()[230:232]
    assert lines[0].strip().startswith("xscale =") and lines[1].strip().startswith("xq ="), lines
    code = compile("\n".join(ln.strip() for ln in lines), "backend.py:231-232", "exec")
    dts = {"f16": torch.float16, "bf16": torch.bfloat16}
    out = {}
    cases = [
        # name, M, K, dtype, seed
        ("a", 8, 5120, "f16", 21),
        ("b", 6, 13824, "bf16", 22),
        ("c", 5, 320, "f16", 23),
        ("d", 5, 64, "bf16", 24),
        ("e", 6, 256, "f16", 25),
        ("f", 6, 128, "bf16", 26),
    ]
    for name, m, k, dt, seed in cases:
        x = outlier_activations(m, k, seed=seed, dtype=dts[dt])
        if name in ("c", "d"):
            x[0].zero_()                                      # all-zero row
            x[1] = x[1].float().mul(1e-8).to(x.dtype)         # fp16 divisor underflows to 0
            x[2] = x[2].float().mul(2000.0).clamp(-60000, 60000).to(x.dtype)
            x[3] = x[3].float().mul(1e-7).to(x.dtype)         # fp16 divisor subnormal
        if name in ("e", "f"):
            # absmax values a with fp32(a / 127) != fp32(a * fp32(1/127)): torch's
            # CPU divides, its CUDA kernel multiplies by the reciprocal.
            x = (x.float() * 0.05).to(x.dtype)
            a = _split_absmax(x.dtype, m)
            x[torch.arange(m), torch.arange(m) * 5 + 3] = a.to(x.dtype)
        ns = {"torch": torch, "x2d": x}
        exec(code, ns)
        out[f"{name}_meta"] = np.array([m, k, list(dts).index(dt) + 1], dtype=np.int64)
        out[f"{name}_x"] = _u16(x)
        out[f"{name}_q"] = ns["xq"].numpy()
        out[f"{name}_scale"] = ns["xscale"].numpy()
    np.savez_compressed(os.path.join(HERE, "rowwise.npz"), **out)
    print("rowwise.npz", os.path.getsize(os.path.join(HERE, "rowwise.npz")), "bytes")


def weight16(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.append(REPO)
    from tilegen.quant.weight import quantize_convrot_weight  # reference
    assert os.path.realpath(sys.modules["tilegen"].__file__).startswith(os.path.realpath(ref_root))
    from tilegen_b200.synthetic import gaussian_weight

    out = {}
    for name, dt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
        w16 = gaussian_weight(16, 5120, seed=12, dtype=dt)
        wq, ws = quantize_convrot_weight(w16.float(), 256)
        out[f"{name}_w"] = _u16(w16)
        out[f"{name}_wq"] = wq.numpy()
        out[f"{name}_wscale"] = ws.numpy()
    np.savez_compressed(os.path.join(HERE, "weight16.npz"), **out)
    print("weight16.npz", os.path.getsize(os.path.join(HERE, "weight16.npz")), "bytes")


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    sys.path.append(REPO)
    from tilegen.kernels.int8_convrot import _eager_quantize  # reference
    from tilegen.quant.int8_ops import int8_matmul_dequant_chunked  # reference
    from tilegen.quant.weight import quantize_convrot_weight  # reference
    assert os.path.realpath(sys.modules["tilegen"].__file__).startswith(os.path.realpath(ref_root))
    from tilegen_b200.synthetic import gaussian_weight, outlier_activations

    torch.set_num_threads(os.cpu_count() or 1)
    dts = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

    # ---- activation quantizer -------------------------------------------------
    quant = {}
    cases = [
        # name, M, K, G, dtype, seed
        ("a", 8, 5120, 256, "f16", 1),
        ("b", 6, 13824, 256, "bf16", 2),
        ("c", 16, 1536, 256, "f32", 3),
        ("d", 8, 3072, 64, "f16", 4),
        ("e", 8, 1024, 16, "bf16", 5),
        ("f", 4, 512, 4, "f32", 6),
        ("g", 5, 256, 256, "f16", 7),
    ]
    for name, m, k, g, dt, seed in cases:
        x = outlier_activations(m, k, seed=seed, dtype=dts[dt])
        if name == "g":
            x[0].zero_()                          # all-zero row -> scale clamps to 1e-30
            x[1] = x[1].float().mul(1e-6).to(x.dtype)  # tiny values
            x[2] = x[2].float().mul(2000.0).clamp(-60000, 60000).to(x.dtype)  # near fp16 max
        q, s = _eager_quantize(x.float(), g)
        quant[f"{name}_meta"] = np.array([m, k, g, list(dts).index(dt)], dtype=np.int64)
        quant[f"{name}_x"] = x.numpy() if dt == "f32" else _u16(x)
        quant[f"{name}_q"] = q.numpy()
        quant[f"{name}_scale"] = s.numpy()
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **quant)

    # ---- weight quantizer -----------------------------------------------------
    w = gaussian_weight(16, 5120, seed=11)
    wq, ws = quantize_convrot_weight(w.float(), 256)
    np.savez_compressed(os.path.join(HERE, "weight.npz"), w=w.numpy(), wq=wq.numpy(), wscale=ws.numpy())

    # ---- int8 GEMM + dequant ----------------------------------------------------
    gemm = {}
    gcases = [
        # name, M, N, K, out, bias, scalar wscale, chunk bytes
        ("a", 33, 72, 512, "f16", True, False, 256 << 20),
        ("b", 17, 64, 5120, "bf16", False, False, 256 << 20),
        ("c", 40, 48, 256, "f32", True, True, 256 << 20),
        ("d", 130, 136, 1024, "f16", False, False, 4096),  # forces many row chunks
    ]
    for name, m, n, k, out, has_bias, scalar, cap in gcases:
        g = torch.Generator().manual_seed(100 + m)
        xq = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
        wq_ = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8)
        xs = torch.rand(m, generator=g) * 0.02 + 1e-4
        wsc = torch.rand(1 if scalar else n, generator=g) * 0.01 + 1e-5
        bias = (torch.randn(n, generator=g) if has_bias else None)
        y = int8_matmul_dequant_chunked(xq, xs, wq_, wsc if not scalar else wsc.reshape(()),
                                        bias, dts[out], max_temp_bytes=cap)
        gemm[f"{name}_meta"] = np.array([m, n, k, list(dts).index(out), int(has_bias), int(scalar)], dtype=np.int64)
        gemm[f"{name}_xq"] = xq.numpy()
        gemm[f"{name}_wq"] = wq_.numpy()
        gemm[f"{name}_xscale"] = xs.numpy()
        gemm[f"{name}_wscale"] = wsc.numpy()
        gemm[f"{name}_bias"] = bias.numpy() if has_bias else np.zeros(0, np.float32)
        gemm[f"{name}_y"] = y.numpy() if out == "f32" else _u16(y)
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **gemm)

    # ---- the CPU reference workload (x [256, 5120], W [5120, 5120]) end to end ------------------------
    x = outlier_activations(256, 5120, seed=0, dtype=torch.float32)
    w = gaussian_weight(5120, 5120, seed=0)
    xq, xs = _eager_quantize(x, 256)
    wq, ws = quantize_convrot_weight(w, 256)
    y = int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.float32)
    dense = x @ w.t()
    rel = ((y - dense).norm() / dense.norm()).item()
    np.savez_compressed(
        os.path.join(HERE, "cpu_workload_256x5120.npz"),
        x_sha=np.array(_sha(x)), w_sha=np.array(_sha(w)),
        xscale=xs.numpy(), wscale=ws.numpy(),
        xq_head=xq[:8].numpy(), wq_head=wq[:8].numpy(),
        y_head=y[:8].numpy(), y_norm=np.array(y.norm().item()),
        rel_vs_dense=np.array(rel),
    )
    print("cpu workload rel-Frobenius vs fp32 dense:", rel)
    for f in ("quant.npz", "weight.npz", "gemm.npz", "cpu_workload_256x5120.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
    rowwise(ref_root)
    weight16(ref_root)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if not args or args[0] in ("rowwise", "weight16"):
        sys.exit("usage: make_golden.py <reference root> [--only rowwise|weight16]")
    root = args[0]
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only == "rowwise":
        rowwise(root)
    elif only == "weight16":
        weight16(root)
    else:
        main(root)
