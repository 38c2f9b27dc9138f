"""Parity of the few-row INT8 GEMV (tg_int8_gemv_dequant) on the GPU.

For one to four activation rows each warp streams four weight rows over one
part of K and sums exact int32 dp4a products; the K parts of a row group meet
in shared memory.  Integer sums are exact and order-independent, so the output
must be bit-identical to the oracle (the reference's torch sequence,
tilegen/quant/int8_ops.py:22-70, restated), to the tiled and split-K kernels,
for every M from 1 to 4, every K-part count (1, 2, 4, 8), ragged N and K, all
output dtypes, bias and scale variants, with and without the L2 prefetch.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests._util import DT_NAME, out_bits
from tilegen_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed, scalar_ws=False, bias_dtype=None):
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


def _run(case, out_dtype, dev, kernel):
    """int8_gemm_dequant on one kernel: "gemv", "splitk" or "tiled"."""
    xq, xs, wq, ws, bias = case
    route, gemv = ops.splitk_route, ops.gemv_route
    ops.gemv_route = lambda m, n, k: kernel == "gemv"
    ops.splitk_route = lambda m, n, k: kernel == "splitk"
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
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bias_dtype", [None, torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("scalar_ws", [False, True])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_against_oracle(cuda, out_dtype, bias_dtype, scalar_ws, m):
    n, k = 640, 1152
    case = _case(m, n, k, seed=m, scalar_ws=scalar_ws, bias_dtype=bias_dtype)
    y = _run(case, out_dtype, cuda, "gemv")
    xq, xs, wq, ws, bias = case
    ref = oracle.int8_gemm_dequant(xq.numpy(), xs.numpy(), wq.numpy(), ws.numpy(),
                                   None if bias is None else bias.float().numpy(), DT_NAME[out_dtype])
    got = out_bits(y)
    if got.dtype == np.float32:
        got, ref = got.view(np.uint32), ref.view(np.uint32)
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} outputs differ, first at {bad[:3].tolist()}"


# (n, k, K parts): each split of K the launch chooses.
PARTS = [(15360, 5120, 1), (5120, 5120, 2), (1536, 2048, 4), (640, 13824, 8)]


@pytest.mark.parametrize("n,k,parts", PARTS)
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_k_parts_bit_exact_vs_tiled_and_splitk(cuda, m, n, k, parts):
    assert _lib.gemv_config(n, k)[0] == parts
    case = _case(m, n, k, seed=n + k + m, bias_dtype=torch.bfloat16)
    a = _run(case, torch.float16, cuda, "gemv")
    assert np.array_equal(_bits(a), _bits(_run(case, torch.float16, cuda, "tiled")))
    assert np.array_equal(_bits(a), _bits(_run(case, torch.float16, cuda, "splitk")))


@pytest.mark.parametrize("n,k", [(8, 16), (8, 48), (136, 144), (1000, 4112), (4000, 1040), (13824, 5120),
                                 (5120, 13824)])
def test_ragged_and_dit_shapes(cuda, n, k):
    for m in (1, 4):
        case = _case(m, n, k, seed=7 * n + k + m)
        y = _run(case, torch.bfloat16, cuda, "gemv")
        xq, xs, wq, ws, _ = case
        # int8 products summed in float64 are exact (|sum| < 2^53); .float()
        # then rounds once, as float(int32) does.
        acc = (xq.to(cuda).double() @ wq.to(cuda).double().t()).float()
        ref = acc * xs.to(cuda)[:, None] * ws.to(cuda)[None, :]
        assert np.array_equal(_bits(y), _bits(ref.to(torch.bfloat16)))


def test_weight_above_prefetch_limit(cuda):
    """A 257 MiB weight streams without the up-front L2 prefetch (limit 256 MiB)."""
    n, k = 65536, 4112
    g = torch.Generator(device=cuda).manual_seed(5)
    wq = torch.randint(-128, 128, (n, k), generator=g, dtype=torch.int8, device=cuda)
    ws = torch.rand(n, generator=g, device=cuda) * 1e-3
    xq = torch.randint(-128, 128, (2, k), generator=g, dtype=torch.int8, device=cuda)
    xs = torch.rand(2, generator=g, device=cuda) * 1e-2
    case = (xq, xs, wq, ws, None)
    a = _run(case, torch.float16, cuda, "gemv")
    b = _run(case, torch.float16, cuda, "tiled")
    assert torch.equal(a, b)


def test_routed_linear_in_graph_matches_eager(cuda):
    """One row through the public path (quantiser, then the GEMV as its
    programmatic dependent), captured in a CUDA graph and replayed."""
    from tilegen_b200.quant.int8_ops import int8_matmul_dequant_chunked
    from tilegen_b200.synthetic import dit_activations, gaussian_weight

    assert ops.gemv_route(1, 5120, 5120)
    x = dit_activations("o_proj", 1, seed=3, dtype=torch.float16, device=cuda)
    wq, ws = ops.rotate_quant(gaussian_weight(5120, 5120, seed=4, dtype=torch.float16, device=cuda), 256)

    def linear():
        xq, xs = ops.rotate_quant(x, 256)
        return int8_matmul_dequant_chunked(xq, xs, wq, ws, None, torch.float16)

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
    xq, xs = ops.rotate_quant(x, 256)
    assert torch.equal(eager, _run((xq, xs, wq, ws, None), torch.float16, cuda, "tiled"))
