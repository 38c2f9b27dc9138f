"""The C ABI's calls inside a captured CUDA graph.

The entry points only enqueue work on the caller's stream (no allocation, no
host synchronisation), so a whole int8_convrot linear -- the quantiser, then the
GEMM as its programmatic dependent -- can be captured once and replayed on new
inputs.  Replays must give exactly what eager calls give, for the tiled GEMM
(M = 4096) and for the small-M split-K GEMM, whose self-clearing scratch is
reused by every replay.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests._util import out_bits
from tilegen_b200 import _lib, ops
from tilegen_b200.synthetic import gaussian_weight

pytestmark = pytest.mark.gpu


def _linear(x, wq, ws):
    q, s = ops.rotate_quant(x, 256)
    return ops.int8_gemm_dequant(q, s, wq, ws, None, torch.float16)


@pytest.mark.parametrize("m,k,n", [(4096, 5120, 5120), (8, 13824, 5120)])
def test_linear_replayed_from_a_cuda_graph(cuda, m, k, n):
    w = gaussian_weight(n, k, seed=2, dtype=torch.float16, device=cuda)
    wq, ws = ops.rotate_quant(w, 256)
    g = torch.Generator(device=cuda).manual_seed(m)
    x = torch.empty(m, k, dtype=torch.float16, device=cuda)
    stream = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(stream):
        # Warm up on the capture stream (the split-K scratch is per stream).
        x.copy_(torch.randn(m, k, generator=g, device=cuda))
        _linear(x, wq, ws)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        y = _linear(x, wq, ws)
    for i in range(3):
        x.copy_(torch.randn(m, k, generator=g, device=cuda) * (1 + i))
        graph.replay()
        torch.cuda.synchronize()
        ref = _linear(x, wq, ws)
        torch.cuda.synchronize()
        assert np.array_equal(out_bits(y), out_bits(ref)), f"replay {i}"
    del graph
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("group,act", [(256, "gelu_tanh"), (1, "gelu"), (1, None)])
def test_quantize_act_replayed_from_a_cuda_graph(cuda, group, act):
    m, k = 1000, 13824
    g = torch.Generator(device=cuda).manual_seed(group)
    x = torch.empty(m, k, dtype=torch.bfloat16, device=cuda)
    stream = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(stream):
        x.copy_(torch.randn(m, k, generator=g, device=cuda))
        ops.quantize_act(x, group, act)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        q, s = ops.quantize_act(x, group, act)
    for i in range(3):
        x.copy_(torch.randn(m, k, generator=g, device=cuda) * (1 + i))
        graph.replay()
        torch.cuda.synchronize()
        rq, rs = ops.quantize_act(x, group, act)
        torch.cuda.synchronize()
        assert torch.equal(q, rq) and torch.equal(s.view(torch.int32), rs.view(torch.int32)), f"replay {i}"
    del graph
    assert _lib.device_status(0) == 0
