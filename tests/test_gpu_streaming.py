"""The host-buffer linear (tilegen_b200.streaming.int8_linear_host) on the GPU.

Its row chunks run the same kernels as the device path on overlapping streams,
so the output must be bit-identical to rotate+quant then the GEMM on the whole
tensor, for ragged row counts, both input dtypes, bias and caller-given output.
"""
from __future__ import annotations

import pytest
import torch

from tilegen_b200 import ops
from tilegen_b200.streaming import int8_linear_host
from tilegen_b200.synthetic import gaussian_weight, outlier_activations

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,chunk", [(1, 512), (511, 512), (1300, 512), (4096, 512), (700, 64)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_host_linear_equals_device_path(cuda, m, chunk, dtype):
    k, n = 5120, 1536
    x = outlier_activations(m, k, seed=m, dtype=dtype)
    w = gaussian_weight(n, k, seed=2, dtype=dtype, device=cuda)
    wq, ws = ops.rotate_quant(w, 256)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(3)).to(cuda)
    y = int8_linear_host(x.pin_memory(), wq, ws, bias, dtype, rows_per_chunk=chunk)
    torch.cuda.current_stream().synchronize()
    ref = ops.int8_gemm_dequant(*ops.rotate_quant(x.to(cuda), 256), wq, ws, bias, dtype).cpu()
    assert not y.is_cuda and y.shape == (m, n)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_host_linear_into_caller_output_on_a_side_stream(cuda):
    m, k, n = 2000, 13824, 5120
    x = outlier_activations(m, k, seed=9, dtype=torch.float16).pin_memory()
    w = gaussian_weight(n, k, seed=4, dtype=torch.float16, device=cuda)
    wq, ws = ops.rotate_quant(w, 256)
    out = torch.full((m, n), 7.0, dtype=torch.float32).pin_memory()
    side = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(side):
        r = int8_linear_host(x, wq, ws, None, torch.float32, out=out)
    side.synchronize()
    assert r is out
    ref = ops.int8_gemm_dequant(*ops.rotate_quant(x.to(cuda), 256), wq, ws, None, torch.float32).cpu()
    assert torch.equal(out.view(torch.int32), ref.view(torch.int32))


@pytest.mark.parametrize("m,k,n,chunk", [(4096, 5120, 1536, 1024), (600, 13824, 640, 128)])
def test_host_linear_graph_replays(cuda, m, k, n, chunk):
    """graph=True: the first call runs and captures, later calls replay on whatever the
    same host buffers hold.  The second case sends its small chunks to the split-K
    kernel, whose scratch the graph keeps."""
    w = gaussian_weight(n, k, seed=5, dtype=torch.bfloat16, device=cuda)
    wq, ws = ops.rotate_quant(w, 256)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(6)).to(cuda).half()
    x_host = torch.empty((m, k), dtype=torch.bfloat16).pin_memory()
    out = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    for i in range(4):
        x = outlier_activations(m, k, seed=10 + i, dtype=torch.bfloat16)
        x_host.copy_(x)
        r = int8_linear_host(x_host, wq, ws, bias, torch.bfloat16, out=out, rows_per_chunk=chunk, graph=True)
        torch.cuda.current_stream().synchronize()
        ref = ops.int8_gemm_dequant(*ops.rotate_quant(x.to(cuda), 256), wq, ws, bias, torch.bfloat16).cpu()
        assert r is out
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {i}"


def test_two_host_linear_graphs_replayed_concurrently(cuda):
    """Two captured graphs whose chunks run the split-K kernel, replayed at the same
    time on two streams: each graph owns its split-K scratch, so both stay exact."""
    from tilegen_b200 import streaming

    m, k, n, chunk = 600, 13824, 640, 128
    w = gaussian_weight(n, k, seed=7, dtype=torch.bfloat16, device=cuda)
    wq, ws = ops.rotate_quant(w, 256)
    xs = [outlier_activations(m, k, seed=20 + j, dtype=torch.bfloat16) for j in range(2)]
    hosts = [x.pin_memory() for x in xs]
    outs = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    refs = [ops.int8_gemm_dequant(*ops.rotate_quant(x.to(cuda), 256), wq, ws, None, torch.bfloat16).cpu() for x in xs]
    streams = [torch.cuda.Stream(device=cuda) for _ in range(2)]
    for j in range(2):  # capture both graphs
        with torch.cuda.stream(streams[j]):
            int8_linear_host(hosts[j], wq, ws, None, torch.bfloat16, out=outs[j], rows_per_chunk=chunk, graph=True)
        streams[j].synchronize()
    held = [e[1] for e in list(streaming._GRAPHS.values())[-2:]]  # the two graphs just captured
    scratch_ptrs = {t.data_ptr() for h in held for t in h if t.dtype == torch.uint8}
    assert len(scratch_ptrs) == 2  # one split-K scratch per graph
    for _ in range(3):
        for o in outs:
            o.zero_()
        for j in range(2):
            with torch.cuda.stream(streams[j]):
                int8_linear_host(hosts[j], wq, ws, None, torch.bfloat16, out=outs[j], rows_per_chunk=chunk, graph=True)
        torch.cuda.synchronize()
        for j in range(2):
            assert torch.equal(outs[j].view(torch.int16), refs[j].view(torch.int16)), j
