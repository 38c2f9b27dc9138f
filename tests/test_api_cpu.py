"""Host-side behaviour of the reference-facing API, on the CPU.

Mirrors the reference's CPU tests (tests/test_comfyui.py) plus the dispatch and
fallback rules of tilegen/kernels/int8_convrot.py and tilegen/comfyui/backend.py.
comfy_kitchen is not installed; a minimal test double (tests/fakes) stands in
for its registry, constraints and eager int8_linear.
"""
from __future__ import annotations

import importlib
import importlib.util
import os
import sys
from pathlib import Path
from unittest.mock import patch

import numpy as np
import pytest
import torch

from tests.conftest import FAKES, GOLDEN, REPO

# ---------------------------------------------------------------- hadamard
def test_hadamard_orthonormal_and_symmetric():
    from tilegen.kernels.hadamard import build_hadamard

    for g in (4, 16, 64, 256):
        h = build_hadamard(g, "cpu", torch.float64)
        assert torch.allclose(h @ h.t(), torch.eye(g, dtype=torch.float64))
        assert torch.equal(h, h.t())
        assert torch.all(h.abs() == 1.0 / g ** 0.5)


def test_hadamard_core_is_the_reference_h4():
    from tilegen.kernels.hadamard import _H4, build_hadamard

    h = build_hadamard(4, "cpu", torch.float32) * 2
    assert h.tolist() == [[float(v) for v in r] for r in _H4]
    assert _H4 == [[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]]


def test_hadamard_rejects_non_powers_of_four():
    from tilegen.kernels.hadamard import build_hadamard

    for g in (2, 8, 128, 100):
        with pytest.raises(ValueError):
            build_hadamard(g, "cpu", torch.float32)


def test_rotate_by_group_preserves_row_norms():
    from tilegen.kernels.hadamard import build_hadamard, rotate_by_group

    x = torch.randn(8, 5120, dtype=torch.float64)
    xr = rotate_by_group(x, build_hadamard(256, "cpu", torch.float64), 256)
    assert torch.allclose(x.norm(dim=-1), xr.norm(dim=-1))
    with pytest.raises(ValueError):
        rotate_by_group(torch.zeros(2, 300), build_hadamard(256, "cpu", torch.float32), 256)


# ---------------------------------------------------------------- quantiser API
def test_eager_quantize_matches_reference_fixtures():
    from tilegen.kernels.int8_convrot import _eager_quantize

    d = np.load(os.path.join(GOLDEN, "quant.npz"))
    for n in ("c", "f"):  # the fp32 fixture cases: identical torch ops on the CPU
        m, k, g, dt = (int(v) for v in d[f"{n}_meta"])
        q, s = _eager_quantize(torch.from_numpy(d[f"{n}_x"]), g)
        assert np.array_equal(q.numpy(), d[f"{n}_q"]) and np.array_equal(s.numpy(), d[f"{n}_scale"])


def test_can_use_fht_on_cpu_is_false_and_quantize_falls_back():
    from tilegen.kernels.int8_convrot import _eager_quantize, can_use_fht, quantize_convrot

    x = torch.randn(4, 5120, dtype=torch.float16)
    assert can_use_fht(x, 256) is False
    q, s = quantize_convrot(x.float(), 256)
    q2, s2 = _eager_quantize(x.float(), 256)
    assert torch.equal(q, q2) and torch.equal(s, s2)


def test_native_entry_points_reject_cpu_tensors():
    from tilegen.kernels.int8_convrot import quantize_convrot_fht

    from tilegen_b200 import ops

    with pytest.raises(ValueError):
        quantize_convrot_fht(torch.zeros(2, 256, dtype=torch.float16))
    with pytest.raises(ValueError):
        ops.rotate_quant(torch.zeros(2, 256, dtype=torch.float16))
    with pytest.raises(ValueError):
        ops.int8_gemm_dequant(torch.zeros(2, 32, dtype=torch.int8), torch.ones(2),
                              torch.zeros(4, 32, dtype=torch.int8), torch.ones(4), None, torch.float16)


def test_cpu_gemm_path_matches_reference_fixtures():
    from tilegen.quant.int8_ops import int8_matmul_dequant_chunked

    d = np.load(os.path.join(GOLDEN, "gemm.npz"))
    dts = [torch.float32, torch.float16, torch.bfloat16]
    for n in "abcd":
        m, nn, k, od, has_bias, scalar = (int(v) for v in d[f"{n}_meta"])
        ws = torch.from_numpy(d[f"{n}_wscale"])
        y = int8_matmul_dequant_chunked(torch.from_numpy(d[f"{n}_xq"]), torch.from_numpy(d[f"{n}_xscale"]),
                                        torch.from_numpy(d[f"{n}_wq"]), ws.reshape(()) if scalar else ws,
                                        torch.from_numpy(d[f"{n}_bias"]) if has_bias else None, dts[od],
                                        max_temp_bytes=4096)
        got = y.contiguous().view(torch.int16).numpy().view(np.uint16) if od else y.numpy()
        assert np.array_equal(got.view(np.uint8), d[f"{n}_y"].view(np.uint8)), n


def test_weight_scale_length_is_checked():
    from tilegen.quant.int8_ops import int8_matmul_dequant_chunked

    with pytest.raises(ValueError):
        int8_matmul_dequant_chunked(torch.zeros(2, 32, dtype=torch.int8), torch.ones(2),
                                    torch.zeros(4, 32, dtype=torch.int8), torch.ones(3), None, torch.float32)


def test_weight_quant_cpu_matches_reference_fixture():
    from tilegen.quant.weight import quantize_convrot_weight

    d = np.load(os.path.join(GOLDEN, "weight.npz"))
    wq, ws = quantize_convrot_weight(torch.from_numpy(d["w"]), 256)
    assert np.array_equal(wq.numpy(), d["wq"]) and np.array_equal(ws.numpy(), d["wscale"])
    with pytest.raises(ValueError):
        quantize_convrot_weight(torch.zeros(4, 300), 256)
    with pytest.raises(ValueError):
        quantize_convrot_weight(torch.zeros(4), 256)


# ---------------------------------------------------------------- ComfyUI surface
def test_drop_in_loader_exports_native_package_nodes():
    from tilegen.comfyui import NODE_CLASS_MAPPINGS

    loader = Path(REPO) / "comfyui" / "__init__.py"
    spec = importlib.util.spec_from_file_location("tilegen_test_loader", loader)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    assert module.NODE_CLASS_MAPPINGS is NODE_CLASS_MAPPINGS
    assert set(NODE_CLASS_MAPPINGS) == {"ConvRotTestTensors", "QuantizeConvRotWeight", "Int8ConvRotLinear",
                                        "TileGenConvRotModelConfig"}


def test_runtime_node_updates_environment_and_passes_model_through():
    from tilegen.comfyui import NODE_CLASS_MAPPINGS

    node = NODE_CLASS_MAPPINGS["TileGenConvRotModelConfig"]()
    model = object()
    with patch.dict(os.environ, {}, clear=True):
        assert node.configure(model, "fht", 5120, "native", 768, False) == (model,)
        assert os.environ["TILEGEN_CONVROT_BACKEND"] == "fht"
        assert os.environ["TILEGEN_FHT_MIN_K"] == "5120"
        assert os.environ["TILEGEN_FHT_IMPL"] == "native"
        assert os.environ["TILEGEN_INT8_TEMP_MB"] == "768"
        assert os.environ["TILEGEN_DIAGNOSTICS"] == "0"


def test_test_tensor_node_and_linear_node_on_cpu():
    from tilegen.comfyui import NODE_CLASS_MAPPINGS

    x, w = NODE_CLASS_MAPPINGS["ConvRotTestTensors"]().create(4, 512, 32, 256, 1, "float16", "cpu")
    assert x.shape == (4, 512) and w.shape == (32, 512) and x.dtype == torch.float16
    wq, ws = NODE_CLASS_MAPPINGS["QuantizeConvRotWeight"]().quantize(w.float(), 256)
    (y,) = NODE_CLASS_MAPPINGS["Int8ConvRotLinear"]().forward(x.float().reshape(2, 2, 512), wq, ws, 256)
    assert y.shape == (2, 2, 32)
    with pytest.raises(ValueError):
        NODE_CLASS_MAPPINGS["ConvRotTestTensors"]().create(4, 500, 32, 256, 1, "float16", "cpu")


def test_env_mode_and_min_k_parsing(monkeypatch):
    from tilegen_b200.comfyui import backend

    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "bogus")
    assert backend._mode() == "auto"
    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", " FHT ")
    assert backend._mode() == "fht"
    monkeypatch.setenv("TILEGEN_FHT_MIN_K", "-5")
    assert backend._fht_min_k() == 0
    monkeypatch.setenv("TILEGEN_FHT_MIN_K", "abc")
    assert backend._fht_min_k() == backend._default_fht_min_k()
    monkeypatch.delenv("TILEGEN_FHT_MIN_K")
    assert backend._fht_min_k() == 8192  # no CUDA device here


def test_install_without_comfy_kitchen_returns_false(monkeypatch):
    from tilegen_b200.comfyui import backend

    monkeypatch.setattr(backend, "_INSTALLED", False)
    monkeypatch.setitem(sys.modules, "comfy_kitchen", None)
    assert backend.install() is False


def test_install_registers_selective_backend_first(fake_kitchen, monkeypatch):
    from tilegen_b200.comfyui import backend

    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "auto")
    assert backend.install() is True
    assert fake_kitchen._priority[0] == "tilegen"
    c = fake_kitchen.get_constraints("tilegen", "int8_linear")
    assert backend._fht_applicable in c.call_rules
    r = backend._fht_applicable({"x": torch.zeros(2, 256, dtype=torch.float16),
                                 "weight": torch.zeros(4, 256, dtype=torch.int8),
                                 "convrot": True, "convrot_groupsize": 256})
    assert not r.success and r.failed_param == "x"
    r = backend._fht_applicable({"x": torch.zeros(2, 256), "convrot": False})
    assert not r.success and r.failed_param == "convrot"
    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "eager")
    r = backend._fht_applicable({"x": torch.zeros(2, 256), "convrot": True})
    assert not r.success and r.failed_param == "__tilegen__"


def test_install_off_is_a_no_op(fake_kitchen, monkeypatch):
    from tilegen_b200.comfyui import backend

    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "off")
    assert backend.install() is False
    assert "tilegen" not in fake_kitchen._priority


def test_cpu_calls_fall_through_to_the_eager_backend(fake_kitchen, monkeypatch):
    from tilegen_b200.comfyui import backend

    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "auto")
    backend.install()
    x = torch.randn(3, 256)
    w = torch.randint(-20, 20, (8, 256), dtype=torch.int8)
    name, _ = fake_kitchen.dispatch("int8_linear", x=x, weight=w, weight_scale=torch.full((8,), 0.01),
                                    convrot=True, convrot_groupsize=256)
    assert name == "eager"


def test_eager_compatibility_accepts_input_act(fake_kitchen, monkeypatch):
    """test_comfyui.py:65-86: eager mode returns exactly comfy_kitchen's eager result."""
    from comfy_kitchen.backends.eager.quantization import int8_linear as eager_int8_linear

    from tilegen_b200.comfyui import backend

    torch.manual_seed(7)
    x = torch.randn(3, 256, dtype=torch.float32)
    weight = torch.randint(-20, 20, (8, 256), dtype=torch.int8)
    weight_scale = torch.full((8,), 0.01, dtype=torch.float32)
    bias = torch.randn(8, dtype=torch.float32)
    kw = dict(bias=bias, out_dtype=torch.float32, convrot=True, convrot_groupsize=256, input_act="gelu_tanh")
    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "eager")
    actual = backend.int8_linear(x, weight, weight_scale, **kw)
    torch.testing.assert_close(actual, eager_int8_linear(x, weight, weight_scale, **kw))


def test_int8_linear_cpu_convrot_path(fake_kitchen, monkeypatch):
    """auto mode on CPU: eager ConvRot quant + the torch GEMM path, shape restored."""
    from tilegen_b200.comfyui import backend

    monkeypatch.setenv("TILEGEN_CONVROT_BACKEND", "auto")
    x = torch.randn(2, 3, 256)
    w = torch.randint(-20, 20, (8, 256), dtype=torch.int8)
    y = backend.int8_linear(x, w, torch.full((8,), 0.01), convrot=True, input_act="gelu_tanh")
    assert y.shape == (2, 3, 8)
    with pytest.raises(ValueError):
        backend.int8_linear(torch.randn(2, 100), torch.zeros(8, 256, dtype=torch.int8), torch.ones(8), convrot=True)


def test_log_decision_dedups(monkeypatch, caplog):
    from tilegen_b200.comfyui import backend

    monkeypatch.setattr(backend, "_LOGGED_DECISIONS", set())
    x = torch.zeros(4, 256)
    with caplog.at_level("WARNING", logger="tilegen.backend"):
        backend._log_decision("KEEP_CUDA", "why", x, None, 256)
        backend._log_decision("KEEP_CUDA", "why", x, None, 256)
    assert sum("KEEP_CUDA" in r.message for r in caplog.records) == 1
    monkeypatch.setenv("TILEGEN_DIAGNOSTICS", "0")
    backend._log_decision("KEEP_CUDA", "other", x, None, 256)
    assert len(backend._LOGGED_DECISIONS) == 1


def test_runtime_shims():
    from tilegen.runtime import bootstrap, ensure_nvrtc, probe, usable_shared_bytes

    assert ensure_nvrtc() is True
    assert bootstrap()["jit"] is False
    assert probe()["sm_count"] >= 1
    assert usable_shared_bytes(headroom=0) >= usable_shared_bytes()


def test_alias_modules_are_shared():
    import tilegen
    import tilegen_b200.quant.int8_ops as mine

    assert tilegen.quant.int8_ops is mine
    assert importlib.import_module("tilegen.comfyui.backend").BACKEND_NAME == "tilegen"


def test_host_linear_argument_checks():
    from tilegen_b200.streaming import int8_linear_host

    x = torch.zeros(4, 256, dtype=torch.float16)
    w = torch.zeros(8, 256, dtype=torch.int8)
    with pytest.raises(ValueError, match="CUDA device"):
        int8_linear_host(x, w, torch.ones(8))
    with pytest.raises(ValueError, match="host memory"):
        int8_linear_host(_FakeCuda(), w, torch.ones(8))


class _FakeCuda:
    is_cuda = True


def test_small_m_routing_boundaries():
    from tilegen_b200.ops import SPLITK_MAX_M, splitk_route

    assert SPLITK_MAX_M == 128
    assert splitk_route(24, 15360, 5120) and not splitk_route(25, 15360, 5120)      # qkv
    assert splitk_route(128, 5120, 5120) and not splitk_route(129, 5120, 5120)      # o_proj
    assert splitk_route(24, 13824, 5120) and not splitk_route(32, 13824, 5120)      # ffn_up
    assert splitk_route(128, 5120, 13824) and not splitk_route(129, 5120, 13824)    # ffn_down
    assert not splitk_route(0, 5120, 5120) and not splitk_route(4096, 5120, 5120)
    from tilegen_b200.ops import GEMV_MAX_M, gemv_route

    assert 0 < GEMV_MAX_M <= 4  # tg_int8_gemv_dequant's limit (TG_GEMV_MAX_M)
    assert gemv_route(1, 15360, 5120) and gemv_route(4, 5120, 5120) and gemv_route(2, 5120, 13824)
    assert not gemv_route(3, 5120, 13824)                                          # ffn_down: split-K
    assert not gemv_route(0, 5120, 5120) and not gemv_route(GEMV_MAX_M + 1, 5120, 5120)


def test_host_linear_chunk_schedule_covers_rows():
    from tilegen_b200.streaming import _chunks

    for m in (1, 7, 255, 256, 1000, 4096, 65520):
        for rows in (1, 3, 64, 512, 1024):
            ch = list(_chunks(m, rows))
            assert ch[0][0] == 0 and ch[-1][1] == m
            assert all(a[1] == b[0] and a[0] < a[1] for a, b in zip(ch, ch[1:] + [(m, m + 1)]))
            sizes = [b - a for a, b in ch]
            assert max(sizes) <= rows and sizes[0] == min(max(1, rows // 4), m)


def test_custom_ops_trace_on_meta_tensors():
    """The torch.library ops have shape functions, so they trace (torch.compile /
    torch.export) without running a kernel: meta tensors in, meta tensors out."""
    from tilegen_b200 import ops  # noqa: F401  (registers the ops)

    x = torch.empty(2, 3, 512, dtype=torch.float16, device="meta")
    vec = torch.empty(2, 1, 512, dtype=torch.float16, device="meta")
    q, s = torch.ops.tilegen.quantize_ln_mod(x, 256, vec, vec, 1e-6)
    assert q.shape == (6, 512) and q.dtype == torch.int8 and s.shape == (6,) and s.dtype == torch.float32
    q, s = torch.ops.tilegen.quantize_act(x.view(6, 512), 256, "gelu_tanh")
    assert q.shape == (6, 512) and s.shape == (6,)
    y = torch.ops.tilegen.int8_gemm_dequant(q, s, torch.empty(8, 512, dtype=torch.int8, device="meta"),
                                            torch.empty(8, device="meta"), None, torch.bfloat16)
    assert y.shape == (6, 8) and y.dtype == torch.bfloat16
