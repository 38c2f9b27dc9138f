"""The C-ABI library loads and exports what include/tilegen_b200.h declares.

No kernel runs here (no GPU): only entry points whose argument checks return
before any device work are called.
"""
from __future__ import annotations

import ctypes

import pytest

from tilegen_b200 import _lib


def test_library_exports_every_declared_function():
    names = _lib.declared_functions()
    assert set(names) >= {"tg_version", "tg_status_string", "tg_rotate_quant", "tg_rotate_quant_max_k",
                          "tg_int8_gemm_dequant", "tg_device_status"}
    L = _lib.lib()
    for n in names:
        assert hasattr(L, n), n


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.tg_version() >= 1
    for code in range(6):
        assert L.tg_status_string(code)
    assert L.tg_status_string(0) == b"ok"
    assert L.tg_rotate_quant_max_k() % 256 == 0


def test_argument_checks_return_before_device_work():
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    # unsupported group / K / dtype
    assert L.tg_rotate_quant(p, _lib.TG_DT_F16, 4, 5120, 128, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_rotate_quant(p, _lib.TG_DT_F16, 4, 5000, 256, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_rotate_quant(p, _lib.TG_DT_F32, 4, 5120, 256, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_rotate_quant(p, _lib.TG_DT_F16, -1, 5120, 256, p, p, None) == _lib.TG_ERR_INVALID_ARG
    # M == 0 is a no-op
    assert L.tg_rotate_quant(None, _lib.TG_DT_F16, 0, 5120, 256, None, None, None) == _lib.TG_OK
    # null pointers with M > 0
    assert L.tg_rotate_quant(None, _lib.TG_DT_F16, 2, 5120, 256, None, None, None) == _lib.TG_ERR_INVALID_ARG
    # GEMM: K % 16, N alignment, wscale length, dtype
    assert L.tg_int8_gemm_dequant(p, p, p, p, 1, None, 0, 4, 64, 24, 1, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemm_dequant(p, p, p, p, 1, None, 0, 4, 12, 32, 1, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemm_dequant(p, p, p, p, 3, None, 0, 4, 64, 32, 1, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemm_dequant(p, p, p, p, 1, None, 0, 4, 64, 32, 7, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemm_dequant(None, None, None, None, 1, None, 0, 0, 64, 32, 1, None, None) == _lib.TG_OK
    assert L.tg_set_gemm_config(100, -1) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_set_gemm_config(256, 2) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_set_gemm_config(0, -1) == _lib.TG_OK


def test_check_maps_status_to_exceptions():
    with pytest.raises(ValueError):
        _lib.check("tg_rotate_quant", _lib.TG_ERR_UNSUPPORTED)
    with pytest.raises(_lib.TileGenError):
        _lib.check("tg_rotate_quant", _lib.TG_ERR_CUDA)
    _lib.check("x", _lib.TG_OK)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="missing"):
        _lib.lib()


def test_small_m_entry_points_check_before_device_work():
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    L.tg_int8_gemm_dequant_splitk_noalloc.argtypes = [ctypes.c_void_p] * 4 + [
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    assert L.tg_int8_gemm_dequant_splitk_max_m() == 128
    # workspace: 128-column tile counters (256-byte rounded), then M x N int32
    assert L.tg_int8_gemm_dequant_splitk_workspace(1, 128) == 256 + 512
    assert L.tg_int8_gemm_dequant_splitk_workspace(64, 15360) == 512 + 64 * 15360 * 4
    assert L.tg_int8_gemm_dequant_splitk_workspace(-1, 128) == 0
    big = 1 << 30
    # M above the limit, workspace missing, too small or misaligned
    assert L.tg_int8_gemm_dequant_splitk(p, p, p, p, 1, None, 0, 129, 128, 64, 1, p, p, big, None) == \
        _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemm_dequant_splitk(p, p, p, p, 1, None, 0, 8, 128, 64, 1, p, None, big, None) == \
        _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemm_dequant_splitk(p, p, p, p, 1, None, 0, 8, 128, 64, 1, p, p, 16, None) == \
        _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemm_dequant_splitk(p, p, p, p, 1, None, 0, 8, 128, 64, 1, p, ctypes.c_void_p(272), big,
                                         None) == _lib.TG_ERR_MISALIGNED
    assert L.tg_int8_gemm_dequant_splitk(None, None, None, None, 1, None, 0, 0, 128, 64, 1, None, None, 0,
                                         None) == _lib.TG_OK
    # the no-allocation variant: its array's limits
    for m, n in ((65, 128), (64, 32768), (8, 65536 + 128)):
        assert L.tg_int8_gemm_dequant_splitk_noalloc(p, p, p, p, 1, None, 0, m, n, 64, 1, p, None) == \
            _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemm_dequant_splitk_noalloc(None, None, None, None, 1, None, 0, 0, 128, 64, 1, None,
                                                 None) == _lib.TG_OK


def test_gemv_entry_points_check_before_device_work():
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    assert {"tg_int8_gemv_dequant", "tg_int8_gemv_dequant_config"} <= set(_lib.declared_functions())
    # M above TG_GEMV_MAX_M (4), null operands, misaligned weight, K not a multiple of 16
    assert L.tg_int8_gemv_dequant(p, p, p, p, 1, None, 0, 5, 128, 64, 1, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemv_dequant(None, p, p, p, 1, None, 0, 1, 128, 64, 1, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemv_dequant(p, p, ctypes.c_void_p(264), p, 1, None, 0, 1, 128, 64, 1, p, None) == \
        _lib.TG_ERR_MISALIGNED
    assert L.tg_int8_gemv_dequant(p, p, p, p, 1, None, 0, 1, 128, 72, 1, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_int8_gemv_dequant(p, p, p, p, 3, None, 0, 1, 128, 64, 1, p, None) == _lib.TG_ERR_INVALID_ARG
    # M == 0 is a no-op
    assert L.tg_int8_gemv_dequant(None, None, None, None, 1, None, 0, 0, 128, 64, 1, None, None) == _lib.TG_OK
    parts, ctas = ctypes.c_int(0), ctypes.c_int(0)
    assert L.tg_int8_gemv_dequant_config(0, 64, ctypes.byref(parts), ctypes.byref(ctas)) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemv_dequant_config(64, 8, ctypes.byref(parts), ctypes.byref(ctas)) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemv_dequant_config(64, 64, None, None) == _lib.TG_ERR_INVALID_ARG


def test_ln_mod_entry_checks_before_device_work():
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    f16 = _lib.TG_DT_F16
    assert "tg_quantize_ln_mod" in _lib.declared_functions()
    # eps negative or NaN, mod_rows < 1, fp32 input, the row-wise group, K not a multiple of 256
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 256, -1.0, p, p, 1, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 256, float("nan"), p, p, 1, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 256, 1e-6, p, p, 0, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_ln_mod(p, _lib.TG_DT_F32, 4, 512, 256, 1e-6, p, p, 1, p, p, None) == \
        _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 1, 1e-6, p, p, 1, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_ln_mod(p, f16, 4, 320, 64, 1e-6, p, p, 1, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    # missing or misaligned modulation vectors; M == 0 is a no-op
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 256, 1e-6, None, p, 1, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_ln_mod(p, f16, 4, 512, 256, 1e-6, p, ctypes.c_void_p(258), 1, p, p, None) == \
        _lib.TG_ERR_MISALIGNED
    assert L.tg_quantize_ln_mod(None, f16, 0, 512, 256, 1e-6, None, None, 1, None, None, None) == _lib.TG_OK


def test_quantize_act_checks_before_device_work():
    L = _lib.lib()
    p = ctypes.c_void_p(16)
    assert "tg_quantize_act" in _lib.declared_functions()
    # unknown activation, unsupported group, K rules (256 rotated, 64 row-wise)
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 5120, 256, 3, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 5120, 256, -1, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 5120, 2, 0, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 5120, 128, 1, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 320, 256, 1, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 96, 1, 0, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_act(p, _lib.TG_DT_F16, 4, 32832, 1, 0, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_quantize_act(p, _lib.TG_DT_F32, 4, 320, 1, 0, p, p, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_act(p, _lib.TG_DT_BF16, -1, 320, 1, 2, p, p, None) == _lib.TG_ERR_INVALID_ARG
    # M == 0 is a no-op; null pointers with M > 0 are rejected; misaligned x
    assert L.tg_quantize_act(None, _lib.TG_DT_F16, 0, 320, 1, 1, None, None, None) == _lib.TG_OK
    assert L.tg_quantize_act(None, _lib.TG_DT_F16, 2, 320, 1, 1, None, None, None) == _lib.TG_ERR_INVALID_ARG
    assert L.tg_quantize_act(ctypes.c_void_p(8), _lib.TG_DT_F16, 2, 320, 1, 1, p, p, None) == \
        _lib.TG_ERR_MISALIGNED
    # tg_rotate_quant keeps rejecting group 1 (the row-wise branch is tg_quantize_act's)
    assert L.tg_rotate_quant(p, _lib.TG_DT_F16, 4, 320, 1, p, p, None) == _lib.TG_ERR_UNSUPPORTED
    assert L.tg_rotate_quant(p, _lib.TG_DT_F16, -1, 320, 1, p, p, None) == _lib.TG_ERR_INVALID_ARG


def test_splitk_config_checks_arguments():
    L = _lib.lib()
    sl, cl = ctypes.c_int(0), ctypes.c_int(0)
    assert "tg_int8_gemm_dequant_splitk_config" in _lib.declared_functions()
    for args in ((0, 64, 64, 1, 0), (129, 64, 64, 1, 0), (4, 0, 64, 1, 0), (4, 64, 0, 1, 0), (4, 64, 64, 9, 0)):
        assert L.tg_int8_gemm_dequant_splitk_config(*args, ctypes.byref(sl), ctypes.byref(cl)) == \
            _lib.TG_ERR_INVALID_ARG
    assert L.tg_int8_gemm_dequant_splitk_config(4, 64, 64, 1, 0, None, None) == _lib.TG_ERR_INVALID_ARG


def test_sm_budget_roundtrip():
    L = _lib.lib()
    assert L.tg_sm_budget() == 0
    assert L.tg_set_sm_budget(-1) == _lib.TG_ERR_INVALID_ARG
    from tilegen_b200 import ops

    with ops.sm_budget(100):
        assert L.tg_sm_budget() == 100
        with ops.sm_budget(64):
            assert L.tg_sm_budget() == 64
        assert L.tg_sm_budget() == 100
    assert L.tg_sm_budget() == 0
