"""The bench's reference arm on the CPU: the JSON line the driver reads.

The arm times the reference's own CPU path of the linear (its eager
rotate+quant and its chunked torch._int_mm GEMM, from the package installed in
baseline/_ref, else this repository's torch restatement of the same functions),
one whole 4096-row linear per step; the line is checked against the bench
contract.
"""
from __future__ import annotations

import argparse
import json
import os

import bench


def _args(**kw):
    base = dict(steps=1, warmup=0, gpus=1, impl="reference", no_cpu=False, quick=False)
    base.update(kw)
    return argparse.Namespace(**base)


def test_reference_arm_prints_the_contract_line(monkeypatch, capsys):
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("RANK", "0")
    bench.run_reference(_args())
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "us" and line["higher_is_better"] is False
    assert line["steps"] == 1 and line["warmup"] == 0 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] in ("reference", "port") and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"] and "4096-row steps" in line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the tilegen arm prints the same dict (bench._config) for the same N
    assert line["config"] == bench._config(1)
    assert line["metric"] == bench.METRIC


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    bench.run_reference(_args())
    assert capsys.readouterr().out == ""


def test_reference_cpu_path_is_the_installed_reference_when_present():
    kind, quant, gemm, wquant, source = bench._reference_cpu()
    installed = os.path.isfile(os.path.join(bench.HERE, "baseline", "_ref", "tilegen", "__init__.py"))
    assert kind == ("reference" if installed else "port")
    if installed:
        # loaded from baseline/_ref under its own name, not this repository's alias package
        assert os.path.realpath(quant.__code__.co_filename).startswith(
            os.path.realpath(os.path.join(bench.HERE, "baseline", "_ref")))
        assert quant.__module__ == "tilegen_ref.kernels.int8_convrot"


def test_clock_sampler_keeps_samples_inside_the_region(tmp_path):
    """NVML samples are stamped with wall-clock time; only those inside the
    with-block count, and the reason bits map to the throttle names."""
    c = bench.ClockSampler(0)
    c.kind, c.path = "nvml", str(tmp_path / "clk.txt")
    c.t0, c.t1 = 100.0, 100.010
    (tmp_path / "clk.txt").write_text("max 1965\n99.9990 1965 0\n100.0010 1965 4\n100.0050 1950 4\n"
                                      "100.0200 1300 8\n")
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1957.5 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    c = bench.ClockSampler(0)
    c.kind, c.path = "nvml", str(tmp_path / "clk2.txt")
    c.t0, c.t1 = 100.0, 100.001
    (tmp_path / "clk2.txt").write_text("max 1965\n99.9990 1965 0\n100.0020 1965 64\n")
    s = c.summary()  # nothing inside: the samples just before and after
    assert s["samples"] == 0 and s["reasons"] == ["hw_thermal_slowdown"]
