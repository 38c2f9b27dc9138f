"""The bench's reference arm on the CPU: the JSON line the driver reads.

The arm times the C oracle (the reference algorithm on the host cores) on a
bounded row sample; here the sample is cut to 8 rows so the test is quick, and
the line is checked against the bench contract.
"""
from __future__ import annotations

import argparse
import json

import bench


def _args(**kw):
    base = dict(steps=2, warmup=1, gpus=1, impl="reference", no_cpu=False, quick=False)
    base.update(kw)
    return argparse.Namespace(**base)


def test_reference_arm_prints_the_contract_line(monkeypatch, capsys):
    monkeypatch.setattr(bench.CpuLinear, "rows_for", lambda self, seconds: 8)
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("RANK", "0")
    bench.run_reference(_args())
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "us" and line["higher_is_better"] is False
    assert line["steps"] == 2 and line["warmup"] == 1 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"] and "8 of 4096 rows" in line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["config"]["M"] == 4096 and line["config"]["K"] == 5120 and line["config"]["N"] == 15360


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    bench.run_reference(_args())
    assert capsys.readouterr().out == ""
