"""The JSON line of ``bench.py --impl reference`` (the driver's CPU reference
arm): one line with the contract's keys and the same workload ``config`` as
the B200 arm, checked without a GPU.  The oracle's step timing is replaced by
a fixed time so the check takes no minutes of CPU work."""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules["bench_under_test"] = module
    spec.loader.exec_module(module)
    return module


def test_reference_arm_prints_one_contract_line(monkeypatch, capsys):
    bench = _bench()
    depths = []

    def fake_step_time(depth, threads):
        depths.append(depth)
        return 0.25 * depth / 32, {}

    monkeypatch.setattr(bench, "cpu_step_time", fake_step_time)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    bench.run_reference(argparse.Namespace(gpus=1, steps=3, warmup=2, impl="reference"), rank=0)
    lines = [line for line in capsys.readouterr().out.splitlines() if line.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["impl"] == "reference" and rec["metric"] == bench.METRIC and rec["unit"] == bench.UNIT
    assert rec["higher_is_better"] is True and (rec["steps"], rec["warmup"]) == (3, 2)
    assert rec["config"] == bench.workload_config(1)  # the same workload the B200 arm reports
    assert abs(rec["value"] - 4.0) < 1e-9  # 0.25 s per full-depth step, whatever depth was sampled
    assert rec["e2e"] == {"value": rec["value"], "unit": rec["unit"], "h2d_bytes_per_step": 0,
                          "d2h_bytes_per_step": 0}
    assert rec["cpu_baseline"]["value"] == rec["value"] and rec["cpu_baseline"]["kind"] == "port"
    assert len(depths) == 1 + 2 + 3  # the depth probe, the warm-up steps, the timed steps


def test_reference_arm_is_silent_on_other_ranks(monkeypatch, capsys):
    bench = _bench()
    monkeypatch.setattr(bench, "cpu_step_time", lambda depth, threads: (_ for _ in ()).throw(AssertionError))
    bench.run_reference(argparse.Namespace(gpus=2, steps=3, warmup=2, impl="reference"), rank=1)
    assert capsys.readouterr().out == ""
