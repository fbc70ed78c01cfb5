"""bench.py's reference arm prints one JSON line with every key the bench
contract names.

Runs on the CPU: `--impl reference` times the oracle port of the path, here with
the sample shrunk to a fraction of a second (two warm-up blocks, a 0.2 s
attention budget) so that the test stays quick.
"""
from __future__ import annotations

import json
import sys

import pytest


def test_reference_arm_line(monkeypatch, capsys):
    import bench
    real = bench.cpu_sample
    monkeypatch.setattr(bench, "cpu_sample",
                        lambda args, budget_s=12.0, warm_blocks=12: real(args, 0.2, 2))
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--steps", "1",
                                      "--warmup", "0"])
    from oracle import pkv_oracle as O
    try:
        bench.main()
    finally:
        O.set_threads(1)   # the sample raises the oracle's pack threads; the tests use one
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["scaling"] == "weak" and "workload" in d["config"]
    cb = d["cpu_baseline"]
    for key in ("value", "unit", "cores", "kind", "sample"):
        assert key in cb, key
    assert cb["kind"] == "port" and cb["value"] == pytest.approx(d["value"])
    e2e = d["e2e"]
    assert e2e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
