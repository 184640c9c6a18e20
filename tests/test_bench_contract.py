"""The benchmark's host-side contract, on CPU: the reference arm's JSON line
(the reference's algorithm, i.e. the pinned numpy oracle, timed on the host
cores) and the bounded CPU baselines carry the keys the round-end driver
reads.  The GPU arm needs a B200 and is exercised there."""

from __future__ import annotations

import argparse
import json

import pytest

import bench


@pytest.mark.parametrize("name", ["rmsnorm", "rope", "mla"])
def test_cpu_baseline_is_a_bounded_oracle_sample(name):
    wl = bench.WORKLOADS[name](None, 0, 1, dict(bench.PEAKS_FALLBACK), "fallback")
    r = wl.cpu_baseline(0.05)
    assert r["value"] > 0 and r["unit"] == wl.unit and r["kind"] == "port"
    assert isinstance(r["cores"], int) and r["cores"] >= 1 and r["sample"]
    cfg = wl.config()
    assert "workload" in cfg and "model" not in cfg


def test_reference_arm_prints_one_contract_line(monkeypatch, capsys):
    cls = bench.WORKLOADS["rmsnorm"]
    orig = cls.cpu_baseline
    monkeypatch.setattr(cls, "cpu_baseline", lambda self, seconds: orig(self, 0.05))
    args = argparse.Namespace(workload="rmsnorm", steps=2, warmup=1)
    assert bench.reference_arm(args, 1, dict(bench.PEAKS_FALLBACK), "fallback") == 0
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == cls.metric and d["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
    assert set(bench.WORKLOADS) == {"rmsnorm", "rope", "moe", "moe_ep", "ffn", "mla"}
