"""The benchmark's host-side contract, on CPU: the reference arm's JSON line
and the bounded CPU baselines carry the keys the round-end driver reads.
The CPU baselines time the reference's own modules (installed in
baseline/_ref) when they are there, else the numpy restatement of the
reference's algorithm (oracle/); both forms are checked.  The GPU arm needs
a B200 and is exercised there."""

from __future__ import annotations

import argparse
import json

import pytest

import bench

HAVE_REF = bench.reference_modules() is not None


@pytest.mark.parametrize("name", ["rmsnorm", "rope", "mla"])
def test_port_baseline_is_a_bounded_oracle_sample(name):
    wl = bench.WORKLOADS[name](None, 0, 1, dict(bench.PEAKS_FALLBACK), "fallback")
    r = wl.port_baseline(0.05)
    assert r["value"] > 0 and r["unit"] == wl.unit and r["kind"] == "port"
    assert isinstance(r["cores"], int) and r["cores"] >= 1 and r["sample"]
    cfg = wl.config()
    assert "workload" in cfg and "model" not in cfg


@pytest.mark.skipif(not HAVE_REF, reason="the reference is not installed in baseline/_ref")
@pytest.mark.parametrize("name", ["rmsnorm", "rope", "mla"])
def test_cpu_baseline_times_the_reference_modules(name):
    wl = bench.WORKLOADS[name](None, 0, 1, dict(bench.PEAKS_FALLBACK), "fallback")
    r = wl.cpu_baseline(0.05)
    assert r["value"] > 0 and r["unit"] == wl.unit and r["kind"] == "reference"
    assert isinstance(r["cores"], int) and r["cores"] >= 1 and "baseline/_ref" in r["sample"]


def test_reference_arm_prints_one_contract_line(capsys):
    cls = bench.WORKLOADS["rmsnorm"]
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
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] == ("reference" if HAVE_REF else "port")
    assert set(bench.WORKLOADS) == {"rmsnorm", "rope", "moe", "moe_ep", "ffn", "mla"}
    assert next(iter(bench.WORKLOADS)) == "moe_ep"  # the headline; the extras follow


def test_compact_extra_keeps_the_numbers():
    res = {"metric": "m", "value": 1.23456789, "unit": "GB/s", "ms_per_step": 0.5,
           "roofline": {"bound": "hbm", "frac": 0.812345, "achieved": 5000.1234, "peak": 6500.0, "unit": "GB/s",
                        "kernel_ms": 0.08, "traffic": 3.7e8, "peak_source": "measured", "kernel": "long text"},
           "cpu_baseline": {"value": 2.5, "kind": "reference", "cores": 16, "sample": "long text"},
           "e2e": {"value": 60.0, "unit": "GB/s"}, "clocks": {"sm_mhz": 1965.0, "reasons": []}, "gpu_launches": 40}
    c = bench.compact(res)
    assert c["value"] == 1.235 and c["roofline"]["frac"] == 0.8123 and "kernel" not in c["roofline"]
    assert c["cpu_baseline"] == {"value": 2.5, "kind": "reference", "cores": 16}
    assert len(json.dumps(c)) < 600
