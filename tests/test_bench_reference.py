"""The reference arm of bench.py (`--impl reference`): bounded in wall time
whatever the step count, one JSON line with the contract's keys.  The oracle
timing itself is replaced by a stub here; bench.py's own run times it."""
import argparse
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _args(steps, warmup=3):
    return argparse.Namespace(config="c2", steps=steps, warmup=warmup, gpus=1,
                              ref_budget=8.0, precision="tf32", bh=0, kv_split=False)


def test_large_step_counts_stop_at_the_wall_time_cap(monkeypatch, capsys):
    calls = []

    def fake_baseline(cfg, budget_s=12.0):
        calls.append(budget_s)
        time.sleep(0.01)
        return {"value": 0.25, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                "sample": "stub", "tier": "stub"}

    monkeypatch.setattr(bench, "cpu_baseline", fake_baseline)
    monkeypatch.setattr(bench, "REF_WALL_S", 0.2)
    t0 = time.perf_counter()
    bench.run_reference(_args(steps=6000))
    assert time.perf_counter() - t0 < 5.0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["steps"] == 6000
    assert 3 <= line["cpu_baseline"]["steps_timed"] < 6000
    assert line["value"] == 0.25 and line["e2e"]["value"] == 0.25
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # every step samples at least ~1 s of the workload
    assert min(calls) >= 1.0


def test_other_ranks_print_nothing(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setattr(bench, "cpu_baseline",
                        lambda *a, **k: (_ for _ in ()).throw(AssertionError("ran")))
    bench.run_reference(_args(steps=10))
    assert capsys.readouterr().out == ""
