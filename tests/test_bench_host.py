"""bench.py's host-side pieces, on CPU: the velocity FLOP count against a hand count, and
the oracle velocity baseline end to end on a small model (the same code the bench's
`nar_velocity.cpu_baseline` runs at the 3B shape)."""
import importlib.util
import os

import pytest

from yue2_rs_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_velocity_flops_hand_count(bench):
    c = synth.config_c2()  # 28 layers, H 3072, 24/8 heads of 128, I 8192
    lin, att = bench.velocity_flops(c, 10, 100)
    per_layer = 3072 * (3072 + 2 * 1024 + 3072 + 3 * 8192)
    assert lin == 2.0 * 10 * 28 * per_layer
    assert att == 4.0 * 10 * 100 * 24 * 128 * 28


def test_cpu_velocity_baseline_runs(bench):
    r = bench.cpu_velocity_baseline(synth.config_c1(), length=200, frames=500, sample_frames=6, layers=2)
    assert r["unit"] == "TFLOP/s" and r["kind"] == "port" and r["value"] > 0
    assert r["full_call_seconds"] > 0 and r["cores"] >= 1
    assert "200-position prefix" in r["sample"]


def test_cpu_baseline_uses_every_host_core_under_torchrun(bench, monkeypatch):
    """torchrun sets OMP_NUM_THREADS=1 for each rank; the CPU baseline still runs on all the
    cores the process may use, so its rate is the same at every GPU count."""
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    r = bench.cpu_baseline(synth.config_c1(), min_tokens=3)
    assert r["cores"] == bench.host_cores()
    assert r["kind"] == "port" and r["value"] > 0
    assert "3 config-1 decode tokens" in r["sample"]
