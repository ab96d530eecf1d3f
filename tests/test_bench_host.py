"""Host-side pieces of bench.py that decide what a bench line reports (no GPU):
the clock record taken during the timed region (which throttle reasons make a
run invalid) and the committed DRAM-traffic figures the roofline quotes."""
from __future__ import annotations

import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _sampler(bench, rows):
    s = bench.ClockSampler.__new__(bench.ClockSampler)  # no nvidia-smi process
    s.rows = rows
    s.proc = None
    return s


def _row(sm, mx=1965, power=600.0, hw="Not Active", hw_th="Not Active", sw_th="Not Active",
         pcap="Not Active"):
    # clocks.sm, clocks.max.sm, power.draw, event_reasons.active, then the four named reasons
    return [str(sm), str(mx), str(power), "0x0", hw, hw_th, sw_th, pcap]


def test_clock_summary_inside_timed_window(bench):
    rows = [(0.5, _row(1000)), (1.0, _row(1900)), (1.2, _row(1950)), (1.4, _row(1965)),
            (3.0, _row(800, hw="Active"))]
    c = _sampler(bench, rows).summary(1.0, 2.0)
    assert c["window"] == "timed" and c["samples"] == 3
    assert c["sm_mhz"] == 1950.0 and c["sm_max_mhz"] == 1965.0
    # a slowdown outside the timed region does not count against the run
    assert c["reasons"] == []


def test_clock_summary_reports_throttle_reasons(bench):
    rows = [(1.0, _row(1400, pcap="Active")), (1.1, _row(1350, sw_th="Active")),
            (1.2, _row(1300, hw="Active", hw_th="Active"))]
    c = _sampler(bench, rows).summary(0.0, 2.0)
    assert c["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap",
                            "sw_thermal_slowdown"]


def test_clock_summary_short_region_falls_back_to_all_samples(bench):
    rows = [(0.1, _row(1965)), (0.3, _row(1965, pcap="Active")), (5.0, _row(1965))]
    c = _sampler(bench, rows).summary(1.0, 1.01)
    assert c["window"] == "ramp+warmup+timed" and c["samples"] == 3
    assert c["reasons"] == ["sw_power_cap"]


def test_clock_summary_without_nvidia_smi(bench):
    c = _sampler(bench, []).summary(0.0, 1.0)
    assert c["samples"] == 0 and c["sm_mhz"] is None and "unavailable" in c["note"]


@pytest.mark.parametrize("name", ["decode_kernel_config3_traffic", "decode_kernel_config5_traffic",
                                  "q4_gemv_kernel_config6_traffic"])
def test_profiled_traffic_files(bench, name):
    v = bench.profiled_traffic(name)
    assert v is not None and v > 0


def test_profiled_traffic_missing_file(bench):
    assert bench.profiled_traffic("no_such_profile") is None


def test_reference_arm_line(tmp_path):
    """bench.py --impl reference (the CPU reference arm the driver runs beside the GPU arm)
    prints one JSON line with the contract's keys, on CPU alone; under torchrun only rank 0
    prints and the other ranks exit 0."""
    import json
    import subprocess
    import sys
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    env["RANK"] = "1"
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=600, cwd=REPO)
    assert r.returncode == 0 and not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_split_is_balanced_by_rows(bench, world):
    """Config 3 at N GPUs: every sequence on exactly one rank, and the ranks' row
    totals (which set the step time, the slowest rank's) within one sequence of each
    other; contiguous blocks of the seed-3 lengths are not."""
    L = bench.config3_lengths()
    sets = bench.strong_assignment(L, world)
    assert sorted(i for s in sets for i in s) == list(range(len(L)))
    sums = [int(L[s].sum()) for s in sets]
    assert max(sums) - min(sums) <= 512, sums  # the shortest sequence bounds the gap
    for r in range(world):
        assert list(bench.rank_lengths(r, world, "strong")) == [int(L[i]) for i in sets[r]]
