"""Host logic of bench.py that the measurement contract depends on, without a
GPU: the clock/throttle summary (a run whose samples show hw_slowdown or a
thermal slowdown is rejected, so the reasons must be read correctly from both
the NVML and the nvidia-smi fallback forms) and the peak lookup."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_from_nvml_rows(bench):
    c = bench.Clocks(0)
    c.rows = [(1965.0, 1965.0, 300.0, []), (1950.0, 1965.0, 310.0, ["sw_power_cap"]),
              (1965.0, 1965.0, 305.0, [])]
    s = c.summary()
    assert s["sm_mhz"] == 1965.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 3 and s["source"] == "nvml"
    assert s["power_w_median"] == 305.0


def test_clock_summary_from_nvidia_smi_text(bench):
    c = bench.Clocks(0)
    c.out = ("0, 1965, 1965, 700.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
             "0, 1410, 1965, 990.1, 0x0000000000000040, Not Active, Active, Not Active, Not Active\n"
             "garbage line\n")
    s = c.summary()
    assert s["samples"] == 2 and s["source"] == "nvidia-smi"
    assert s["reasons"] == ["hw_thermal_slowdown"]
    assert s["sm_max_mhz"] == 1965.0 and s["sm_mhz"] == pytest.approx((1965 + 1410) / 2)


def test_clock_summary_unsampled(bench):
    s = bench.Clocks(0).summary()
    assert s["reasons"] == ["unsampled"] and s["sm_mhz"] is None


def test_peaks_come_from_the_measured_file_when_present(bench):
    peak, kind = bench._peaks()
    assert peak > 1000.0
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        assert kind == "measured"


def test_parity_check_against_the_cpu_pipeline(bench):
    """The bench's parity field: the CPU pipeline's own outputs pass, a
    planted error in one row (on the CPU side) fails, and the gathered-unit
    count must equal the pipeline's misses."""
    import numpy as np

    from ferry_b200.workload import small

    w = small(num_requests=3, num_layers=1, q_heads=4, kv_heads=2, ctx_tokens=512, top_k=8, steps=4)
    _, _, _, per_tick = bench.cpu_baseline(w, threads=2, ticks=6, keep=6)
    outs = [None if x[3] is None else x[3].reshape(-1, w.num_layers, w.q_heads, 128).copy() for x in per_tick]
    misses = sum(x[2] for x in per_tick)
    assert misses > 0 and any(o is not None for o in outs)
    p = bench.parity_vs_cpu(w, outs, misses, per_tick)
    assert p["status"] == "ok" and p["attn_max_rel_err"] == 0.0 and p["ticks"] == 6
    bad = [None if o is None else o.copy() for o in outs]
    j = next(i for i, o in enumerate(bad) if o is not None)
    bad[j].reshape(-1, 128)[0, 5] += 1.0
    assert bench.parity_vs_cpu(w, bad, misses, per_tick)["status"] == "FAIL"
    assert bench.parity_vs_cpu(w, outs, misses + 1, per_tick)["status"] == "FAIL"
