"""bench.py's host-side pieces on CPU: the algorithmic byte counts quoted for
each leg, the leg summary lines, the clock sampler's fallback and the per-leg
clock summary over the timed windows."""
from __future__ import annotations

import json

import bench


def test_step_bytes_match_the_quoted_algorithmic_bytes():
    # K+V pages + q/out + tables
    assert bench.step_bytes(32, 4096) == 2_148_040_832
    # configs[2] INT4: codes + fp16 scales + q/out + tables
    assert bench.step_bytes(16, 16384, "int4") == 1_141_178_432


def test_leg_summary_lines_are_plain_text_with_north_star_last(capsys):
    extra = {"int4_decode": {"value": 1.0, "unit": "GB/s", "frac_of_hbm_peak": 0.8, "ms_per_step": 0.2},
             "prefill": {"value": 2.0, "unit": "TFLOP/s", "frac_of_tensor_peak": 0.6, "ms_per_step": 4.0},
             "evict_tokens": {"value": 3.0, "unit": "GB/s", "ms_per_call": 0.05},
             "something_new": {"value": 4.0, "unit": "GB/s"}}
    bench.print_leg_summary(extra, 1)
    lines = capsys.readouterr().out.strip().splitlines()
    assert [ln.split()[1] for ln in lines] == ["evict_tokens", "prefill", "int4_decode", "something_new"]
    assert all(ln.startswith("leg ") for ln in lines)
    for ln in lines:  # none of them parses as the JSON result line
        try:
            json.loads(ln)
            raise AssertionError(ln)
        except json.JSONDecodeError:
            pass
    assert "frac 0.800" in lines[2]


def test_clock_sampler_without_a_gpu_reports_no_samples():
    with bench.Clocks(0) as c:
        pass
    s = c.summary()
    assert s["samples"] == 0 or s["source"] in ("nvml", "nvidia-smi")


def test_leg_clock_summary_counts_only_samples_inside_the_timed_windows(capsys):
    c = bench.Clocks(0)
    c.mx = 1965.0
    c.samples = [(1.0, 1965.0, "0000"), (2.0, 1700.0, "0001"), (2.5, 1710.0, "0001"), (4.0, 1200.0, "1000")]
    s = c.windows_summary([(1.5, 3.0)])
    assert s == {"sm_mhz": 1705.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 2}
    s = c.windows_summary([(0.5, 1.5), (3.5, 4.5)])
    assert s["samples"] == 2 and s["reasons"] == ["hw_slowdown"]
    assert c.windows_summary([])["sm_mhz"] is None
    bench.print_leg_summary({"prefill": {"value": 2.0, "unit": "TFLOP/s", "ms_per_step": 4.0,
                                         "clocks": {"sm_mhz": 1705.0, "reasons": ["sw_power_cap"]}}}, 1)
    assert capsys.readouterr().out.strip().endswith("sm 1705 MHz sw_power_cap")


def test_timed_loops_record_their_wall_windows():
    class _S:  # a stream stand-in (no GPU here); the events and synchronize are faked below
        pass

    n0 = len(bench.TIMED_WINDOWS)
    calls = []
    ev = type("E", (), {"record": lambda self, s: None, "elapsed_time": lambda self, o: 2.0})
    fake = type("T", (), {"cuda": type("C", (), {"Event": staticmethod(lambda enable_timing: ev()),
                                                  "synchronize": staticmethod(lambda: None)})})
    ms = bench.time_loop(fake, lambda: calls.append(1), 4, 3, lambda: None, _S())
    assert ms == 0.5 and len(calls) == 7
    assert bench.time_each(fake, lambda: calls.append(1), 3, _S()) == 2.0
    w = bench.TIMED_WINDOWS[n0:]
    assert len(w) == 2 and all(a <= b for a, b in w)
