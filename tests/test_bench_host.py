"""bench.py's host-side pieces on CPU: the algorithmic byte counts quoted for
each leg, the leg summary lines and the clock sampler's fallback."""
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
