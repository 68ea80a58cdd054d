"""The bench's host-side arithmetic: roofline figures from stage timings and
pair counts, the measured-traffic table lookup, and the launch accounting."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def test_blend_roofline_is_algorithmic_flops_over_event_time(bench):
    # three blend-backward launches of 0.5 ms, each 1e8 replayed pairs: 70 FLOP per pair
    stages = {"blend_bwd": (3, 1.5, [{"pairs": (100_000_000, 0)}] * 3),
              "blend_fwd": (3, 0.6, [{"pairs": (200_000_000, 50_000_000)}] * 3)}
    roof, table = bench.roofline_from_stages(stages, {"hbm_gbs": 6500.0}, "measured", [1000], fp32_peak=70.0)
    assert roof["kernel"] == "blend_bwd" and roof["bound"] == "fp32" and roof["unit"] == "TFLOP/s"
    assert roof["flops_per_launch"] == 7_000_000_000
    assert roof["ms_per_launch"] == 0.5
    assert roof["achieved"] == pytest.approx(14.0) and roof["frac"] == pytest.approx(0.2)
    assert table["blend_fwd"] == {"calls": 3, "ms_total": 0.6}


def test_ncu_traffic_table_is_per_stage_bytes(bench):
    """Traffic figures come from a table in bench.py (no file is parsed at
    bench time); each entry is a positive byte count for a stage the
    roofline names."""
    for stage, t in bench.NCU_TRAFFIC.items():
        assert stage in ("blend_bwd", "blend_fwd", "preprocess_fwd", "preprocess_bwd", "binning")
        assert isinstance(t, int) and t > 0, stage


def test_launch_accounting(bench):
    # one single-GPU view: the 14 native kernels of the ncu launch list
    assert bench.LAUNCHES_PER_VIEW == 14
    assert bench.DIST_LAUNCHES_PER_BAND == 14 and bench.DIST_LAUNCHES_PER_CAMERA == 4
