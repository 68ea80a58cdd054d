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


def test_stage_rooflines_bound_and_fraction(bench):
    """Each stage's lower time bound is max(FLOP / FP32 peak, bytes / copy
    bandwidth) of its modelled work; frac = bound / event-timed time."""
    px = 3 * 864 * 1152
    stages = {
        # 2 launches of 1e8 replayed pairs in 1.0 ms: 1.4e10 FLOP / 1e-3 s = 14 TFLOP/s of 70
        "blend_bwd": (2, 1.0, [{"pairs": (100_000_000,)}] * 2),
        # the view's own totals (R, V), not the capacities in R / n_vis
        "binning": (1, 0.1, [{"P": 1_000_000, "R": 999_999, "n_vis": 999_999, "totals": (500_000, 100_000)}]),
        "loss_fwd": (1, 0.05, [{"pixels": px, "gt_bytes": 1}]),
        "loss_bwd": (1, 0.05, [{"pixels": px, "gt_bytes": 1}]),
        "preprocess_bwd": (1, 0.05, [{"P": 8_000_000, "n_list": 250_000}]),
        # the batched form reports no list length: no model
        "preprocess_fwd": (1, 0.2, [{"P": 16_000_000}]),
    }
    t = bench.stage_rooflines(stages, {"hbm_gbs": 6500.0}, "measured", 70.0)
    b = t["blend_bwd"]
    assert b["bound"] == "fp32" and b["unit"] == "TFLOP/s"
    assert b["achieved"] == pytest.approx(14.0) and b["frac"] == pytest.approx(0.2)
    assert b["flop_per_launch"] == 7_000_000_000
    g = t["binning"]
    byts = 4 * 1_000_000 + 4 * 100_000 + 20 * 500_000
    assert g["bound"] == "hbm" and g["bytes_per_launch"] == byts
    assert g["frac"] == pytest.approx(byts / 6500e9 / 1e-4, abs=1e-4)  # rounded to 4 places
    lf = t["loss_fwd"]
    t_f, t_b = 258 * px / 70e12, 17 * px / 6500e9
    assert lf["bound"] == ("fp32" if t_f >= t_b else "hbm")
    assert lf["frac"] == pytest.approx(max(t_f, t_b) / 5e-5, abs=1e-4)
    assert lf["flop_per_launch"] == 258 * px and lf["bytes_per_launch"] == 17 * px
    assert t["loss_bwd"]["bytes_per_launch"] == 21 * px
    assert t["preprocess_bwd"]["bytes_per_launch"] == 508 * 250_000
    assert t["preprocess_fwd"]["model"] is None
    assert t["peaks"]["hbm_gbs"] == 6500.0 and t["peaks"]["fp32_tflops"] == 70.0
    # without an FP32 peak the FLOP-only stages report no fraction
    t2 = bench.stage_rooflines({"blend_fwd": (1, 0.2, [{"pairs": (10, 5)}])}, {"hbm_gbs": 6500.0}, "measured", None)
    assert t2["blend_fwd"]["frac"] is None and t2["blend_fwd"]["flop_per_launch"] == 165


def test_stage_rooflines_without_model_metadata(bench):
    """A launch without the metadata a model needs (the full rasterizer's
    statistics blend has no pair counters) gets no fraction rather than an
    error; a binning launch sized by its exact totals needs no "totals"."""
    stages = {"blend_fwd": (2, 0.4, [{"pairs": (10, 5)}, {"P": 7}]),
              "binning": (1, 0.1, [{"P": 100, "R": 50, "n_vis": 10}]),
              "adam": (1, 0.1, [{}])}
    t = bench.stage_rooflines(stages, {"hbm_gbs": 6500.0}, "measured", 70.0)
    assert t["blend_fwd"]["model"] is None and t["adam"]["model"] is None
    assert t["binning"]["bytes_per_launch"] == 4 * 100 + 4 * 10 + 20 * 50


def test_bench_functions_name_only_defined_globals():
    """Every global name a function of bench.py reads is defined at module
    level or is a builtin: the reference arm and the GPU-only paths cannot
    run here, so an undefined name there would only surface on a GPU box."""
    import ast
    import builtins
    import symtable
    path = os.path.join(ROOT, "bench.py")
    src = open(path).read()
    defined = set(dir(builtins)) | {"__file__", "__name__"}
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, (ast.Import, ast.ImportFrom)):
            defined |= {(a.asname or a.name).split(".")[0] for a in node.names}
    top = symtable.symtable(src, path, "exec")
    defined |= {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported()}
    missing = []

    def walk(t):
        for s in t.get_symbols():
            if s.is_global() and s.is_referenced() and s.get_name() not in defined:
                missing.append((t.get_name(), t.get_lineno(), s.get_name()))
        for c in t.get_children():
            walk(c)

    for c in top.get_children():
        walk(c)
    assert not missing, missing


def test_clock_sampler_summary(bench):
    """Clock samples count only inside the marked timed regions; a region
    shorter than the sampling period takes its nearest sample; throttle
    reason bits are named."""
    cs = bench.ClockSampler(0)
    ms = 1_000_000  # ns per ms
    # (t_ns, sm_mhz, max_mhz, reason bits): 1965 inside region 1, a capped sample outside
    cs.samples = [(0 * ms, 900.0, 1965.0, 0x8), (100 * ms, 1965.0, 1965.0, 0), (150 * ms, 1965.0, 1965.0, 0),
                  (200 * ms, 1950.0, 1965.0, 0x4), (400 * ms, 1800.0, 1965.0, 0)]
    cs.windows = [[90 * ms, 210 * ms], [395 * ms, 396 * ms]]
    out = cs.stop()
    assert out["samples"] == 4  # three inside region 1, region 2 takes its nearest (400 ms)
    assert out["sm_mhz"] == 1965.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]  # the hw_slowdown sample at 0 ms lies outside both regions
    empty = bench.ClockSampler(0)
    empty.windows = [[0, 1]]
    assert empty.stop() is None
