"""CPU-only checks of the native boundary: the C-ABI library loads, exports
every entry point include/blitzgs_b200.h declares, and rejects bad arguments
with a status and a message (no GPU needed: validation precedes any CUDA
call)."""
import ctypes
import os
import re

import pytest

from blitzgs_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "blitzgs_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(blitz_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_entry_points():
    fns = header_functions()
    for n in ("blitz_preprocess_forward", "blitz_preprocess_backward", "blitz_render_count",
              "blitz_render_forward", "blitz_render_backward", "blitz_loss_forward", "blitz_loss_backward",
              "blitz_get_local2j_ids_bool", "blitz_render_scratch_bytes", "blitz_last_error", "blitz_version"):
        assert n in fns


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for n in header_functions():
        assert hasattr(lib, n), f"{n} declared in include/blitzgs_b200.h but not exported"
    assert set(header_functions()) <= set(_lib.SIGNATURES), "ctypes signatures missing for some entry points"


def header_prototypes():
    """{name: (return type, [parameter types])} parsed from the header."""
    src = open(os.path.join(ROOT, "include", "blitzgs_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for ret, name, params in re.findall(r"\b((?:const\s+)?[a-z0-9_]+\s*\*?)\s*(blitz_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        protos[name] = (ret.strip(), [p.rsplit(" ", 1)[0].replace(" *", "*").strip() if "*" not in p.rsplit(" ", 1)[-1]
                                      else p.rsplit(" ", 1)[0].strip() + "*" for p in ps])
    return protos


def _ctype_of(c):
    c = c.replace("const ", "").strip()
    if c.endswith("*"):
        return ctypes.c_char_p if c == "char*" else ctypes.c_void_p
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float, "size_t": ctypes.c_size_t,
            "int32_t": ctypes.c_int32, "uint32_t": ctypes.c_uint32}[c]


def test_ctypes_signatures_match_the_header():
    """Every binding in blitzgs_b200._lib has the header's parameter count and
    types, so a changed prototype cannot silently shift arguments."""
    protos = header_prototypes()
    assert set(protos) == set(header_functions())
    for name, (ret, params) in protos.items():
        sig_ret, sig_args = _lib.SIGNATURES[name]
        assert len(sig_args) == len(params), f"{name}: {len(sig_args)} ctypes args, header has {len(params)}"
        for k, (a, c) in enumerate(zip(sig_args, params)):
            assert ctypes.sizeof(a) == ctypes.sizeof(_ctype_of(c)) and \
                (a is ctypes.c_void_p) == c.endswith("*"), f"{name} arg {k}: {a} vs {c}"
        assert ctypes.sizeof(sig_ret) == ctypes.sizeof(_ctype_of(ret)), f"{name} return: {sig_ret} vs {ret}"


def test_version_string():
    assert b"sm_100a" in _lib.load().blitz_version()


def test_argument_validation_without_gpu():
    lib = _lib.load()
    rc = lib.blitz_render_count(-1, 10, 10, None, None, None, None, None, None)
    assert rc == 10001
    assert b"bad arguments" in lib.blitz_last_error()
    rc = lib.blitz_loss_forward(3, 4, 4, None, None, None, None, None, None, None)
    assert rc == 10001
    with pytest.raises(RuntimeError, match="blitz_render_count"):
        _lib.call("blitz_render_count", -1, 10, 10, None, None, None, None, None, None)


def test_step_and_exchange_entries_validate_arguments_without_gpu():
    """The loss combination, totals readback, zero fill, exchange unpack /
    gradient pack and the strip-list arguments of the blend entries reject
    bad arguments with BLITZ_EINVAL and a message before any CUDA call."""
    lib = _lib.load()
    EINVAL = 10001

    def rejects(name, *args, msg=None):
        rc = getattr(lib, name)(*args)
        assert rc == EINVAL, (name, rc)
        text = lib.blitz_last_error().decode()
        assert name in text and (msg is None or msg in text), text

    # loss combination: the sums pointer and a positive N3 are required
    rejects("blitz_loss_combine", None, None, 0.8, 0.2, 100.0, 10.0, 1, None)
    rejects("blitz_loss_combine", 8, None, 0.8, 0.2, 0.0, 10.0, 8, None)
    rejects("blitz_loss_combine_backward", None, None, None, None, 0.8, 0.2, 100.0, 10.0, 8, None)
    # totals readback: vis_count and host_vis go together, and so do status and host_status
    rejects("blitz_read_totals", None, None, None, 8, None, None, None)
    rejects("blitz_read_totals", 8, 8, None, 8, None, None, None)
    rejects("blitz_read_totals", 8, None, 8, 8, None, None, None)
    # zero fill: negative count, or a non-empty list without arrays
    rejects("blitz_zero_fill_async", -1, None, None, None)
    rejects("blitz_zero_fill_async", 2, None, None, None)
    # exchange unpack / gradient pack: at most 32 runs, non-negative runs, pointers when rows exist
    n = 33
    starts = (ctypes.c_int64 * n)(*range(n))
    counts = (ctypes.c_int64 * n)(*([1] * n))
    rejects("blitz_exchange_unpack", n, starts, counts, None, None, None, None, None, None, None, None,
            msg="segments")
    neg = (ctypes.c_int64 * 1)(-5)
    one = (ctypes.c_int64 * 1)(1)
    rejects("blitz_exchange_unpack", 1, neg, one, None, None, None, None, None, None, None, None, msg="segments")
    rejects("blitz_exchange_unpack", 1, one, one, None, None, None, None, None, None, None, None,
            msg="null pointer")
    rejects("blitz_grad_records_pack", n, starts, counts, None, None, None, None, None, msg="segments")
    rejects("blitz_grad_records_pack", 1, one, one, None, None, None, None, None, msg="null pointer")
    # ordered pack: needs its scratch; the batched forms check sizes and host arrays
    offs = (ctypes.c_int64 * 2)(0, 0)
    rejects("blitz_exchange_pack", 10, 2, 16, 16, offs, 16, 16, 0, None, 0, None, msg="null pointer")
    rejects("blitz_exchange_pack", 10, 33, 16, 16, offs, 16, 16, 0, 16, 0, None, msg="bad sizes")
    rejects("blitz_exchange_pack_batch", 2, 0, None, 8, None, None, None, None, None, None, None, 0, None,
            msg="bad sizes")
    rejects("blitz_exchange_pack_batch", 2, 2, None, 8, None, None, None, None, None, None, None, 0, None,
            msg="null pointer")
    tan = (ctypes.c_float * 4)(0.5, 0.5, 0.5, 0.5)
    params = [None] * 5 + [0, None, 0, 1.0]  # xyz, _scaling, _rotation, _opacity, dc, dc_stride, rest, stride, mod
    cams = [None, None, None, tan, 8, 8]      # views, projections, centres, tan(fov), H, W
    rejects("blitz_preprocess_forward_raw_batch", 2, 100, 3, 15, *params, *cams, 50, *([None] * 7), 0, None, None,
            None, None, 0, None, msg="bad sizes")
    rejects("blitz_preprocess_forward_raw_batch", 2, 100, 3, 15, *params, *cams, 100, *([None] * 7), 0, None, None,
            None, None, 0, None, msg="null pointer")
    rows0 = (ctypes.c_int64 * 2)(0, 0)
    rejects("blitz_preprocess_backward_raw_batch", 2, 100, 3, 15, None, None, None, None, 0, 100, *params[:4],
            *params[4:], *cams, None, rows0, None, None, None, None, None, 0, None, 0, None, msg="bad sizes")
    # empty runs are a no-op, not an error
    zero = (ctypes.c_int64 * 1)(0)
    assert lib.blitz_exchange_unpack(1, one, zero, None, None, None, None, None, None, None, None) == 0
    assert lib.blitz_grad_records_pack(0, None, None, None, None, None, None, None) == 0
    # strip lists: all three pointers or none
    rejects("blitz_render_blend", 10, 16, 16, 8, 16, 8, 8, None, 8, 8, 8, 8, 8, 8, 8, 8, 8, 8, None, None, None,
            msg="go together")
    rejects("blitz_render_backward", 10, 16, 16, 8, 8, 8, 8, 8, 16, 8, 8, None, 8, None, 8, None, 8, 16, None,
            msg="go together")


def test_scratch_size_query_is_host_only():
    lib = _lib.load()
    a = lib.blitz_render_scratch_bytes(1000, 100, 500, 64, 64)
    b = lib.blitz_render_scratch_bytes(1000, 200, 5000, 64, 64)
    assert 0 < a < b


def test_ops_refuse_cpu_tensors():
    import torch
    from blitzgs_b200 import ops, scene as S
    sc = S.tiny(seed=8, P=16, H=32, W=32)
    rs = S.raster_settings(sc.cameras[0])
    shs = torch.cat((sc.features_dc, sc.features_rest), 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.preprocess_forward(sc.xyz, torch.exp(sc.scaling), sc.rotation, sc.opacity.reshape(-1),
                               ops.sh_layout(shs=shs), rs)


def test_compat_import_names():
    import importlib
    import sys
    compat = os.path.join(ROOT, "blitzgs_b200", "compat")
    sys.path.insert(0, compat)
    try:
        f = importlib.import_module("diff_gaussian_rasterization_f")
        r = importlib.import_module("diff_gaussian_rasterization_r")
        for m in (f, r):
            assert hasattr(m, "GaussianRasterizationSettings") and hasattr(m, "GaussianRasterizer")
            for op in ("preprocess_gaussians", "preprocess_gaussians_backward", "render_gaussians",
                       "render_gaussians_backward", "get_local2j_ids_bool"):
                assert hasattr(m._C, op)
        assert list(f.GaussianRasterizationSettings._fields) == [
            "image_height", "image_width", "tanfovx", "tanfovy", "bg", "scale_modifier", "viewmatrix",
            "projmatrix", "sh_degree", "campos", "prefiltered", "debug"]
    finally:
        sys.path.remove(compat)
        for n in ("diff_gaussian_rasterization_f", "diff_gaussian_rasterization_r"):
            sys.modules.pop(n, None)


# The reference's public wrapper API that its renderer glue, model and trainer
# call (diff_gaussian_rasterization_f/_r __init__.py): method and function
# parameter names in order.  A drop-in must accept the same names.
_REF_API = {
    ("f", "GaussianRasterizer", "__init__"): ["self", "raster_settings"],
    ("f", "GaussianRasterizer", "markVisible"): ["self", "positions"],
    ("f", "GaussianRasterizer", "preprocess_gaussians"): ["self", "means3D", "scales", "rotations", "shs",
                                                          "opacities", "cuda_args"],
    ("f", "GaussianRasterizer", "render_gaussians"): ["self", "means2D", "means2D_abs", "conic_opacity", "rgb",
                                                      "all_map", "depths", "radii", "compute_locally",
                                                      "extended_compute_locally", "cuda_args"],
    ("f", "GaussianRasterizer", "forward"): ["self", "means3D", "means2D", "opacities", "culling", "dc", "shs",
                                             "colors_precomp", "scales", "rotations", "cov3D_precomp",
                                             "flag_max_count"],
    ("f", "GaussianRasterizer", "render_simp"): ["self", "means3D", "means2D", "opacities", "culling", "dc", "shs",
                                                 "colors_precomp", "scales", "rotations", "cov3D_precomp"],
    ("f", "GaussianRasterizer", "render_depth"): ["self", "means3D", "means2D", "opacities", "culling", "dc", "shs",
                                                  "colors_precomp", "scales", "rotations", "cov3D_precomp"],
    ("f", "SparseGaussianAdam", "__init__"): ["self", "params", "lr", "eps"],
    ("f", None, "preprocess_gaussians"): ["means3D", "scales", "rotations", "sh", "opacities", "raster_settings",
                                          "cuda_args"],
    ("f", None, "render_gaussians"): ["means2D", "means2D_abs", "conic_opacity", "rgb", "all_map", "depths", "radii",
                                      "compute_locally", "extended_compute_locally", "raster_settings", "cuda_args"],
    ("f", None, "rasterize_gaussians"): ["means3D", "means2D", "dc", "sh", "colors_precomp", "opacities", "scales",
                                         "rotations", "cov3Ds_precomp", "flag_max_count", "culling",
                                         "raster_settings"],
    ("r", "GaussianRasterizer", "preprocess_gaussians"): ["self", "means3D", "scales", "rotations", "shs",
                                                          "opacities", "cuda_args"],
    ("r", "GaussianRasterizer", "render_gaussians"): ["self", "means2D", "means2D_abs", "conic_opacity", "rgb",
                                                      "all_map", "depths", "radii", "compute_locally",
                                                      "extended_compute_locally", "cuda_args"],
}


def test_compat_signatures_match_the_reference_api():
    import importlib
    import inspect
    import sys
    compat = os.path.join(ROOT, "blitzgs_b200", "compat")
    sys.path.insert(0, compat)
    try:
        mods = {k: importlib.import_module(f"diff_gaussian_rasterization_{k}") for k in ("f", "r")}
        for (m, cls, name), params in _REF_API.items():
            obj = getattr(mods[m], cls) if cls else mods[m]
            got = list(inspect.signature(getattr(obj, name)).parameters)
            assert got[:len(params)] == params, (m, cls, name, got)
            # anything added after the reference's parameters must be optional
            extra = list(inspect.signature(getattr(obj, name)).parameters.values())[len(params):]
            assert all(p.default is not inspect.Parameter.empty for p in extra), (m, cls, name, extra)
        # SparseGaussianAdam.step(visibility, N) as the trainer calls it (train_internal.py:517-545)
        step = list(inspect.signature(mods["f"].SparseGaussianAdam.step).parameters)
        assert step[:3] == ["self", "visibility", "N"]
        for op in ("get_local2j_ids_bool", "get_local2j_ids_bool_adjust_mode6", "adamUpdate"):
            assert callable(getattr(mods["f"]._C, op))
    finally:
        sys.path.remove(compat)
        for n in ("diff_gaussian_rasterization_f", "diff_gaussian_rasterization_r"):
            sys.modules.pop(n, None)
