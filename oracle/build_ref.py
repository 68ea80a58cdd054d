"""Build recipe for the reference rasterizer used as the GPU-side parity checker.

TEST INFRASTRUCTURE ONLY.  The product never imports anything built here.

This script compiles the two native modules of the reference BlitzGS
rasterizer (``diff_gaussian_rasterization_f._C`` and
``diff_gaussian_rasterization_r._C``) straight from their source files in the
read-only reference checkout, with nvcc for Blackwell, and lays them out as an
importable package tree under ``oracle/_ref/`` (git-ignored; it travels to the
GPU box with the working tree).  The reference's own ``setup.py`` is not run:
this recipe lists the sources and flags itself (the same source lists and
include paths as submodule/diff-gaussian-rasterization_{f,r}/setup.py).

The reference's Python autograd wrappers
(submodule/diff-gaussian-rasterization_{f,r}/diff_gaussian_rasterization_*/__init__.py)
and its loss helpers (utils/loss_utils.py) are installed beside the built
modules, as ``pip install --target`` would, so the reference arm of
``bench.py`` and the golden-vector generator can run the stock code path.
The renderer glue (gaussian_renderer/*.py and the utils modules it imports)
goes to ``oracle/_ref/refsrc`` for the drop-in test, which runs it on top of
either rasterizer.

Usage:  python oracle/build_ref.py [--ref /path/to/reference] [--force]
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

# (package, sources relative to the submodule dir) -- mirrors the reference's
# source lists in diff-gaussian-rasterization_{f,r}/setup.py.
MODULES = {
    "diff_gaussian_rasterization_r": (
        "submodule/diff-gaussian-rasterization_r",
        ["cuda_rasterizer/rasterizer_impl.cu", "cuda_rasterizer/forward.cu",
         "cuda_rasterizer/backward.cu", "cuda_rasterizer/timers.cu",
         "rasterize_points.cu", "ext.cpp"],
    ),
    "diff_gaussian_rasterization_f": (
        "submodule/diff-gaussian-rasterization_f",
        ["cuda_rasterizer/rasterizer_impl.cu", "cuda_rasterizer/forward.cu",
         "cuda_rasterizer/backward.cu", "cuda_rasterizer/adam.cu",
         "rasterize_points.cu", "conv.cu", "ext.cpp"],
    ),
}

# reference Python modules the renderer-glue test imports (installed under
# oracle/_ref/refsrc; scene.*, pytorch3d, plyfile and simple_knn are stubbed
# by the test itself)
GLUE = {
    "gaussian_renderer": ["__init__.py", "workload_division.py", "loss_distribution.py"],
    "utils": ["general_utils.py", "loss_utils.py", "sh_utils.py", "graphics_utils.py", "system_utils.py"],
}

_CHILD = r"""
import sys, torch.utils.cpp_extension as ce
name, build_dir, glm, *srcs = sys.argv[1:]
ce.load(name="_C", sources=srcs, build_directory=build_dir,
        extra_include_paths=[glm],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "-std=c++17", "-gencode", "arch=compute_100,code=sm_100"],
        is_python_module=False, verbose=False)
"""


def built(pkg):
    return os.path.exists(os.path.join(OUT, pkg, "_C.so"))


def build(ref, force=False):
    if not os.path.isdir(ref):
        print(f"[build_ref] reference checkout {ref} absent; skipping")
        return False
    os.makedirs(OUT, exist_ok=True)
    ok = True
    procs = []
    for pkg, (sub, srcs) in MODULES.items():
        src_dir = os.path.join(ref, sub)
        pkg_out = os.path.join(OUT, pkg)
        os.makedirs(pkg_out, exist_ok=True)
        shutil.copyfile(os.path.join(src_dir, pkg, "__init__.py"),
                        os.path.join(pkg_out, "__init__.py"))
        if built(pkg) and not force:
            continue
        bdir = os.path.join(OUT, "build_" + pkg)
        os.makedirs(bdir, exist_ok=True)
        env = dict(os.environ, MAX_JOBS=os.environ.get("MAX_JOBS", "4"),
                   TORCH_CUDA_ARCH_LIST="10.0")
        cmd = [sys.executable, "-c", _CHILD, pkg, bdir,
               os.path.join(src_dir, "third_party", "glm")] + \
              [os.path.join(src_dir, s) for s in srcs]
        procs.append((pkg, bdir, subprocess.Popen(cmd, env=env)))
    for pkg, bdir, p in procs:
        rc = p.wait()
        so = os.path.join(bdir, "_C.so")
        if rc != 0 or not os.path.exists(so):
            print(f"[build_ref] {pkg}: build failed (rc={rc})")
            ok = False
            continue
        shutil.copyfile(so, os.path.join(OUT, pkg, "_C.so"))
    # stock loss helpers (plain PyTorch) used by the reference training loop
    lu = os.path.join(ref, "utils", "loss_utils.py")
    if os.path.exists(lu):
        shutil.copyfile(lu, os.path.join(OUT, "ref_loss_utils.py"))
    # the reference's renderer glue and the utils modules it imports, as
    # installed packages, so a GPU test can run the stock
    # distributed_preprocess3dgs_and_all2all_final -> render_final ->
    # batched_loss_computation path on either rasterizer
    glue = os.path.join(OUT, "refsrc")
    for pkg, files in GLUE.items():
        dst = os.path.join(glue, pkg)
        os.makedirs(dst, exist_ok=True)
        for f in files:
            src = os.path.join(ref, pkg, f)
            if os.path.exists(src):
                shutil.copyfile(src, os.path.join(dst, f))
    open(os.path.join(glue, "utils", "__init__.py"), "a").close()
    return ok


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BLITZ_REFERENCE_DIR", "/root/reference"))
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    sys.exit(0 if build(a.ref, a.force) else 1)
