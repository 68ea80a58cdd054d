"""Import-name shim: ``import diff_gaussian_rasterization_f`` resolves to the
B200 implementation when ``blitzgs_b200/compat`` is on sys.path ahead of
any installed reference build.  Same public names as the reference package
(submodule/diff-gaussian-rasterization_f/diff_gaussian_rasterization_f/__init__.py)."""
from blitzgs_b200.rasterizer import (  # noqa: F401
    _C,
    GaussianRasterizationSettings,
    GaussianRasterizer,
    _PreprocessGaussians,
    _RasterizeGaussians,
    _RenderGaussians,
    SparseGaussianAdam,
    preprocess_gaussians,
    rasterize_gaussians,
    rasterize_gaussians_depth,
    rasterize_gaussians_simp,
    render_gaussians,
)
