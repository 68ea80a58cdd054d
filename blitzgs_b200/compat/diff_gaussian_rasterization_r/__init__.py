"""Import-name shim for ``diff_gaussian_rasterization_r`` (the reference's split
render backend, imported by the _f wrapper and by gaussian_renderer); it
exposes the same B200 operators as diff_gaussian_rasterization_f."""
from blitzgs_b200.rasterizer import (  # noqa: F401
    _C,
    GaussianRasterizationSettings,
    GaussianRasterizer,
    _PreprocessGaussians,
    _RenderGaussians,
    preprocess_gaussians,
    render_gaussians,
)
