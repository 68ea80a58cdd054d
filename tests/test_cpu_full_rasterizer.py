"""GaussianRasterizer.forward / render_simp / render_depth / markVisible (the
reference's full rasterizer, f/__init__.py:666-810) on the CPU: the argument
checks with the reference's messages, the SH layouts the three entry points
accept, and the refusal of CPU tensors (the kernels themselves are checked
against the reference on the GPU in tests/test_gpu_full_rasterizer.py)."""
import pytest
import torch

from blitzgs_b200 import rasterizer as RZ


class _Settings:
    image_height, image_width = 8, 8
    tanfovx = tanfovy = 0.5
    bg = torch.zeros(3)
    scale_modifier = 1.0
    viewmatrix = torch.eye(4)
    projmatrix = torch.eye(4)
    sh_degree = 3
    campos = torch.zeros(3)
    prefiltered = False
    debug = False


def _args(P=3):
    return torch.zeros(P, 3), torch.zeros(P, 3), torch.ones(P, 1), torch.ones(P, 3), torch.ones(P, 4)


@pytest.mark.parametrize("method", ["forward", "render_simp", "render_depth"])
def test_argument_checks_use_the_reference_messages(method):
    rast = RZ.GaussianRasterizer(_Settings())
    fn = getattr(rast, method)
    x, m2, o, s, q = _args()
    sh = torch.zeros(3, 15, 3)
    with pytest.raises(Exception, match="excatly one of either SHs or precomputed colors"):
        fn(x, m2, o, None, scales=s, rotations=q)
    with pytest.raises(Exception, match="excatly one of either SHs or precomputed colors"):
        fn(x, m2, o, None, shs=sh, colors_precomp=torch.zeros(3, 3), scales=s, rotations=q)
    with pytest.raises(Exception, match="exactly one of either scale/rotation pair"):
        fn(x, m2, o, None, shs=sh, scales=s)
    with pytest.raises(Exception, match="exactly one of either scale/rotation pair"):
        fn(x, m2, o, None, shs=sh, scales=s, rotations=q, cov3D_precomp=torch.zeros(3, 6))


def test_precomputed_covariances_are_refused():
    rast = RZ.GaussianRasterizer(_Settings())
    x, m2, o, _, _ = _args()
    with pytest.raises(NotImplementedError, match="precomputed 3D covariances"):
        rast(x, m2, o, None, shs=torch.zeros(3, 15, 3), cov3D_precomp=torch.zeros(3, 6))


def test_cpu_tensors_are_refused():
    rast = RZ.GaussianRasterizer(_Settings())
    x, m2, o, s, q = _args()
    dc, rest = torch.zeros(3, 1, 3), torch.zeros(3, 15, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        rast(x, m2, o, None, dc=dc, shs=rest, scales=s, rotations=q, flag_max_count=True)
    with pytest.raises(RuntimeError, match="CUDA"):
        rast.render_simp(x, m2, o, None, dc=dc, shs=rest, scales=s, rotations=q)
    with pytest.raises(RuntimeError, match="CUDA"):
        rast.markVisible(x)


def test_sh_layouts():
    P = 4
    dc = torch.arange(P * 3, dtype=torch.float32).reshape(P, 1, 3)
    rest = torch.arange(P * 45, dtype=torch.float32).reshape(P, 15, 3)
    # dc + rest read in place, rest = the coefficients beyond DC
    (d, ds, r, rs, M, _), deg = RZ._full_sh(dc, rest, None, P, "cpu")
    assert d is dc and r is rest and (ds, rs, M, deg) == (3, 45, 15, None)
    # without dc, shs carries every coefficient
    full = torch.cat((dc, rest), 1)
    (d, ds, r, rs, M, _), deg = RZ._full_sh(None, full, None, P, "cpu")
    assert d is full and (ds, rs, M, deg) == (48, 48, 15, None)
    # precomputed colours: a zero DC at degree 0 stands in
    (d, ds, r, rs, M, _), deg = RZ._full_sh(torch.Tensor([]), torch.Tensor([]), torch.ones(P, 3), P, "cpu")
    assert d.shape == (P, 1, 3) and not d.any() and M == 0 and deg == 0
