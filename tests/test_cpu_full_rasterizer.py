"""GaussianRasterizer.forward (the reference's full rasterizer) is composed
from the two training-path operators; on the CPU the composition is checked
with stand-ins for those operators (the operators themselves are checked on
the GPU): argument validation with the reference's messages, SH assembly
from dc + rest, culled Gaussians dropped through their radii, and the
screen-space gradient routed to the caller's means2D."""
import pytest
import torch

from blitzgs_b200 import rasterizer as RZ


class _Settings:
    image_height, image_width = 8, 8


def _fakes(monkeypatch, seen):
    def pre(means3D, scales, rotations, sh, opacities, rs, cuda_args):
        seen["sh"] = sh
        m2 = means3D[:, :2] * 2.0
        rgb = sh[:, 0, :] * 1.0
        conic = torch.cat([scales, opacities], 1)
        radii = torch.full((means3D.shape[0],), 5, dtype=torch.int32)
        return m2, rgb, conic, radii, means3D[:, 2].detach()

    def render(m2, m2_abs, conic, rgb, all_map, depths, radii, cl, ecl, rs, cuda_args):
        seen["radii"] = radii.clone()
        w = (radii > 0).float()[:, None]
        v = (m2 * w).sum() + 3.0 * (rgb * w).sum()
        color = v * torch.ones((3, rs.image_height, rs.image_width))
        return color, None, None, None, None, None, None

    monkeypatch.setattr(RZ, "preprocess_gaussians", pre)
    monkeypatch.setattr(RZ, "render_gaussians", render)


def test_forward_composes_preprocess_culling_and_render(monkeypatch):
    seen = {}
    _fakes(monkeypatch, seen)
    P = 6
    g = torch.Generator().manual_seed(1)
    means3D = torch.randn(P, 3, generator=g, requires_grad=True)
    dc = torch.randn(P, 1, 3, generator=g, requires_grad=True)
    rest = torch.randn(P, 15, 3, generator=g, requires_grad=True)
    screen = torch.zeros(P, 3, requires_grad=True)
    culling = torch.tensor([False, True, False, False, True, False])
    rast = RZ.GaussianRasterizer(_Settings())
    color, radii, accum = rast(means3D, screen, torch.rand(P, 1, generator=g), culling, dc=dc, shs=rest,
                               scales=torch.rand(P, 3, generator=g), rotations=torch.randn(P, 4, generator=g))
    assert seen["sh"].shape == (P, 16, 3) and torch.equal(seen["sh"][:, 0], dc[:, 0]) and torch.equal(seen["sh"][:, 1:], rest)
    assert torch.equal(radii, torch.tensor([5, 0, 5, 5, 0, 5], dtype=torch.int32))
    assert torch.equal(seen["radii"], radii)
    assert accum.shape == (P,) and not accum.any()
    color.sum().backward()
    keep = (~culling).float()[:, None]
    n = color.numel()
    # d color.sum / d screen[:, :2] = n * w; the third column gets nothing
    assert torch.equal(screen.grad[:, :2], n * keep.expand(P, 2))
    assert not screen.grad[:, 2].any()
    assert torch.equal(dc.grad[:, 0], 3.0 * n * keep.expand(P, 3))
    assert not rest.grad.any()


def test_forward_argument_validation(monkeypatch):
    _fakes(monkeypatch, {})
    rast = RZ.GaussianRasterizer(_Settings())
    P = 3
    x, s, q, o = torch.zeros(P, 3), torch.ones(P, 3), torch.ones(P, 4), torch.ones(P, 1)
    sh = torch.zeros(P, 16, 3)
    with pytest.raises(Exception, match="excatly one of either SHs or precomputed colors"):
        rast(x, torch.zeros(P, 3), o, None, scales=s, rotations=q)
    with pytest.raises(Exception, match="exactly one of either scale/rotation pair"):
        rast(x, torch.zeros(P, 3), o, None, shs=sh, scales=s)
    with pytest.raises(NotImplementedError, match="precomputed colours"):
        rast(x, torch.zeros(P, 3), o, None, colors_precomp=torch.zeros(P, 3), scales=s, rotations=q)
    with pytest.raises(NotImplementedError, match="precomputed 3D covariances"):
        rast(x, torch.zeros(P, 3), o, None, shs=sh, cov3D_precomp=torch.zeros(P, 6))
    with pytest.raises(NotImplementedError, match="flag_max_count"):
        rast(x, torch.zeros(P, 3), o, None, shs=sh, scales=s, rotations=q, flag_max_count=True)
    # without dc, shs carries every coefficient
    color, radii, _ = rast(x, torch.zeros(P, 3), o, None, shs=sh, scales=s, rotations=q)
    assert color.shape == (3, 8, 8) and torch.all(radii == 5)
