"""The fused training step (blitzgs_b200.step.view_loss, the benchmarked path)
against the REFERENCE rasterizer run live on the same GPU, at BASELINE's
own scene sizes.

The reference is BlitzGS's diff_gaussian_rasterization_f / _r CUDA modules
built unmodified from the reference sources (oracle/build_ref.py ->
oracle/_ref/), driven through its stock Python wrappers and loss helpers
(tests/ref_runner.py).  Both sides get the same seeded synthetic scene and
cameras (blitzgs_b200.scene) and the same uint8 target.

Bit-exact: radii (the culling mask), screen means and depths of every
visible Gaussian, the sorted per-tile Gaussian lists, tile ranges, per-pixel
contributor counts and final transmittance, per-tile statistics and
per-Gaussian observation counts.
Within tolerance: the image within 1e-5 absolute (IMG_ATOL); the loss within
1e-6 relative; the gradients of the six raw parameter tensors within 1e-4
relative, normwise per tensor (GRAD_RTOL), which allows for the reordering of
floating-point sums the reference leaves to atomics.

The fused path runs a conservative cull before the reference computation
(preprocess_cull_kernel), reads only the listed rows, and replays per-strip
contributor lists in the backward; these tests pin all three at the scale
the bench measures.  A planted case puts Gaussians on both sides of the near
plane (view depth 0.2 +- 5e-5) at world coordinates around 1000, where the
rounding of the view transform (~1e-4) is larger than the spread, so the
cull's near-plane and screen margins must cover the reference's own
rounding.
"""
import math

import numpy as np
import pytest
import torch

from blitzgs_b200 import distributed as D, ops, scene as S, step as ST
from tests import ref_runner as REF
from tests.helpers import GRAD_RTOL, IMG_ATOL, normwise_rel

pytestmark = pytest.mark.gpu

if not REF.available():
    pytest.skip("reference build oracle/_ref absent (python oracle/build_ref.py)", allow_module_level=True)

NAMES = ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest")


def _zorder(sc):
    order = D.zorder_shards(sc.xyz, 1)[0]
    for name in NAMES:
        setattr(sc, name, getattr(sc, name)[order].contiguous())
    return sc


_SCENES = {}


def _scene(name):
    """2 = mid (1M uniform), 3 = city (8M clustered, z-order
    layout as the bench stores it), 5 = skew (8M, heavy-tailed tiles)."""
    if name not in _SCENES:
        _SCENES.clear()  # one 8M scene resident at a time
        if name == "city":
            _SCENES[name] = _zorder(S.city(seed=0))
        elif name == "mid":
            _SCENES[name] = S.mid(seed=0)
        else:
            _SCENES[name] = S.skew(seed=0)
    return _SCENES[name]


class _Capture:
    """Records what the fused step's forward hands between its kernels."""

    def __init__(self, monkeypatch):
        self.pre = None
        self.render = None
        real_pre, real_render = ops.preprocess_forward_raw, ops.render_forward

        def pre(*a, **k):
            self.pre = real_pre(*a, **k)
            return self.pre

        def render(*a, **k):
            self.render = real_render(*a, **k)
            return self.render

        monkeypatch.setattr(ops, "preprocess_forward_raw", pre)
        monkeypatch.setattr(ops, "render_forward", render)


def _bits(t):
    return REF.as_np(t).view(np.uint32)


def _check_view(sc, ci, dev, monkeypatch):
    cam = sc.cameras[ci]
    H, W = cam.image_height, cam.image_width
    gt = S.target_image(ci, H, W)
    model_cpu = [getattr(sc, n) for n in NAMES]

    ref = REF.train_view(model_cpu, cam, gt, dev)

    cap = _Capture(monkeypatch)
    model = [t.to(dev).requires_grad_(True) for t in model_cpu]
    rs = S.raster_settings(cam.to(dev), device=dev)
    loss, l1, ss, radii, out_observe, color = ST.view_loss(model, rs, gt.to(dev))
    loss.backward()
    torch.cuda.synchronize()

    # culling mask and integer radii
    r_ours, r_ref = REF.as_np(radii), REF.as_np(ref["radii"])
    bad = np.nonzero(r_ours != r_ref)[0]
    assert len(bad) == 0, (f"radii differ at {len(bad)} Gaussians; first {bad[:5].tolist()}: "
                           f"ours {r_ours[bad[:5]].tolist()} reference {r_ref[bad[:5]].tolist()}")
    vis = torch.from_numpy(r_ref > 0)
    n_vis = int(vis.sum())
    assert n_vis > 1000, f"camera {ci} sees only {n_vis} Gaussians"
    # listed rows of the fused preprocess (only these are written)
    m2, depths, _, conic, rgb = cap.pre[:5]
    idx = torch.nonzero(vis).flatten().to(dev)
    assert np.array_equal(_bits(m2[idx]), _bits(ref["means2D"][idx])), "means2D differ"
    assert np.array_equal(_bits(depths[idx]), _bits(ref["depths"][idx])), "depths differ"
    for name, a, b in (("conic_opacity", conic[idx], ref["conic_opacity"][idx]), ("rgb", rgb[idx], ref["rgb"][idx])):
        err = (a - b).abs().max().item()
        assert err <= 1e-6 * max(1.0, b.abs().max().item()), f"{name} max error {err}"

    # binning: sorted per-tile lists and ranges
    color_r, n_render, n_consider, n_contrib_tile, _, st = cap.render
    R = ref["point_list"].numel()
    assert st.R == R, f"R {st.R} vs reference {R}"
    assert np.array_equal(_bits(st.point_list[:R]), _bits(ref["point_list"])), "sorted tile lists differ"
    assert np.array_equal(_bits(st.ranges), _bits(ref["ranges"])), "tile ranges differ"
    # blend: per-pixel counts and transmittance, tile statistics, observations
    nc_ours, nc_ref = REF.as_np(st.n_contrib), REF.as_np(ref["n_contrib"])
    bad = np.nonzero(nc_ours != nc_ref)[0]
    assert len(bad) == 0, f"n_contrib differs at {len(bad)} pixels; first {bad[:5].tolist()}"
    bad = np.nonzero(_bits(st.final_T) != _bits(ref["final_T"]))[0]
    assert len(bad) == 0, f"final_T differs at {len(bad)} pixels; first {bad[:5].tolist()}"
    for k, a in (("n_render", n_render), ("n_consider", n_consider), ("n_contrib_tile", n_contrib_tile),
                 ("out_observe", out_observe)):
        assert np.array_equal(REF.as_np(a), REF.as_np(ref[k])), f"{k} differs"
    err = (color - ref["image"]).abs().max().item()
    assert err <= IMG_ATOL, f"image max abs error {err}"

    # loss and raw-parameter gradients
    assert abs(loss.item() - ref["loss"]) <= 1e-6 * abs(ref["loss"]), (loss.item(), ref["loss"])
    for name, p, g in zip(NAMES, model, ref["grads"]):
        r = normwise_rel(p.grad.cpu(), g.cpu())
        assert r <= GRAD_RTOL, f"grad {name}: normwise relative error {r:.3e} (camera {ci}, {n_vis} visible)"
    return n_vis, R


@pytest.mark.parametrize("config,cams", [("city", (0, 1)), ("mid", (0, 1)), ("skew", (0,))],
                         ids=["config3_city_8M", "config2_mid_1M", "config5_skew_8M"])
def test_fused_step_matches_reference(cuda_device, monkeypatch, config, cams):
    sc = _scene(config)
    for ci in cams:
        n_vis, R = _check_view(sc, ci, cuda_device, monkeypatch)
        print(f"{config} camera {ci}: {n_vis} visible Gaussians, {R} tile instances: bit-exact")
    torch.cuda.empty_cache()


def near_plane_scene(seed=5, n_planted=8192, n_random=8192, H=864, W=1152):
    """Gaussians planted at view depth 0.2 +- 5e-5 in front of a camera at
    world coordinates around 1000 (the city's scale), with lateral offsets
    reaching past the image edges, plus random Gaussians of the city's kind."""
    g = torch.Generator().manual_seed(seed)
    pos = np.array([950.0, -880.0, 60.0])
    cam = S.look_at_camera(pos, pos + np.array([0.6, 0.5, -0.62]), [0, 0, 1.0], W, H, math.radians(70))
    wv = cam.world_view_transform.double().t()  # world -> view, column vectors
    R, t = wv[:3, :3], wv[:3, 3]
    z = 0.2 + (torch.rand(n_planted, generator=g, dtype=torch.float64) - 0.5) * 1e-4
    lat = (torch.rand(n_planted, 2, generator=g, dtype=torch.float64) - 0.5) * 0.6
    view = torch.stack([lat[:, 0], lat[:, 1], z], 1)
    world_planted = ((view - t) @ R).float()  # R^T (v - t), row vectors
    world_random = torch.from_numpy(pos).float() + (torch.rand(n_random, 3, generator=g) - 0.5) * torch.tensor(
        [200.0, 200.0, 80.0])
    xyz = torch.cat([world_planted, world_random], 0)
    P = xyz.shape[0]
    scaling = torch.cat([torch.randn(n_planted, 3, generator=g) * 0.3 - 6.0,
                         torch.randn(n_random, 3, generator=g) * 0.5 - 1.5], 0)
    rotation = torch.randn(P, 4, generator=g)
    opacity = torch.randn(P, 1, generator=g) + 2.0
    dc = torch.randn(P, 1, 3, generator=g) * 0.5
    rest = torch.randn(P, 15, 3, generator=g) * 0.05
    return S.Scene("near_plane", xyz, scaling, rotation, opacity, dc, rest, [cam]), n_planted


def test_near_plane_cull_at_city_coordinates(cuda_device):
    sc, n_planted = near_plane_scene()
    cam = sc.cameras[0]
    model = [getattr(sc, n).to(cuda_device) for n in NAMES]
    ref = REF.preprocess(model, cam, cuda_device)
    r_ref = REF.as_np(ref[3])
    kept = int((r_ref[:n_planted] > 0).sum())
    # the planted band must straddle the reference's own near-plane decision
    assert 0 < kept < n_planted, f"{kept} of {n_planted} planted Gaussians visible: the case tests nothing"
    rs = S.raster_settings(cam.to(cuda_device), device=cuda_device)
    sh = ops.sh_layout(dc=model[4], rest=model[5])
    for two_pass in (True, False):
        out = ops.preprocess_forward_raw(model[0], model[1], model[2], model[3].reshape(-1), sh, rs,
                                         want_counts=True, two_pass=two_pass)
        r = REF.as_np(out[2])
        bad = np.nonzero(r != r_ref)[0]
        assert len(bad) == 0, (f"two_pass={two_pass}: radii differ at {len(bad)} Gaussians "
                               f"(planted: {int((bad < n_planted).sum())}); first {bad[:5].tolist()}")
    # the operator API's preprocess (activated inputs, same cull) as well
    xyz, s, q, o = model[0], torch.exp(model[1]), torch.nn.functional.normalize(model[2]), torch.sigmoid(model[3])
    m2, d, r, *_ = ops.preprocess_forward(xyz, s, q, o.reshape(-1), ops.sh_layout(dc=model[4], rest=model[5]), rs)
    assert np.array_equal(REF.as_np(r), r_ref), "operator-API radii differ"
    vis = torch.from_numpy(r_ref > 0).to(cuda_device)
    assert np.array_equal(_bits(m2[vis]), _bits(ref[0][vis]))
    assert np.array_equal(_bits(d[vis]), _bits(ref[4][vis]))
