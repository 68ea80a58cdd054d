"""The CPU oracle: internal consistency, and pinned against the reference's
own outputs (golden vectors produced by running BlitzGS's CUDA rasterizer)."""
import numpy as np
import pytest
import torch

from blitzgs_b200 import scene as S
from oracle import rasterizer_oracle as O
from tests.conftest import golden_path
from tests.golden.make_golden import input_checksum, small_scene
from tests.helpers import GRAD_RTOL, IMG_ATOL, activated, normwise_rel, scene_params


def _pre(sc, cam):
    xyz, s, q, shs, o = activated(sc)
    return O.preprocess_forward(xyz, s, q, shs, o, cam.world_view_transform, cam.full_proj_transform,
                                cam.camera_center, cam.tanfovx, cam.tanfovy, cam.image_height, cam.image_width, 3)


def _diff_render(m2, co, rgb, bg, pl, ranges, H, W):
    """Autograd-able restatement of the blend with the reference's skip/stop
    decisions frozen from a no-grad pass and the 0.99 clamp ignored in the
    gradient (as the reference backward does)."""
    gx = (W + 15) // 16
    img = torch.zeros(3, H, W)
    img = img + bg.view(3, 1, 1) * 0
    out = []
    for t in range(ranges.shape[0]):
        s, e = int(ranges[t][0]), int(ranges[t][1])
        xs, ys = O._tile_pixels(t, gx, H, W)
        if e == s or len(xs) == 0:
            continue
        ids = torch.as_tensor(pl[s:e])
        with torch.no_grad():
            _, _, _, _, alpha0, ok, _ = O._pair_terms(ids, m2.detach(), co.detach(), xs, ys)
            contrib, _, _, _ = O._transmittance(alpha0, ok)
        xy = m2[ids]
        c = co[ids]
        dx = xy[None, :, 0] - xs[:, None].float()
        dy = xy[None, :, 1] - ys[:, None].float()
        power = -0.5 * (c[None, :, 0] * dx * dx + c[None, :, 2] * dy * dy) - c[None, :, 1] * dx * dy
        a_raw = c[None, :, 3] * torch.exp(power)
        a = a_raw + (torch.clamp(a_raw, max=0.99) - a_raw).detach()
        a = torch.where(contrib, a, torch.zeros_like(a))
        Tc = torch.cumprod(1 - a, 1)
        Tb = torch.cat([torch.ones(len(xs), 1), Tc[:, :-1]], 1)
        col = (a * Tb) @ rgb[ids] + Tc[:, -1:] * bg.view(1, 3)
        out.append((ys, xs, col))
    for ys, xs, col in out:
        img = img.index_put((torch.arange(3)[:, None], ys[None, :], xs[None, :]), col.t())
    return img


def test_render_backward_closed_form_matches_autograd():
    sc = S.tiny(seed=21, P=300, H=48, W=64)
    cam = sc.cameras[0]
    pre = _pre(sc, cam)
    H, W = cam.image_height, cam.image_width
    pl, ranges, _ = O.binning(pre["means2D"].numpy(), pre["depths"].numpy(), pre["radii"].numpy(), H, W)
    gen = torch.Generator().manual_seed(0)
    dpix = torch.randn(3, H, W, generator=gen)
    rec = O.render_backward(pre["means2D"], pre["conic_opacity"], pre["rgb"], torch.zeros(3), pl, ranges, H, W, dpix)
    m2 = pre["means2D"].clone().requires_grad_(True)
    co = pre["conic_opacity"].clone().requires_grad_(True)
    rgb = pre["rgb"].clone().requires_grad_(True)
    img = _diff_render(m2, co, rgb, torch.zeros(3), pl, ranges, H, W)
    fwd = O.render_forward(pre["means2D"], pre["conic_opacity"], pre["rgb"], torch.zeros(3), pl, ranges, H, W)
    assert torch.allclose(img.detach(), fwd["color"], atol=1e-5)
    (img * dpix).sum().backward()
    assert normwise_rel(rec[:, 0], m2.grad[:, 0] * (0.5 * W)) < 1e-4
    assert normwise_rel(rec[:, 1], m2.grad[:, 1] * (0.5 * H)) < 1e-4
    assert normwise_rel(rec[:, 8], co.grad[:, 0]) < 1e-4
    assert normwise_rel(rec[:, 9], 0.5 * co.grad[:, 1]) < 1e-4   # half off-diagonal convention
    assert normwise_rel(rec[:, 10], co.grad[:, 2]) < 1e-4
    assert normwise_rel(rec[:, 11], co.grad[:, 3]) < 1e-4
    assert normwise_rel(rec[:, 12:15], rgb.grad) < 1e-4


def test_preprocess_backward_matches_finite_differences():
    sc = S.tiny(seed=22, P=40, H=64, W=64)
    cam = sc.cameras[0]
    xyz, s, q, shs, o = activated(sc)
    xyz, s, q, shs, o = (t.double().float() for t in (xyz, s, q, shs, o))
    pre = _pre(sc, cam)
    gen = torch.Generator().manual_seed(1)
    gm = torch.randn(40, 2, generator=gen)
    gc = torch.randn(40, 4, generator=gen)
    gr = torch.randn(40, 3, generator=gen)
    args = (cam.world_view_transform, cam.full_proj_transform, cam.camera_center, cam.tanfovx, cam.tanfovy, 64, 64, 3)
    dm, ds, dq, dsh, dop = O.preprocess_backward(xyz, s, q, shs, o, *args, pre["radii"], gm, gc, gr)

    def L(xyz_, s_, q_, shs_, o_):
        p = O.preprocess_forward(xyz_, s_, q_, shs_, o_, *args)
        W = 64
        ndc = (p["means2D"].double() * 2 + 1) / torch.tensor([W, 64.0]) - 1  # inverse ndc2pix
        vis = (pre["radii"] > 0).double()[:, None]
        conic = p["conic_opacity"].double()
        return float(((ndc * gm.double()) * vis).sum() + (conic[:, :3] * gc[:, :3].double() * torch.tensor([1.0, 2.0, 1.0]) * vis).sum()
                     + (p["rgb"].double() * gr.double() * vis).sum() + (p["conic_opacity"][:, 3].double() * gc[:, 3].double()).sum())

    eps = 1e-3
    for (name, t, g) in (("scale", s, ds), ("xyz", xyz, dm)):
        for i in range(0, 40, 7):
            if pre["radii"][i] == 0:
                continue
            for k in range(3):
                tp = t.clone()
                tp[i, k] += eps
                tm = t.clone()
                tm[i, k] -= eps
                a = [xyz, s, q, shs, o]
                idx = 1 if name == "scale" else 0
                a[idx] = tp
                lp = L(*a)
                a[idx] = tm
                lm = L(*a)
                fd = (lp - lm) / (2 * eps)
                assert abs(fd - g[i, k].item()) <= 2e-2 * max(1.0, abs(fd)), (name, i, k, fd, g[i, k].item())


def test_route_restatement_semantics():
    m2 = np.array([[8.0, 8.0], [8.0, 40.0], [100.0, 100.0]], np.float32)
    r = np.array([3, 3, 0], np.int64)
    out = O.route_bool(m2, r, 64, 64, [0, 8, 16])   # 4x4 tiles; ranks own 2 rows each
    assert out[0].tolist() == [True, False]
    assert out[1].tolist() == [False, True]
    assert out[2].tolist() == [False, False]


# ---- pinned against the reference (golden vectors) ----

def _golden(name):
    p = golden_path(name)
    if p is None:
        pytest.skip(f"{name} not generated yet")
    return dict(np.load(p))


def test_oracle_binning_equals_reference():
    g = _golden("golden_tiny.npz")
    pl, ranges, _ = O.binning(g["means2D"], g["depths"], g["radii"], 256, 256)
    assert np.array_equal(pl, g["point_list"].astype(np.int64))
    assert np.array_equal(ranges, g["ranges"].astype(np.int64))


def test_oracle_routing_equals_reference():
    g = _golden("golden_tiny.npz")
    ref = np.unpackbits(g["route_packed"])[: int(np.prod(g["route_shape"]))].reshape(g["route_shape"]).astype(bool)
    out = O.route_bool(g["means2D"], g["radii"], 256, 256, np.array([0, 4, 8, 12, 16]) * 16)
    assert np.array_equal(out, ref)


def test_oracle_preprocess_close_to_reference():
    g = _golden("golden_tiny.npz")
    sc = S.tiny()
    assert str(g["input_sha256"]) == input_checksum(sc)
    p = _pre(sc, sc.cameras[0])
    assert np.array_equal(p["radii"].numpy(), g["radii"])
    both = (p["radii"].numpy() > 0) & (g["radii"] > 0)
    assert np.abs(p["means2D"].numpy()[both] - g["means2D"][both]).max() <= 1e-5
    assert np.abs(p["depths"].numpy()[both] - g["depths"][both]).max() <= 1e-6


def test_oracle_render_close_to_reference():
    g = _golden("golden_small.npz")
    sc = small_scene()
    cam = sc.cameras[0]
    H, W = cam.image_height, cam.image_width
    f = O.render_forward(torch.from_numpy(g["means2D"]), torch.from_numpy(g["conic_opacity"]),
                         torch.from_numpy(g["rgb"]), torch.zeros(3), g["point_list"].astype(np.int64),
                         g["ranges"].astype(np.int64), H, W)
    assert np.abs(f["color"].numpy() - g["image"]).max() <= IMG_ATOL
    assert np.array_equal(f["n_contrib"].numpy(), g["n_contrib"])


def test_oracle_gradients_close_to_reference():
    g = _golden("golden_small.npz")
    sc = small_scene()
    cam = sc.cameras[0]
    gt = S.target_image(1, cam.image_height, cam.image_width)
    out = O.train_step(scene_params(sc), cam, gt)
    assert abs(out["loss"].item() - float(g["loss"])) <= 1e-6 * abs(float(g["loss"]))
    rec = out["rec"]
    assert normwise_rel(rec[:, 12:15], g["g_rgb"]) <= GRAD_RTOL
    assert normwise_rel(rec[:, 8:12], g["g_conic_opacity"]) <= GRAD_RTOL
    assert normwise_rel(rec[:, 0:2], g["g_means2D"]) <= GRAD_RTOL


def test_oracle_tiny_gradient_rows_match_reference():
    """Every gradient row of config 1 (the reference's activated-parameter
    gradients, chained through exp / normalize / sigmoid in float64)."""
    g = _golden("golden_tiny.npz")
    sc = S.tiny()
    cam = sc.cameras[0]
    gt = S.target_image(0, cam.image_height, cam.image_width)
    out = O.train_step(scene_params(sc), cam, gt)
    assert abs(out["loss"].item() - float(g["loss"])) <= 1e-6 * abs(float(g["loss"]))
    raw = [t.double().requires_grad_(True) for t in scene_params(sc)]
    acts = (raw[0], torch.exp(raw[1]), torch.nn.functional.normalize(raw[2]), torch.cat((raw[4], raw[5]), 1),
            torch.sigmoid(raw[3]))
    ups = [torch.from_numpy(g[k]).double().reshape(a.shape)
           for k, a in zip(("g_means3D", "g_scales", "g_rotations", "g_shs", "g_opacities"), acts)]
    torch.autograd.backward(acts, ups)
    for name, mine, r in zip(("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"),
                             out["grads"], raw):
        assert normwise_rel(mine, r.grad) <= GRAD_RTOL, name


def _golden_optim():
    import os
    import sys
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    import make_golden_optim as G
    g = np.load(os.path.join(here, "golden_optim.npz"))
    adam, route = G.inputs()
    assert str(g["input_sha256"]) == G.checksum(adam, route)
    return G, g, adam, route


def test_oracle_adam_bit_exact_against_reference():
    """The reference's _C.adamUpdate, three lazy-Adam steps: parameter and
    both moments of the visible rows bit for bit; the other rows untouched."""
    G, g, adam, _ = _golden_optim()
    for (M, N), (param, grads, vis) in zip(G.ADAM_CASES, adam):
        p, m, v = param.clone(), torch.zeros_like(param), torch.zeros_like(param)
        for t, gr in enumerate(grads, start=1):
            O.adam_update(p, gr, m, v, vis, G.lr_at(t), 0.9, 0.999, G.EPS)
        assert np.array_equal(p[vis].numpy().view(np.uint32), g[f"adam{M}_param"].view(np.uint32))
        assert np.array_equal(m[vis].numpy().view(np.uint32), g[f"adam{M}_exp_avg"].view(np.uint32))
        assert np.array_equal(v[vis].numpy().view(np.uint32), g[f"adam{M}_exp_avg_sq"].view(np.uint32))
        assert torch.equal(p[~vis], param[~vis]) and not m[~vis].any() and not v[~vis].any()


def test_oracle_fma32_is_correctly_rounded():
    """fma32 against exact rational arithmetic (round to nearest, ties to
    even) on seeded operands, a quarter of them with c cancelling a*b down to
    its float32 rounding error."""
    from fractions import Fraction
    gen = torch.Generator().manual_seed(3)
    a = torch.randn(400, generator=gen)
    b = torch.randn(400, generator=gen)
    c = torch.randn(400, generator=gen)
    # c = float32(a*b) - a*b: the exact product minus its own rounding
    ab32 = (a.double() * b.double()).float()
    c[:100] = (-(a[:100].double() * b[:100].double()) + ab32[:100].double()).float()
    got = O.fma32(a, b, c)
    for i in range(400):
        exact = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        lo = float(np.float32(float(exact)))  # float64 rounding first: bracket the answer
        cand = [np.float32(lo), np.nextafter(np.float32(lo), np.float32(np.inf)),
                np.nextafter(np.float32(lo), np.float32(-np.inf))]
        best = min(cand, key=lambda x: (abs(Fraction(float(x)) - exact),
                                        int(np.array(x, np.float32).view(np.uint32)) & 1))
        assert np.float32(got[i]) == best, i


def test_oracle_mode6_routing_equals_reference():
    """The reference's _C.get_local2j_ids_bool_adjust_mode6 on seeded screen
    means, radii (zeros included) and four tile rectangles, with and without
    avoid_pixel_all2all."""
    G, g, _, (means2D, radii, rects) = _golden_optim()
    for avoid in (False, True):
        got = O.route_rect_bool(means2D.numpy(), radii.numpy(), G.H, G.W, rects.numpy(), avoid)
        assert np.array_equal(got, g[f"mode6_avoid{int(avoid)}"])


# ---- the full rasterizer (rasterize_gaussians / _simp / mark_visible) ----

def test_oracle_full_binning_equals_reference():
    """The exact tile test over the float rectangles reproduces the
    reference's per-tile lists and ranges bit for bit."""
    from tests.golden.make_golden_full import full_scene
    g = _golden("golden_full.npz")
    sc, cam, culling, weight, colors = full_scene()
    H, W = int(cam.image_height), int(cam.image_width)
    pl, ranges, counts = O.full_binning(g["means2D"], g["depths"], g["radii"], g["rects"], g["conic_opacity"], H, W)
    assert np.array_equal(ranges, g["ranges"].astype(np.int64))
    assert np.array_equal(pl, g["point_list"].astype(np.int64))
    # the exact test drops tiles of the rectangle: fewer instances than rect tiles
    x0, y0, x1, y1 = O.tile_rect_float(g["means2D"], g["rects"], (W + 15) // 16, (H + 15) // 16)
    rect_tiles = ((x1 - x0) * (y1 - y0))[g["radii"] > 0].sum()
    assert 0 < counts.sum() < rect_tiles


def test_oracle_full_render_statistics_match_reference():
    """Image, accum_max_count and the simp accumulators from the oracle's
    blend over the reference's lists (CPU expf may differ from CUDA's in the
    last bit, so a near-tie may flip: at most 0.1 % of the Gaussians)."""
    from tests.golden.make_golden_full import BG, full_scene
    g = _golden("golden_full.npz")
    sc, cam, culling, weight, colors = full_scene()
    H, W = int(cam.image_height), int(cam.image_width)
    P = len(g["radii"])
    pl, rg = g["point_list"].astype(np.int64), g["ranges"].astype(np.int64)
    f = O.render_forward(torch.from_numpy(g["means2D"]), torch.from_numpy(g["conic_opacity"]),
                         torch.from_numpy(g["rgb"]), torch.tensor(BG), pl, rg, H, W)
    assert np.abs(f["color"].numpy() - g["image"]).max() <= IMG_ATOL
    assert np.array_equal(f["n_contrib"].numpy(), g["n_contrib"])
    mx, aw, an = O.render_stats(g["means2D"], g["conic_opacity"], pl, rg, H, W, P)
    assert mx.sum().item() == g["accum_max_count"].sum() > 0
    assert (mx.numpy() != g["accum_max_count"]).sum() <= max(2, P // 1000)
    assert np.array_equal(an.numpy(), g["accum_weights_count"])
    w = g["accum_weights_ptr"].astype(np.float64)
    assert np.abs(aw.numpy() - w).max() <= 1e-5 * max(1.0, np.abs(w).max())


def test_oracle_mark_visible_equals_reference():
    from tests.golden.make_golden_full import full_scene
    g = _golden("golden_full.npz")
    sc, cam, culling, weight, colors = full_scene()
    vis = O.mark_visible(sc.xyz * 3.0, cam.world_view_transform)
    assert np.array_equal(vis, g["mark_visible"]) and 0 < vis.sum() < len(vis)
