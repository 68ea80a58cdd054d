"""CUDA path vs the REFERENCE rasterizer's own outputs (golden vectors made by
tests/golden/make_golden.py running BlitzGS's CUDA modules on a B200).

Bit-exact: radii, screen means, depths, per-tile sorted Gaussian lists, tile
ranges, n_contrib, tile statistics, observation counts, routing mask.
Images within 1e-5 absolute; gradients within 1e-4 relative (normwise per
tensor), allowing for the reordering of floating-point sums.
"""
import numpy as np
import pytest
import torch

from blitzgs_b200 import ops, scene as S, step as ST
from blitzgs_b200 import rasterizer as RZ
from tests.conftest import golden_path
from tests.golden.make_golden import input_checksum, small_scene
from tests.helpers import GRAD_RTOL, IMG_ATOL, activated, assert_grad_close, scene_params

pytestmark = pytest.mark.gpu


def _load(name):
    p = golden_path(name)
    if p is None:
        pytest.skip(f"{name} not generated yet")
    return dict(np.load(p))


def _run(sc, cam, dev, compute_locally=None):
    xyz, s, q, shs, o = activated(sc, dev)
    rs = S.raster_settings(cam, device=dev)
    m2, d, r, co, rgb, _, _ = ops.preprocess_forward(xyz, s, q, o.reshape(-1), ops.sh_layout(shs=shs), rs)
    H, W = cam.image_height, cam.image_width
    cl = compute_locally.to(dev) if compute_locally is not None else None
    color, nr, nc, nct, obs, st = ops.render_forward(m2, d, r, co, rgb, rs.bg, cl, H, W)
    return dict(radii=r, means2D=m2, depths=d, conic_opacity=co, rgb=rgb, image=color, n_render=nr,
                n_consider=nc, n_contrib_tile=nct, out_observe=obs, state=st, rs=rs)


def _local_pixel_mask(H, W, band_rows=None):
    m = np.ones((H, W), bool)
    if band_rows is not None:
        m[:] = False
        m[band_rows[0] * 16: min(H, band_rows[1] * 16)] = True
    return m.reshape(-1)


def _check_forward(g, o, prefix="", band_rows=None):
    assert np.array_equal(o["radii"].cpu().numpy(), g[prefix + "radii"]), "radii differ from the reference"
    assert np.array_equal(o["means2D"].cpu().numpy().view(np.uint32), g[prefix + "means2D"].view(np.uint32))
    assert np.array_equal(o["depths"].cpu().numpy().view(np.uint32), g[prefix + "depths"].view(np.uint32))
    st = o["state"]
    R = len(g[prefix + "point_list"])
    assert st.R == R
    assert np.array_equal(st.point_list[:R].cpu().numpy().view(np.uint32), g[prefix + "point_list"])
    assert np.array_equal(st.ranges.cpu().numpy().view(np.uint32), g[prefix + "ranges"])
    H, W = o["image"].shape[1], o["image"].shape[2]
    loc = _local_pixel_mask(H, W, band_rows)
    assert np.array_equal(st.n_contrib.cpu().numpy().astype(np.int64)[loc], g[prefix + "n_contrib"].astype(np.int64)[loc])
    if prefix + "final_T" in g:
        mine = st.final_T.cpu().numpy()[loc]
        ref = g[prefix + "final_T"][loc]
        bad = np.nonzero(mine.view(np.uint32) != ref.view(np.uint32))[0]
        assert len(bad) == 0, (f"final_T differs at {len(bad)} local pixels; first {bad[:5].tolist()}: "
                               f"ours {mine[bad[:5]].tolist()} reference {ref[bad[:5]].tolist()}")
    for k in ("n_render", "n_consider", "n_contrib_tile", "out_observe"):
        assert np.array_equal(o[k].cpu().numpy(), g[prefix + k]), k
    err = np.abs(o["image"].cpu().numpy() - g[prefix + "image"]).max()
    assert err <= IMG_ATOL, f"image max abs error {err}"


def test_tiny_forward_bit_exact(cuda_device):
    g = _load("golden_tiny.npz")
    sc = S.tiny()
    assert str(g["input_sha256"]) == input_checksum(sc)
    o = _run(sc, sc.cameras[0], cuda_device)
    _check_forward(g, o)


def test_tiny_routing_mask_exact(cuda_device):
    g = _load("golden_tiny.npz")
    sc = S.tiny()
    o = _run(sc, sc.cameras[0], cuda_device)
    gx = 16
    dist = torch.tensor([0, 4, 8, 12, 16], dtype=torch.int32, device=cuda_device) * gx
    m = ops.local2j_ids_bool(256, 256, 0, 4, o["means2D"], o["radii"], dist).cpu().numpy()
    ref = np.unpackbits(g["route_packed"])[: int(np.prod(g["route_shape"]))].reshape(g["route_shape"]).astype(bool)
    assert np.array_equal(m, ref)


def test_tiny_loss_and_gradients(cuda_device):
    """Operator API (activated inputs) against every gradient row the
    reference produced for config 1."""
    g = _load("golden_tiny.npz")
    if "g_shs" not in g:
        pytest.skip("golden_tiny.npz predates the full gradient rows (tests/golden/make_golden.py --only tiny)")
    sc = S.tiny()
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(0, cam.image_height, cam.image_width).to(cuda_device)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    rs = S.raster_settings(cam, device=cuda_device)
    # gradients w.r.t. the activated parameters, as the golden stores them
    xyz, s_raw, q_raw, o_raw, dc, rest = model
    acts = [xyz, torch.exp(s_raw).detach().requires_grad_(True),
            torch.nn.functional.normalize(q_raw).detach().requires_grad_(True),
            torch.cat((dc, rest), 1).detach().requires_grad_(True), torch.sigmoid(o_raw).detach().requires_grad_(True)]
    rast = RZ.GaussianRasterizer(rs)
    m2, rgb, co, radii, depths = rast.preprocess_gaussians(*acts[:4], acts[4], {"stats_collector": {}})
    m2.retain_grad()
    rgb.retain_grad()
    co.retain_grad()
    H, W = cam.image_height, cam.image_width
    cl = torch.ones((16, 16), dtype=torch.bool, device=cuda_device)
    color, *_ = rast.render_gaussians(m2, torch.zeros_like(xyz, requires_grad=True) + 0, co, rgb, torch.zeros((xyz.shape[0], 5),
                                      device=cuda_device), depths, radii, cl, None, {})
    from blitzgs_b200.loss import band_loss
    l1, ss = band_loss(color, gt)
    n3 = H * W * 3
    loss = 0.8 * l1 / n3 + 0.2 * (1 - ss / n3)
    assert abs(l1.item() - float(g["l1_sum"])) <= 1e-5 * abs(float(g["l1_sum"]))
    assert abs(ss.item() - float(g["ssim_sum"])) <= 1e-4 * max(1.0, abs(float(g["ssim_sum"])))
    loss.backward()
    for name, t in (("g_means3D", acts[0]), ("g_scales", acts[1]), ("g_rotations", acts[2]), ("g_shs", acts[3]),
                    ("g_opacities", acts[4]), ("g_means2D", m2), ("g_conic_opacity", co), ("g_rgb", rgb)):
        assert_grad_close(t.grad.cpu(), torch.from_numpy(g[name]).reshape(t.grad.shape), GRAD_RTOL, name)


def test_tiny_fused_step_gradients(cuda_device):
    """The fused step (raw parameters, activations in the kernels) against the
    same reference gradient rows, chained through exp / normalize / sigmoid
    in float64 on the host."""
    g = _load("golden_tiny.npz")
    if "g_shs" not in g:
        pytest.skip("golden_tiny.npz predates the full gradient rows (tests/golden/make_golden.py --only tiny)")
    sc = S.tiny()
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(0, cam.image_height, cam.image_width).to(cuda_device)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    rs = S.raster_settings(cam, device=cuda_device)
    loss, l1, ss, radii, obs, color = ST.view_loss(model, rs, gt, scale_reg_weight=0.0)
    loss.backward()
    assert abs(loss.item() - float(g["loss"])) <= 1e-6 * abs(float(g["loss"]))
    assert np.array_equal(radii.cpu().numpy(), g["radii"])
    assert np.array_equal(obs.cpu().numpy(), g["out_observe"])
    assert np.abs(color.detach().cpu().numpy() - g["image"]).max() <= IMG_ATOL
    raw = [t.double().requires_grad_(True) for t in scene_params(sc)]
    acts = (raw[0], torch.exp(raw[1]), torch.nn.functional.normalize(raw[2]), torch.cat((raw[4], raw[5]), 1),
            torch.sigmoid(raw[3]))
    ups = [torch.from_numpy(g[k]).double().reshape(a.shape)
           for k, a in zip(("g_means3D", "g_scales", "g_rotations", "g_shs", "g_opacities"), acts)]
    torch.autograd.backward(acts, ups)
    for name, p, r in zip(("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"), model, raw):
        assert_grad_close(p.grad.cpu(), r.grad, GRAD_RTOL, name)


def test_small_edge_cases_full(cuda_device):
    g = _load("golden_small.npz")
    sc = small_scene()
    assert str(g["input_sha256"]) == input_checksum(sc)
    cam = sc.cameras[0]
    o = _run(sc, cam, cuda_device)
    _check_forward(g, o)
    assert np.abs(o["conic_opacity"].cpu().numpy() - g["conic_opacity"]).max() <= 1e-6 * max(
        1.0, np.abs(g["conic_opacity"]).max())
    assert np.abs(o["rgb"].cpu().numpy() - g["rgb"]).max() <= 1e-6
    # band render
    H, W = cam.image_height, cam.image_width
    band = torch.zeros(((H + 15) // 16, (W + 15) // 16), dtype=torch.bool)
    r0, r1 = g["band_rows"]
    band[r0:r1] = True
    ob = _run(sc, cam, cuda_device, compute_locally=band)
    _check_forward(g, ob, "band_", band_rows=(r0, r1))


def test_small_gradients(cuda_device):
    g = _load("golden_small.npz")
    sc = small_scene()
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(1, cam.image_height, cam.image_width).to(cuda_device)
    rs = S.raster_settings(cam, device=cuda_device)
    xyz, s_raw, q_raw, o_raw, dc, rest = [t.to(cuda_device) for t in scene_params(sc)]
    acts = [xyz.clone().requires_grad_(True), torch.exp(s_raw).requires_grad_(True),
            torch.nn.functional.normalize(q_raw).requires_grad_(True), torch.cat((dc, rest), 1).requires_grad_(True),
            torch.sigmoid(o_raw).requires_grad_(True)]
    rast = RZ.GaussianRasterizer(rs)
    m2, rgb, co, radii, depths = rast.preprocess_gaussians(*acts[:4], acts[4], {})
    m2.retain_grad()
    rgb.retain_grad()
    co.retain_grad()
    H, W = cam.image_height, cam.image_width
    cl = torch.ones(((H + 15) // 16, (W + 15) // 16), dtype=torch.bool, device=cuda_device)
    abs_pts = torch.zeros_like(acts[0], requires_grad=True) + 0
    abs_pts.retain_grad()
    color, *_ = rast.render_gaussians(m2, abs_pts, co, rgb, torch.zeros((xyz.shape[0], 5), device=cuda_device),
                                      depths, radii, cl, None, {})
    from blitzgs_b200.loss import band_loss
    l1, ss = band_loss(color, gt)
    n3 = H * W * 3
    loss = 0.8 * l1 / n3 + 0.2 * (1 - ss / n3)
    assert abs(loss.item() - float(g["loss"])) <= 1e-6
    loss.backward()
    pairs = [("g_means2D", m2.grad), ("g_conic_opacity", co.grad), ("g_rgb", rgb.grad), ("g_means2D_abs", abs_pts.grad),
             ("g_means3D", acts[0].grad), ("g_scales", acts[1].grad), ("g_rotations", acts[2].grad),
             ("g_shs", acts[3].grad), ("g_opacities", acts[4].grad)]
    for name, t in pairs:
        assert_grad_close(t.cpu(), torch.from_numpy(g[name]), GRAD_RTOL, name)


# ---- the full rasterizer (golden_full.npz, tests/golden/make_golden_full.py) ----

def test_full_rasterizer_matches_reference_golden(cuda_device):
    """GaussianRasterizer.forward (flag_max_count), render_simp and
    markVisible against the reference's outputs: lists, ranges, n_contrib,
    final T, radii and the counts bit-exact; images within 1e-5; with
    precomputed colours, the gradients within 1e-4 (normwise)."""
    from tests.golden.make_golden_full import activated_inputs, full_scene, input_checksum, settings
    g = _load("golden_full.npz")
    dev = cuda_device
    sc, cam, culling, weight, colors = full_scene()
    assert str(g["checksum"]) == input_checksum(sc, cam, culling, weight, colors)
    inp = activated_inputs(sc, dev)
    cull = culling.to(dev)
    rast = RZ.GaussianRasterizer(settings(RZ, cam, dev))
    x = {k: v.clone().requires_grad_(True) for k, v in inp.items()}
    color, radii, amc = rast(x["means3D"], torch.zeros_like(inp["means3D"], requires_grad=True), x["opacities"],
                             cull, dc=x["dc"], shs=x["shs"], scales=x["scales"], rotations=x["rotations"],
                             flag_max_count=True)
    st = color.grad_fn.state
    R = len(g["point_list"])
    assert np.array_equal(radii.cpu().numpy(), g["radii"])
    assert np.array_equal(st.ranges.cpu().numpy(), g["ranges"])
    assert np.array_equal(st.point_list[:R].cpu().numpy(), g["point_list"])
    assert np.array_equal(st.n_contrib.cpu().numpy(), g["n_contrib"])
    assert np.array_equal(st.final_T.cpu().numpy().view(np.uint32), g["final_T"].view(np.uint32))
    assert np.abs(color.detach().cpu().numpy() - g["image"]).max() <= IMG_ATOL
    assert np.array_equal(amc.cpu().numpy(), g["accum_max_count"])
    with torch.no_grad():
        _, _, acc_w, acc_n, acc_m = rast.render_simp(inp["means3D"], torch.zeros_like(inp["means3D"]),
                                                     inp["opacities"], cull, dc=inp["dc"], shs=inp["shs"],
                                                     scales=inp["scales"], rotations=inp["rotations"])
        vis = rast.markVisible(inp["means3D"] * 3.0)
    assert np.array_equal(acc_n.cpu().numpy(), g["accum_weights_count"])
    assert np.array_equal(acc_m.cpu().numpy(), g["accum_max_count"])
    w = g["accum_weights_ptr"]
    assert np.abs(acc_w.cpu().numpy() - w).max() <= 1e-5 * max(1.0, float(np.abs(w).max()))
    assert np.array_equal(vis.cpu().numpy(), g["mark_visible"])
    # precomputed colours: image and gradients
    y = {k: inp[k].clone().requires_grad_(True) for k in ("means3D", "opacities", "scales", "rotations")}
    y["means2D"] = torch.zeros_like(inp["means3D"], requires_grad=True)
    y["colors_precomp"] = colors.to(dev).requires_grad_(True)
    color_pc, _, _ = rast(y["means3D"], y["means2D"], y["opacities"], cull, colors_precomp=y["colors_precomp"],
                          scales=y["scales"], rotations=y["rotations"])
    assert np.abs(color_pc.detach().cpu().numpy() - g["image_precomp"]).max() <= IMG_ATOL
    (color_pc * weight.to(dev)).sum().backward()
    for k in ("means3D", "means2D", "opacities", "scales", "rotations", "colors_precomp"):
        assert_grad_close(y[k].grad.cpu(), torch.from_numpy(g["grad_" + k]), GRAD_RTOL, k)
