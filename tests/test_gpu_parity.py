"""CUDA path vs the CPU oracle on identical seeded inputs, stage by stage.

Each stage is fed the GPU's own upstream outputs, so the comparison isolates
that stage: binning is integer work and must match exactly; float stages are
compared with the tolerances of tests/helpers.py.  Calls go through the C ABI
(blitzgs_b200.ops wraps libblitzgs_b200.so with ctypes).
"""
import numpy as np
import pytest
import torch

from blitzgs_b200 import _lib, ops, rasterizer as RZ, scene as S, step as ST
from oracle import rasterizer_oracle as O
from tests.helpers import GRAD_RTOL, IMG_ATOL, activated, assert_grad_close, normwise_rel, scene_params

pytestmark = pytest.mark.gpu


def _raster(cam, dev, bg=None):
    return S.raster_settings(cam, device=dev, bg=bg)


def _gpu_preprocess(sc, cam, dev):
    xyz, s, q, shs, o = activated(sc, dev)
    rs = _raster(cam, dev)
    sh = ops.sh_layout(shs=shs)
    m2, d, r, co, rgb, _, cl = ops.preprocess_forward(xyz, s, q, o.reshape(-1), sh, rs, want_clamped=True)
    return dict(means2D=m2, depths=d, radii=r, conic_opacity=co, rgb=rgb, clamped=cl), rs


def _oracle_preprocess(sc, cam):
    xyz, s, q, shs, o = activated(sc)
    return O.preprocess_forward(xyz, s, q, shs, o, cam.world_view_transform, cam.full_proj_transform,
                                cam.camera_center, cam.tanfovx, cam.tanfovy, cam.image_height, cam.image_width, 3)


@pytest.fixture(scope="module")
def tiny(cuda_device):
    sc = S.tiny()
    cam = sc.cameras[0]
    g, rs = _gpu_preprocess(sc, cam, cuda_device)
    return sc, cam, g, rs


def test_preprocess_forward_matches_oracle(tiny):
    sc, cam, g, _ = tiny
    o = _oracle_preprocess(sc, cam)
    gr = g["radii"].cpu()
    mism = int((gr != o["radii"]).sum())
    assert mism == 0, f"radii differ at {mism} Gaussians"
    both = (gr > 0) & (o["radii"] > 0)
    assert torch.allclose(g["means2D"].cpu()[both], o["means2D"][both], atol=1e-5, rtol=0)
    assert torch.allclose(g["depths"].cpu()[both], o["depths"][both], rtol=1e-6, atol=1e-6)
    assert normwise_rel(g["conic_opacity"].cpu()[both], o["conic_opacity"][both]) < 1e-5
    assert torch.allclose(g["rgb"].cpu()[both], o["rgb"][both], atol=1e-6)
    assert torch.equal(g["clamped"].cpu()[both], o["clamped"][both])
    # culled Gaussians have all-zero outputs
    z = gr == 0
    assert torch.all(g["conic_opacity"].cpu()[z] == 0) and torch.all(g["means2D"].cpu()[z] == 0)


def test_binning_exact(tiny):
    sc, cam, g, rs = tiny
    H, W = cam.image_height, cam.image_width
    color, nr, nc, nct, obs, st = ops.render_forward(g["means2D"], g["depths"], g["radii"], g["conic_opacity"],
                                                     g["rgb"], rs.bg, None, H, W)
    pl, ranges, counts = O.binning(g["means2D"].cpu().numpy(), g["depths"].cpu().numpy(), g["radii"].cpu().numpy(),
                                   H, W)
    assert st.R == len(pl)
    assert np.array_equal(st.point_list[: st.R].cpu().numpy().astype(np.int64), pl)
    assert np.array_equal(st.ranges.cpu().numpy().astype(np.int64), ranges)
    assert np.array_equal(nr.cpu().numpy(), ranges[:, 1] - ranges[:, 0])


def _render_inputs(g):
    return g["means2D"].cpu(), g["conic_opacity"].cpu(), g["rgb"].cpu()


def test_render_forward_matches_oracle(tiny):
    sc, cam, g, rs = tiny
    H, W = cam.image_height, cam.image_width
    color, nr, nc, nct, obs, st = ops.render_forward(g["means2D"], g["depths"], g["radii"], g["conic_opacity"],
                                                     g["rgb"], rs.bg, None, H, W)
    m2, co, rgb = _render_inputs(g)
    pl = st.point_list[: st.R].cpu().numpy().astype(np.int64)
    ranges = st.ranges.cpu().numpy().astype(np.int64)
    f = O.render_forward(m2, co, rgb, torch.zeros(3), pl, ranges, H, W)
    assert float((color.cpu() - f["color"]).abs().max()) <= IMG_ATOL
    assert np.array_equal(st.n_contrib.cpu().numpy(), f["n_contrib"].numpy())
    assert float((st.final_T.cpu() - f["final_T"]).abs().max()) <= 1e-5
    assert np.array_equal(obs.cpu().numpy(), f["out_observe"].numpy())
    assert np.array_equal(nc.cpu().numpy(), f["n_consider"].numpy())


def test_render_backward_matches_oracle(tiny):
    sc, cam, g, rs = tiny
    H, W = cam.image_height, cam.image_width
    color, nr, nc, nct, obs, st = ops.render_forward(g["means2D"], g["depths"], g["radii"], g["conic_opacity"],
                                                     g["rgb"], rs.bg, None, H, W)
    gen = torch.Generator().manual_seed(5)
    dpix = torch.randn(3, H, W, generator=gen) * 1e-3
    rec = ops.render_backward(st, g["means2D"], g["conic_opacity"], g["rgb"], rs.bg, None, dpix.to(color.device))
    m2, co, rgb = _render_inputs(g)
    pl = st.point_list[: st.R].cpu().numpy().astype(np.int64)
    ranges = st.ranges.cpu().numpy().astype(np.int64)
    orec = O.render_backward(m2, co, rgb, torch.zeros(3), pl, ranges, H, W, dpix)
    rec = rec.cpu()
    for name, sl in (("means2D", slice(0, 2)), ("means2D_abs", slice(4, 6)), ("conic", slice(8, 11)),
                     ("opacity", slice(11, 12)), ("rgb", slice(12, 15))):
        r = normwise_rel(rec[:, sl], orec[:, sl])
        assert r <= GRAD_RTOL, f"{name}: {r}"
    assert torch.all(rec[:, [2, 3, 6, 7, 15]] == 0)


def test_loss_matches_oracle(cuda_device):
    gen = torch.Generator().manual_seed(3)
    img = torch.rand(3, 70, 93, generator=gen)
    gt = torch.randint(0, 256, (3, 70, 93), generator=gen, dtype=torch.uint8)
    sums, partials = ops.loss_forward(img.to(cuda_device), gt.to(cuda_device))
    l1, ss = O.band_loss_sums(img, gt)
    assert abs(sums[0].item() - l1.item()) <= 1e-5 * abs(l1.item())
    assert abs(sums[1].item() - ss.item()) <= 1e-4 * max(1.0, abs(ss.item()))
    scale = torch.tensor([0.7, -0.3], device=cuda_device)
    g = ops.loss_backward(img.to(cuda_device), gt.to(cuda_device), partials, scale).cpu()
    x = img.clone().requires_grad_(True)
    a, b = O.band_loss_sums(x, gt)
    (0.7 * a - 0.3 * b).backward()
    assert_grad_close(g, x.grad, 1e-4, "dL/dimg")


def test_full_step_gradients_match_oracle(cuda_device):
    sc = S.tiny(seed=2, P=4096, H=128, W=160)
    cam = sc.cameras[0]
    gt = S.target_image(2, cam.image_height, cam.image_width)
    ref = O.train_step(scene_params(sc), cam, gt)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    rs = _raster(cam.to(cuda_device), cuda_device)
    loss, l1, ss, radii, obs, color = ST.view_loss(model, rs, gt.to(cuda_device), scale_reg_weight=0.0)
    loss.backward()
    assert abs(loss.item() - ref["loss"].item()) <= 1e-6 * abs(ref["loss"].item())
    assert float((color.detach().cpu() - ref["fwd"]["color"]).abs().max()) <= IMG_ATOL
    names = ["xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"]
    for n, p, r in zip(names, model, ref["grads"]):
        assert_grad_close(p.grad.cpu(), r, GRAD_RTOL, n)


def test_fused_regulariser_matches_oracle(cuda_device):
    sc = S.tiny(seed=9, P=3000, H=96, W=128)
    cam = sc.cameras[0]
    gt = S.target_image(9, cam.image_height, cam.image_width)
    ref = O.train_step(scene_params(sc), cam, gt, reg_weight=10.0)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    rs = _raster(cam.to(cuda_device), cuda_device)
    loss, *_ = ST.view_loss(model, rs, gt.to(cuda_device), scale_reg_weight=10.0)
    loss.backward()
    assert abs(loss.item() - ref["loss"].item()) <= 1e-6 * abs(ref["loss"].item())
    for n, p, r in zip(["xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"], model, ref["grads"]):
        assert_grad_close(p.grad.cpu(), r, GRAD_RTOL, n)


@pytest.mark.parametrize("with_reg", [False, True])
def test_device_loss_combination_bit_identical_to_torch(cuda_device, with_reg):
    """blitz_loss_combine and its backward against the same expression on
    0-dim float32 tensors and PyTorch's autograd of it, bit for bit, over
    seeded sums (the step used to form the loss that way)."""
    gen = torch.Generator().manual_seed(12)
    lam, w, n3 = 0.2, 10.0, 864 * 1152 * 3
    for _ in range(50):
        sums = (torch.rand(2, generator=gen, dtype=torch.float64) * torch.tensor([n3 * 0.3, n3])).to(cuda_device)
        reg = torch.tensor([float(torch.rand(1, generator=gen)) * 5e3, float(torch.randint(0, 9, (1,), generator=gen))],
                           dtype=torch.float64, device=cuda_device)
        g_up = [torch.randn((), generator=gen).to(cuda_device) for _ in range(3)]
        out = ops.loss_combine(sums, reg if with_reg else None, lam, n3, w)
        scales = ops.loss_combine_backward(g_up[0], g_up[1], g_up[2], out, lam, n3, w if with_reg else 0.0)
        l1 = sums[0].to(torch.float32).requires_grad_(True)
        ss = sums[1].to(torch.float32).requires_grad_(True)
        r = reg[0].to(torch.float32).requires_grad_(True)
        cnt = reg[1].to(torch.float32)
        loss = (1.0 - lam) * (l1 / n3) + lam * (1.0 - ss / n3)
        if with_reg:
            loss = loss + w * r / cnt.clamp(min=1.0)
        assert torch.equal(out[0], loss.detach()) and torch.equal(out[1], l1.detach()) and torch.equal(out[2], ss.detach())
        torch.autograd.backward([loss, l1, ss], [g_up[0], g_up[1], g_up[2]])
        assert torch.equal(scales[0], l1.grad) and torch.equal(scales[1], ss.grad)
        if with_reg:
            assert torch.equal(scales[2], r.grad)


def test_raw_preprocess_bit_identical_to_torch_activations(cuda_device):
    """Activations fused into the kernel (exp, sigmoid, division by PyTorch's
    rotation norm) give the same bits as the operator API fed with PyTorch's
    exp / normalize / sigmoid, so the fused step culls and bins exactly as the
    reference pipeline does."""
    sc = S.tiny(seed=10, P=20000, H=96, W=128)
    cam = sc.cameras[0].to(cuda_device)
    rs = _raster(cam, cuda_device)
    xyz, s, q, o, dc, rest = [t.to(cuda_device) for t in scene_params(sc)]
    a = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), ops.sh_layout(dc=dc, rest=rest), rs, q.norm(dim=1),
                                   want_list=False)
    shs = torch.cat((dc, rest), 1)
    b = ops.preprocess_forward(xyz, torch.exp(s), torch.nn.functional.normalize(q), torch.sigmoid(o).reshape(-1),
                               ops.sh_layout(shs=shs), rs)
    for x, y in zip(a[:5], b[:5]):
        assert torch.equal(x, y)


def test_in_kernel_rotation_norm_is_bit_identical_to_torch(cuda_device):
    """The fused step normalises _rotation in the kernel; its norm must equal
    PyTorch's norm bit for bit, or radii could differ from the reference's."""
    g = torch.Generator().manual_seed(77)
    sc = S.tiny(seed=12, P=200000, H=96, W=128)
    sc.rotation = torch.randn(200000, 4, generator=g) * torch.rand(200000, 1, generator=g) * 3
    cam = sc.cameras[0].to(cuda_device)
    rs = _raster(cam, cuda_device)
    xyz, s, q, o, dc, rest = [t.to(cuda_device) for t in scene_params(sc)]
    sh = ops.sh_layout(dc=dc, rest=rest)
    a = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, q.norm(dim=1), want_list=False)
    b = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, None, want_list=False)
    for x, y in zip(a[:5], b[:5]):
        assert torch.equal(x, y)


def _separate_count(m2, r, cl, H, W):
    P = m2.shape[0]
    counts = torch.empty((P,), dtype=torch.int32, device=m2.device)
    totals = torch.empty((2,), dtype=torch.int64, device=m2.device)
    mask = None if cl is None else cl.contiguous().view(-1)
    _lib.call("blitz_render_count", P, H, W, ops.ptr(m2), ops.ptr(r), ops.ptr(mask), ops.ptr(counts), ops.ptr(totals),
              _lib.stream_ptr())
    return counts, totals


@pytest.mark.parametrize("two_pass", [True, False], ids=["cull+full", "one-kernel"])
@pytest.mark.parametrize("case", ["mid_full", "mid_masked", "huge_grid_masked"])
def test_fused_count_and_listed_rows_match_separate_passes(cuda_device, case, two_pass):
    """The fused step's preprocess writes radii for every Gaussian, full rows
    only for the listed ones (radius > 0), and the binning's tile counts under
    the tile mask.  All of it must equal the dense preprocess followed by the
    separate count pass.  1.5M Gaussians take several chunks per persistent
    block, so survivors carried from one chunk to the next are covered; the
    4112x2048 image has more tiles than the kernel stages in shared memory."""
    if case == "huge_grid_masked":
        sc = S.tiny(seed=21, P=300000, H=2048, W=4112)
    else:
        sc = S.mid(seed=3, P=1_500_000, n_cams=1)
    cam = sc.cameras[0].to(cuda_device)
    rs = _raster(cam, cuda_device)
    H, W = cam.image_height, cam.image_width
    gx, gy = ops.grid_dims(H, W)
    cl = None
    if case != "mid_full":
        g = torch.Generator().manual_seed(5)
        cl = (torch.rand(gy, gx, generator=g) < 0.6).to(cuda_device)
    xyz, s, q, o, dc, rest = [t.to(cuda_device) for t in scene_params(sc)]
    sh = ops.sh_layout(dc=dc, rest=rest)
    dense = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, None, want_list=False, two_pass=False)
    fused = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, None, want_list=True, want_counts=True,
                                       compute_locally=cl, two_pass=two_pass)
    assert torch.equal(dense[2], fused[2])  # radii, every Gaussian
    n = int(fused[7].item())
    listed = fused[6][:n].long()
    assert n > 1000
    assert torch.equal(torch.sort(listed).values, torch.nonzero(dense[2] > 0).flatten())
    for a, b in zip(dense[:5], fused[:5]):
        assert torch.equal(a[listed], b[listed])
    assert torch.equal(dense[5], fused[5])  or torch.allclose(dense[5], fused[5], rtol=1e-12)  # regulariser sums
    counts, totals = _separate_count(dense[0], dense[2], cl, H, W)
    assert torch.equal(counts, fused[8])
    assert torch.equal(totals, fused[9])


@pytest.mark.parametrize("scene", ["tiny", "mid"])
def test_sparse_gradients_equal_dense_rows(cuda_device, scene):
    """sparse_grad=True returns the same gradient as the dense path: the
    listed rows hold the values the dense path scatters, and the dense path is
    zero everywhere else.  (Not bit for bit: the render backward sums each
    Gaussian's record with float atomics, whose order varies run to run.)
    torch.optim.SparseAdam accepts it."""
    sc = S.tiny(seed=9, P=20000, H=128, W=160) if scene == "tiny" else S.mid(seed=2, P=600_000, n_cams=1)
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(2, cam.image_height, cam.image_width).to(cuda_device)
    rs = _raster(cam, cuda_device)
    grads = []
    for sparse in (False, True):
        model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
        loss, *_ = ST.view_loss(model, rs, gt, sparse_grad=sparse)
        loss.backward()
        grads.append([p.grad for p in model])
        if sparse:
            assert all(p.grad.is_sparse for p in model)
            opt = torch.optim.SparseAdam(model, lr=1e-3)
            opt.step()
    for n, d, sp in zip(["xyz", "scaling", "rotation", "opacity", "dc", "rest"], *grads):
        sd = sp.to_dense()
        assert normwise_rel(sd.cpu(), d.cpu()) < 1e-5, n
        rows = sp.coalesce().indices()[0]
        assert rows.numel() > 0
        outside = torch.ones(d.shape[0], dtype=torch.bool, device=d.device)
        outside[rows] = False
        assert not d[outside].any(), n  # the dense gradient is zero off the listed rows


def test_drop_in_api_autograd_matches_fused(cuda_device):
    """GaussianRasterizer.preprocess_gaussians/render_gaussians (reference API)
    give the same loss and parameter gradients as the fused step."""
    sc = S.tiny(seed=4, P=4096, H=96, W=128)
    cam = sc.cameras[0].to(cuda_device)
    gt = S.target_image(4, cam.image_height, cam.image_width).to(cuda_device)
    rs = _raster(cam, cuda_device)
    model = [t.to(cuda_device).requires_grad_(True) for t in scene_params(sc)]
    loss_f, *_ = ST.view_loss(model, rs, gt, scale_reg_weight=0.0)
    loss_f.backward()
    fused = [p.grad.clone() for p in model]
    for p in model:
        p.grad = None
    xyz, s_raw, q_raw, o_raw, dc, rest = model
    rast = RZ.GaussianRasterizer(rs)
    ca = {"avoid_pixel_all2all": False, "stats_collector": {}}
    m2, rgb, co, radii, depths = rast.preprocess_gaussians(xyz, torch.exp(s_raw), torch.nn.functional.normalize(q_raw),
                                                           torch.cat((dc, rest), 1), torch.sigmoid(o_raw), ca)
    m2.retain_grad()
    H, W = cam.image_height, cam.image_width
    cl = torch.ones(((H + 15) // 16, (W + 15) // 16), dtype=torch.bool, device=cuda_device)
    abs_pts = torch.zeros_like(xyz, requires_grad=True) + 0
    abs_pts.retain_grad()
    color, nr, nc, nct, obs, _, _ = rast.render_gaussians(m2, abs_pts, co, rgb, torch.zeros((xyz.shape[0], 5),
                                                          device=cuda_device), depths, radii, cl, None, ca)
    sums, _ = O.band_loss_sums(color.cpu(), gt.cpu())
    from blitzgs_b200.loss import band_loss
    l1, ss = band_loss(color, gt)
    n3 = H * W * 3
    loss = 0.8 * l1 / n3 + 0.2 * (1 - ss / n3)
    loss.backward()
    assert abs(loss.item() - loss_f.item()) < 1e-6
    for a, b in zip(model, fused):
        assert_grad_close(a.grad, b, 1e-5)
    assert "forward_render_time" in ca["stats_collector"] and "backward_render_time" in ca["stats_collector"]
    assert m2.grad is not None and abs_pts.grad is not None


def test_band_compute_locally(cuda_device):
    sc = S.tiny(seed=6, P=3000, H=120, W=184)
    cam = sc.cameras[0]
    g, rs = _gpu_preprocess(sc, cam, cuda_device)
    H, W = cam.image_height, cam.image_width
    gx, gy = (W + 15) // 16, (H + 15) // 16
    band = torch.zeros((gy, gx), dtype=torch.bool)
    band[2:5] = True
    color, nr, nc, nct, obs, st = ops.render_forward(g["means2D"], g["depths"], g["radii"], g["conic_opacity"],
                                                     g["rgb"], rs.bg, band.to(cuda_device), H, W)
    pl, ranges, counts = O.binning(g["means2D"].cpu().numpy(), g["depths"].cpu().numpy(), g["radii"].cpu().numpy(),
                                   H, W, band.numpy())
    assert np.array_equal(st.point_list[: st.R].cpu().numpy().astype(np.int64), pl)
    assert np.array_equal(st.ranges.cpu().numpy().astype(np.int64), ranges)
    c = color.cpu()
    assert torch.all(c[:, :32] == 0) and torch.all(c[:, 80:] == 0)
    assert torch.all(nr.cpu().view(gy, gx)[~band] == 0)
    m2, co, rgb = _render_inputs(g)
    f = O.render_forward(m2, co, rgb, torch.zeros(3), pl, ranges, H, W, band.numpy())
    assert float((c - f["color"]).abs().max()) <= IMG_ATOL


@pytest.mark.parametrize("banded", [False, True])
def test_strip_lists_replay_the_same_pairs(cuda_device, banded):
    """The forward's per-strip contributor lists (strip_lists=True) leave the
    forward outputs bit-identical, list every Gaussian that contributed to a
    pixel of the strip exactly once in list order, and give the backward the
    same gradient record as the full list walk (up to atomic ordering)."""
    sc = S.mid(seed=3, P=200_000, n_cams=1, H=216, W=296)
    cam = sc.cameras[0]
    g, rs = _gpu_preprocess(sc, cam, cuda_device)
    H, W = cam.image_height, cam.image_width
    gx, gy = (W + 15) // 16, (H + 15) // 16
    cl = None
    if banded:
        band = torch.zeros((gy, gx), dtype=torch.bool)
        band[3:9] = True
        cl = band.to(cuda_device)
    args = (g["means2D"], g["depths"], g["radii"], g["conic_opacity"], g["rgb"], rs.bg, cl, H, W)
    out_w = ops.render_forward(*args, strip_lists=False)
    out_l = ops.render_forward(*args, strip_lists=True)
    for a, b in zip(out_w[:5], out_l[:5]):
        assert torch.equal(a, b)
    st = out_l[5]
    assert st.strip_ids is not None and out_w[5].strip_ids is None
    # lists are increasing positions of the tile list, each entry the Gaussian at that position
    cnt = st.strip_counts.cpu().view(-1, 8)
    ranges = st.ranges.cpu().numpy().astype(np.int64)
    ids, pos, pl = st.strip_ids.cpu().numpy(), st.strip_pos.cpu().numpy(), st.point_list.cpu().numpy()
    tiles = range(gx * gy) if cl is None else np.nonzero(band.view(-1).numpy())[0]
    checked = 0
    for t in list(tiles)[:: max(1, len(tiles) // 40)]:
        lo, hi = ranges[t]
        for s in range(8):
            n = int(cnt[t, s])
            off = 8 * lo + s * (hi - lo)
            p_ = pos[off:off + n]
            assert n <= hi - lo and np.all(np.diff(p_) > 0) and np.all(p_ < hi - lo)
            assert np.array_equal(ids[off:off + n], pl[lo + p_])
            checked += n
    assert checked > 0
    dL = torch.randn(3, H, W, generator=torch.Generator().manual_seed(4)).to(cuda_device)
    rec_w = ops.render_backward(out_w[5], g["means2D"], g["conic_opacity"], g["rgb"], rs.bg, cl, dL)
    rec_l = ops.render_backward(st, g["means2D"], g["conic_opacity"], g["rgb"], rs.bg, cl, dL)
    assert normwise_rel(rec_l.cpu(), rec_w.cpu()) < 1e-5


def test_edge_cases(cuda_device):
    dev = cuda_device
    sc = S.tiny(seed=7, P=64, H=40, W=56)
    cam = sc.cameras[0]
    rs = _raster(cam, dev)
    # P = 0
    e = torch.zeros((0, 3), device=dev)
    m2, d, r, co, rgb, _, _ = ops.preprocess_forward(e, e, torch.zeros((0, 4), device=dev), torch.zeros((0,), device=dev),
                                                     ops.sh_layout(shs=torch.zeros((0, 16, 3), device=dev)), rs)
    assert m2.shape == (0, 2)
    color, nr, *_rest, st = ops.render_forward(m2, d, r, co, rgb, rs.bg, None, 40, 56)
    assert st.R == 0 and torch.all(color == 0)
    # everything behind the camera: nothing rendered, image = background
    sc.xyz[:] = torch.tensor([0.0, 0.0, -3.5])
    g, rs = _gpu_preprocess(sc, cam, dev)
    assert int((g["radii"] > 0).sum()) == 0
    bg = torch.tensor([0.25, 0.5, 1.0], device=dev)
    color, nr, nc, nct, obs, st = ops.render_forward(g["means2D"], g["depths"], g["radii"], g["conic_opacity"],
                                                     g["rgb"], bg, None, 40, 56)
    assert st.R == 0
    assert torch.allclose(color, bg.view(3, 1, 1).expand(3, 40, 56))


def test_ops_refuse_cpu_tensors():
    sc = S.tiny(seed=8, P=16, H=32, W=32)
    rs = S.raster_settings(sc.cameras[0])
    xyz, s, q, shs, o = activated(sc)
    with pytest.raises(RuntimeError):
        ops.preprocess_forward(xyz, s, q, o.reshape(-1), ops.sh_layout(shs=shs), rs)


def test_exchange_records_routing_and_pack(cuda_device):
    """The fused exchange outputs of the raw preprocess (records, destination
    masks, per-rank counts) equal what the operator API gives: the same
    per-Gaussian outputs and get_local2j_ids_bool on the reference's tile
    intervals, here for 4 ranks.  blitz_exchange_pack then puts every routed
    row exactly once into each destination's segment, in list order."""
    sc = S.mid(seed=4, P=400_000, n_cams=1)
    cam = sc.cameras[0].to(cuda_device)
    rs = _raster(cam, cuda_device)
    H, W = cam.image_height, cam.image_width
    gx, gy = ops.grid_dims(H, W)
    division = [0, 11, 23, 40, gy]
    ranks = len(division) - 1
    lo = torch.tensor([d * gx for d in division[:-1]], dtype=torch.int32, device=cuda_device)
    hi = torch.tensor([d * gx for d in division[1:]], dtype=torch.int32, device=cuda_device)
    xyz, s, q, o, dc, rest = [t.to(cuda_device) for t in scene_params(sc)]
    sh = ops.sh_layout(dc=dc, rest=rest)
    P = xyz.shape[0]
    rec = torch.empty((P, 12), dtype=torch.float32, device=cuda_device)
    mask = torch.empty((P,), dtype=torch.int32, device=cuda_device)
    cnt = torch.zeros((ranks,), dtype=torch.int32, device=cuda_device)
    out = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, None, want_list=True,
                                     exchange=(lo, hi, rec, mask, cnt))
    dense = ops.preprocess_forward_raw(xyz, s, q, o.reshape(-1), sh, rs, None, want_list=False, two_pass=False)
    m2, d, r, co, rgb = dense[:5]
    L = int(out[7].item())
    ids = out[6][:L].long()
    assert L > 1000
    # the two-kernel preprocess lists the visible Gaussians in ascending index order
    assert bool((ids[1:] > ids[:-1]).all())
    assert torch.equal(ids, torch.nonzero(dense[2] > 0).flatten())
    route = ops.local2j_ids_bool(H, W, 0, ranks, m2, r, torch.tensor(division, dtype=torch.int32,
                                                                       device=cuda_device) * gx)
    assert not route[r <= 0].any()  # only listed Gaussians are ever sent
    smin = torch.exp(s).min(dim=1).values
    want = torch.cat([co[ids], m2[ids], rgb[ids], d[ids, None], r[ids].view(torch.float32)[:, None],
                      smin[ids, None]], 1)
    assert torch.equal(rec[:L].view(torch.int32), want.view(torch.int32))
    bits = torch.stack([(mask[:L] >> k) & 1 for k in range(ranks)], 1).bool()
    assert torch.equal(bits, route[ids])
    assert torch.equal(cnt.long(), bits.sum(0))
    # pack: segment k of the send buffer holds exactly the rows routed to rank k
    counts = cnt.tolist()
    offs = [sum(counts[:k]) for k in range(ranks)]
    n_send = sum(counts)
    send = torch.empty((n_send, 12), dtype=torch.float32, device=cuda_device)
    send_row = torch.empty((n_send,), dtype=torch.int32, device=cuda_device)
    ops.exchange_pack(L, rec, mask, offs, send, send_row, 7)
    for k in range(ranks):
        # each segment keeps the list order: the routed rows in ascending order
        rows = send_row[offs[k]:offs[k] + counts[k]].long() - 7
        assert torch.equal(rows, torch.nonzero(bits[:, k]).flatten())
        assert torch.equal(send[offs[k]:offs[k] + counts[k]], rec[rows])
    st = ops.queue_scan_status(cuda_device)
    torch.cuda.synchronize()
    ops.check_scan_status(st)


def test_exchange_unpack_and_gradient_pack(cuda_device):
    """blitz_exchange_unpack splits received records (several runs, in order)
    exactly like slicing them, with the min-scale sum/count over rows of
    radius > 0; blitz_grad_records_pack writes the 12-float gradient records
    at the runs' rows."""
    gen = torch.Generator().manual_seed(21)
    rows = torch.randn(500, 12, generator=gen)
    rad = torch.randint(-2, 30, (500,), generator=gen).to(torch.int32)
    rows[:, 10] = rad.view(torch.float32)
    recs = rows.to(cuda_device)
    segs = [(7, 40), (100, 0), (200, 123), (400, 61)]
    sel = torch.cat([rows[s:s + c] for s, c in segs if c])
    reg = torch.zeros(2, dtype=torch.float64, device=cuda_device)
    conic, m2, rgb, depth, radii = ops.exchange_unpack(recs, segs, reg)
    assert torch.equal(conic.cpu(), sel[:, 0:4]) and torch.equal(m2.cpu(), sel[:, 4:6])
    assert torch.equal(rgb.cpu(), sel[:, 6:9]) and torch.equal(depth.cpu(), sel[:, 9])
    assert torch.equal(radii.cpu(), sel[:, 10].contiguous().view(torch.int32))
    vis = radii.cpu() > 0
    assert reg[1].item() == vis.sum().item()
    assert abs(reg[0].item() - sel[vis, 11].double().sum().item()) < 1e-9
    n = sel.shape[0]
    rec16 = torch.randn(n, 16, generator=gen).to(cuda_device)
    scale = torch.tensor([0.37], device=cuda_device)
    send = torch.full((700, 12), -7.0, device=cuda_device)
    dst = [(0, 40), (300, 123), (600, 61)]
    ops.grad_records_pack(rec16, radii, scale, dst, send)
    r = rec16.cpu()
    want = torch.cat([r[:, 8:12], r[:, 0:2], r[:, 12:15], r[:, 4:6],
                      torch.where(vis, torch.tensor(0.37), torch.tensor(0.0))[:, None]], 1)
    got = send.cpu()
    assert torch.equal(got[0:40], want[0:40]) and torch.equal(got[300:423], want[40:163])
    assert torch.equal(got[600:661], want[163:224])
    assert torch.all(got[40:300] == -7.0) and torch.all(got[423:600] == -7.0)


def test_preprocess_backward_matches_finite_differences(cuda_device):
    """The preprocess backward against central differences of the preprocess
    forward kernel itself.  Every Gaussian is independent, so one parameter
    component of all Gaussians is perturbed at once and each Gaussian's own
    scalar L_i = <ndc_i, g_m> + <conic_i, g_c (x2 off-diagonal)> +
    <rgb_i, g_rgb> is differenced.  Float32 forward outputs and a step of
    1e-3 (relative for scales) bound the agreement at ~1e-3 normwise."""
    dev = cuda_device
    sc = S.tiny(seed=4, P=600, H=96, W=128)
    cam = sc.cameras[0]
    rs = _raster(cam.to(dev), dev)
    xyz, s, q, shs, o = [t.to(dev) for t in activated(sc)]
    o = o.reshape(-1)
    P = xyz.shape[0]
    gen = torch.Generator().manual_seed(8)
    gm = torch.randn(P, 2, generator=gen).to(dev)
    gc = torch.randn(P, 4, generator=gen).to(dev)
    gr = torch.randn(P, 3, generator=gen).to(dev)
    w3 = torch.tensor([1.0, 2.0, 1.0], dtype=torch.float64, device=dev)
    # the screen-mean gradient of the operator contract is per NDC unit
    # (pixel = (ndc + 1) W / 2 - 1/2): weight pixels by 2/W and 2/H
    w2 = torch.tensor([2.0 / cam.image_width, 2.0 / cam.image_height], dtype=torch.float64, device=dev)

    def fwd(xyz_, s_, q_, shs_):
        m2, d, r, co, rgb, _, cl = ops.preprocess_forward(xyz_, s_, q_, o, ops.sh_layout(shs=shs_), rs,
                                                          want_clamped=True)
        L = ((m2.double() * gm.double() * w2).sum(1) + (co[:, :3].double() * gc[:, :3].double() * w3).sum(1) +
             (rgb.double() * gr.double()).sum(1))
        return L, r, cl

    L0, r0, cl0 = fwd(xyz, s, q, shs)
    dm, ds, dq, _, dsh = ops.preprocess_backward(r0, xyz, s, q, ops.sh_layout(shs=shs), rs, gm, gc, gr)
    keep = r0 > 0
    # outside +-1.3 tan(fov) the operator contract holds the clamped centre
    # constant (not the derivative of the clamp): leave those out
    t = torch.cat([xyz, torch.ones(P, 1, device=dev)], 1) @ rs.viewmatrix
    keep &= ((t[:, 0] / t[:, 2]).abs() < 0.99 * 1.3 * rs.tanfovx) & ((t[:, 1] / t[:, 2]).abs() < 0.99 * 1.3 * rs.tanfovy)
    analytic, numeric = [], []
    for which, base, grad, rel in (("xyz", xyz, dm, False), ("scale", s, ds, True), ("rot", q, dq, False),
                                   ("sh", shs.reshape(P, -1), dsh.reshape(P, -1), False)):
        for c in range(base.shape[1]):
            step = (1e-3 * base[:, c].abs()) if rel else torch.full((P,), 1e-3, device=dev)
            outs = []
            for sign in (1.0, -1.0):
                pert = base.clone()
                pert[:, c] += sign * step
                if which == "xyz":
                    args = (pert, s, q, shs)
                elif which == "scale":
                    args = (xyz, pert, q, shs)
                elif which == "rot":
                    args = (xyz, s, pert, shs)
                else:
                    args = (xyz, s, q, pert.reshape(shs.shape))
                L, r, cl = fwd(*args)
                outs.append(L)
                # a Gaussian that crosses the cull or a colour clamp is not differentiable there
                keep &= (r > 0) & (cl == cl0).all(1)
            numeric.append((outs[0] - outs[1]) / (2.0 * step.double()))
            analytic.append(grad[:, c].double())
    A = torch.stack(analytic, 1)[keep]
    N = torch.stack(numeric, 1)[keep]
    assert keep.sum() > 100
    err = normwise_rel(A.cpu(), N.cpu())
    assert err <= 2e-3, f"finite differences: normwise relative error {err:.3e}"
