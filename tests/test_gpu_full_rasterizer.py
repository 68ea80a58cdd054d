"""The full (non-distributed) rasterizer against the REFERENCE's, run live on
the same GPU: GaussianRasterizer.forward (with flag_max_count), render_simp,
render_depth and markVisible of diff_gaussian_rasterization_f
(f/__init__.py:666-810 -> _C.rasterize_gaussians / _simp / _depth /
mark_visible), built unmodified from the reference sources into oracle/_ref.

Both sides get the same activated parameters, a culling mask that drops ~10 %
of the Gaussians, and a non-zero background.

Bit-exact: radii, the per-tile Gaussian lists and tile ranges (binned over
each Gaussian's float rectangle with the exact tile test), the per-pixel
contributor counts and final transmittance, accum_max_count,
accum_weights_count, markVisible.
Within tolerance: images within 1e-5 absolute (IMG_ATOL); accum_weights_ptr
within 1e-5 relative (float atomics in both); gradients within 1e-4
relative, normwise (GRAD_RTOL).  render_depth: gidx equal on all but 1e-4 of
the pixels; where gidx agrees, depth and out_pts within 5e-4 relative,
normwise, and the sign of the discriminant on 99.9 % of the pixels where it
is not near zero.  Each pixel's ray comes from
the inverse of the projection matrix, which is ill-conditioned in its depth
row (znear 0.01); both invert it in float, in different orders, and the
two rays differ by ~1e-4 relative; the discriminant b^2 - 4ac cancels and
amplifies that by orders of magnitude for distant cameras.

The reference's backward of this path is run with precomputed colours only.
With SH colours it writes the DC gradient through a null pointer:
Rasterizer::backward passes nullptr for dL_ddc to BACKWARD::preprocess
(f/cuda_rasterizer/rasterizer_impl.cu:933-955) and computeColorFromSH
stores dL_ddirect_color[0] = dL_ddc + idx unconditionally (backward.cu:
45-50), an illegal address for every visible Gaussian.  So the gradients of
means3D, means2D, opacities, scales, rotations and colors_precomp are
compared with precomputed colours; with SH colours the forward (lists,
image, counts) is compared, and the SH part of this backward is the
training path's, pinned against the reference's training backward elsewhere.
"""
import pytest
import torch

from blitzgs_b200 import rasterizer as RZ, scene as S
from tests import ref_runner as REF
from tests.helpers import GRAD_RTOL, IMG_ATOL, normwise_rel

pytestmark = pytest.mark.gpu

if not REF.available():
    pytest.skip("reference build oracle/_ref absent (python oracle/build_ref.py)", allow_module_level=True)


def _case(name):
    if name == "tiny":
        return S.tiny(seed=0), 0
    if name == "tiny_side":
        sc = S.tiny(seed=5, P=30000)
        sc.cameras.append(S.look_at_camera([2.4, -1.0, -1.6], [0.1, 0, 0], [0, -1, 0], 320, 200, 1.1, uid=1))
        return sc, 1
    sc = S.mid(seed=2, P=300_000, n_cams=1)
    return sc, 0


def _inputs(sc, dev, seed):
    g = torch.Generator().manual_seed(seed)
    P = sc.xyz.shape[0]
    culling = (torch.rand(P, generator=g) < 0.1).to(dev)
    return dict(means3D=sc.xyz.to(dev), scales=torch.exp(sc.scaling).to(dev),
                rotations=torch.nn.functional.normalize(sc.rotation).to(dev),
                opacities=torch.sigmoid(sc.opacity).to(dev), dc=sc.features_dc.to(dev).contiguous(),
                shs=sc.features_rest.to(dev).contiguous(), culling=culling)


def _settings(pkg, cam, dev):
    return pkg.GaussianRasterizationSettings(
        image_height=int(cam.image_height), image_width=int(cam.image_width), tanfovx=cam.tanfovx,
        tanfovy=cam.tanfovy, bg=torch.tensor([0.1, 0.25, 0.4], device=dev), scale_modifier=1.0,
        viewmatrix=cam.world_view_transform.to(dev), projmatrix=cam.full_proj_transform.to(dev), sh_degree=3,
        campos=cam.camera_center.to(dev), prefiltered=False, debug=False)


def _ref_pkg():
    ref, _ = REF._modules()
    return ref


def _leaves(inp):
    out = {k: (v.clone().requires_grad_(True) if k != "culling" else v) for k, v in inp.items()}
    out["means2D"] = torch.zeros_like(inp["means3D"], requires_grad=True)
    return out


def _run_forward(rast, x, flag, colors=None):
    if colors is not None:
        return rast(x["means3D"], x["means2D"], x["opacities"], x["culling"], colors_precomp=colors,
                    scales=x["scales"], rotations=x["rotations"], flag_max_count=flag)
    return rast(x["means3D"], x["means2D"], x["opacities"], x["culling"], dc=x["dc"], shs=x["shs"],
                scales=x["scales"], rotations=x["rotations"], flag_max_count=flag)


def _ref_lists(color_ref, H, W):
    """point_list, ranges, final_T, n_contrib of the reference forward, from
    the autograd node's saved buffers (f/cuda_rasterizer/rasterizer_impl.cu:
    288-300, 319-331: 128-byte aligned consecutive arrays; the image buffer
    starts with accum_alpha f32[N], n_contrib u32[N], ranges uint2[N]; the
    binning buffer with point_list u32[num_rendered])."""
    saved = color_ref.grad_fn.saved_tensors
    binning_buf, img_buf = saved[9], saved[10]
    N = H * W
    T = ((W + 15) // 16) * ((H + 15) // 16)
    al = lambda x: (x + 127) // 128 * 128  # noqa: E731
    o1 = al(4 * N)
    o2 = al(o1 + 4 * N)
    final_T = img_buf[: 4 * N].view(torch.float32)
    n_contrib = img_buf[o1:o1 + 4 * N].view(torch.int32)
    ranges = img_buf[o2:o2 + 8 * T].view(torch.int32).reshape(T, 2)
    R = int(ranges[:, 1].max().item()) if T else 0
    return binning_buf[: 4 * R].view(torch.int32), ranges, final_T, n_contrib


def _compare_forward(st, pl_ref, rg_ref, fT_ref, nc_ref, c_our, c_ref, r_our, r_ref, m_our, m_ref, culling, flag):
    assert torch.equal(r_our, r_ref), f"radii differ at {int((r_our != r_ref).sum())} Gaussians"
    assert int((r_ref > 0).sum()) > 1000
    assert not (r_ref[culling] != 0).any(), "culled Gaussians kept a radius"
    assert torch.equal(st.ranges, rg_ref), "tile ranges differ"
    assert torch.equal(st.point_list[: pl_ref.numel()], pl_ref), "per-tile Gaussian lists differ"
    assert torch.equal(st.n_contrib, nc_ref), "per-pixel contributor counts differ"
    assert torch.equal(st.final_T, fT_ref), "final transmittance differs"
    err = (c_our - c_ref).abs().max().item()
    assert err <= IMG_ATOL, f"image max abs error {err}"
    if flag:
        assert torch.equal(m_our, m_ref), "accum_max_count differs"
        assert m_ref.sum().item() > 0
    else:
        assert not m_our.any()


@pytest.mark.parametrize("case", ["tiny", "tiny_side", "mid300k"])
@pytest.mark.parametrize("flag", [False, True])
def test_sh_forward_matches_reference(cuda_device, case, flag):
    """SH colours: the whole forward state, bit for bit (no reference backward)."""
    dev = cuda_device
    sc, ci = _case(case)
    cam = sc.cameras[ci]
    H, W = int(cam.image_height), int(cam.image_width)
    inp = _inputs(sc, dev, seed=11)
    ref = _ref_pkg()
    xr = _leaves(inp)
    c_ref, r_ref, m_ref = _run_forward(ref.GaussianRasterizer(_settings(ref, cam, dev)), xr, flag)
    pl_ref, rg_ref, fT_ref, nc_ref = (t.clone() for t in _ref_lists(c_ref, H, W))
    c_ref = c_ref.detach().clone()
    xo = _leaves(inp)
    c_our, r_our, m_our = _run_forward(RZ.GaussianRasterizer(_settings(RZ, cam, dev)), xo, flag)
    st = c_our.grad_fn.state
    torch.cuda.synchronize()
    _compare_forward(st, pl_ref, rg_ref, fT_ref, nc_ref, c_our.detach(), c_ref, r_our, r_ref, m_our, m_ref,
                     inp["culling"], flag)


@pytest.mark.parametrize("case", ["tiny", "tiny_side", "mid300k"])
def test_forward_and_gradients_match_reference(cuda_device, case):
    """Precomputed colours: forward state and the gradients of every input."""
    dev = cuda_device
    sc, ci = _case(case)
    cam = sc.cameras[ci]
    H, W = int(cam.image_height), int(cam.image_width)
    inp = _inputs(sc, dev, seed=11)
    colors = torch.rand((sc.xyz.shape[0], 3), generator=torch.Generator().manual_seed(5)).to(dev)
    weight = torch.rand((3, H, W), generator=torch.Generator().manual_seed(3)).to(dev)
    ref = _ref_pkg()

    xr = _leaves(inp)
    cr = colors.clone().requires_grad_(True)
    c_ref, r_ref, m_ref = _run_forward(ref.GaussianRasterizer(_settings(ref, cam, dev)), xr, True, cr)
    pl_ref, rg_ref, fT_ref, nc_ref = (t.clone() for t in _ref_lists(c_ref, H, W))
    (c_ref * weight).sum().backward()
    xo = _leaves(inp)
    co = colors.clone().requires_grad_(True)
    c_our, r_our, m_our = _run_forward(RZ.GaussianRasterizer(_settings(RZ, cam, dev)), xo, True, co)
    st = c_our.grad_fn.state
    (c_our * weight).sum().backward()
    torch.cuda.synchronize()
    _compare_forward(st, pl_ref, rg_ref, fT_ref, nc_ref, c_our.detach(), c_ref.detach(), r_our, r_ref, m_our, m_ref,
                     inp["culling"], True)
    grads = [(k, xo[k].grad, xr[k].grad) for k in ("means3D", "means2D", "opacities", "scales", "rotations")]
    grads.append(("colors_precomp", co.grad, cr.grad))
    for k, a, b in grads:
        r = normwise_rel(a, b)
        assert r <= GRAD_RTOL, f"grad {k}: normwise relative error {r:.3e}"


@pytest.mark.parametrize("case", ["tiny", "mid300k"])
def test_render_simp_matches_reference(cuda_device, case):
    dev = cuda_device
    sc, ci = _case(case)
    cam = sc.cameras[ci]
    inp = _inputs(sc, dev, seed=12)
    ref = _ref_pkg()
    args = (inp["means3D"], torch.zeros_like(inp["means3D"]), inp["opacities"], inp["culling"])
    kw = dict(dc=inp["dc"], shs=inp["shs"], scales=inp["scales"], rotations=inp["rotations"])
    with torch.no_grad():
        out_ref = ref.GaussianRasterizer(_settings(ref, cam, dev)).render_simp(*args, **kw)
        out_our = RZ.GaussianRasterizer(_settings(RZ, cam, dev)).render_simp(*args, **kw)
    torch.cuda.synchronize()
    c_ref, r_ref, w_ref, n_ref, m_ref = out_ref
    c_our, r_our, w_our, n_our, m_our = out_our
    assert torch.equal(r_our, r_ref)
    assert (c_our - c_ref).abs().max().item() <= IMG_ATOL
    assert n_ref.dtype == n_our.dtype == torch.int32 and torch.equal(n_our, n_ref), "accum_weights_count differs"
    assert torch.equal(m_our, m_ref), "accum_max_count differs"
    assert int(n_ref.sum()) > 0
    rel = ((w_our - w_ref).abs() / w_ref.abs().clamp_min(1e-12)).max().item()
    assert rel <= 1e-5, f"accum_weights_ptr max relative error {rel:.3e}"


@pytest.mark.parametrize("case", ["tiny", "mid300k"])
def test_render_depth_matches_reference(cuda_device, case):
    dev = cuda_device
    sc, ci = _case(case)
    cam = sc.cameras[ci]
    inp = _inputs(sc, dev, seed=13)
    ref = _ref_pkg()
    args = (inp["means3D"], torch.zeros_like(inp["means3D"]), inp["opacities"], inp["culling"])
    kw = dict(dc=inp["dc"], shs=inp["shs"], scales=inp["scales"], rotations=inp["rotations"])
    with torch.no_grad():
        d_ref = ref.GaussianRasterizer(_settings(ref, cam, dev)).render_depth(*args, **kw)
        d_our = RZ.GaussianRasterizer(_settings(RZ, cam, dev)).render_depth(*args, **kw)
    torch.cuda.synchronize()
    assert set(d_our) == set(d_ref)
    for k in d_ref:
        assert d_our[k].shape == d_ref[k].shape and d_our[k].dtype == d_ref[k].dtype, k
    assert (d_our["render"] - d_ref["render"]).abs().max().item() <= IMG_ATOL
    same = d_our["gidx"] == d_ref["gidx"]
    assert same.float().mean().item() >= 1 - 1e-4, f"gidx differs on {int((~same).sum())} pixels"
    hit = same & (d_ref["gidx"] != 0)
    assert int(hit.sum()) > 100
    a, b = d_our["rendered_depth"][hit], d_ref["rendered_depth"][hit]
    assert normwise_rel(a, b) <= 5e-4, f"rendered_depth: normwise relative error {normwise_rel(a, b):.3e}"
    # the discriminant b^2 - 4ac cancels catastrophically for distant cameras
    # (the aerial case), so only its sign -- does the ray cross the 3-sigma
    # ellipsoid -- is compared where it is not close to zero
    a, b = d_our["discriminants"][hit], d_ref["discriminants"][hit]
    clear = b.abs() > 0.1 * b.abs().median()
    assert ((a > 0) == (b > 0))[clear].float().mean().item() >= 0.999
    pts_hit = hit.expand(3, -1, -1)
    assert normwise_rel(d_our["out_pts"][pts_hit], d_ref["out_pts"][pts_hit]) <= 5e-4
    same_a = (d_our["accum_alpha"] - d_ref["accum_alpha"]).abs().max().item()
    assert same_a <= IMG_ATOL, f"accum_alpha max abs error {same_a}"


def test_mark_visible_matches_reference(cuda_device):
    dev = cuda_device
    sc, ci = _case("tiny_side")
    cam = sc.cameras[ci]
    ref = _ref_pkg()
    x = sc.xyz.to(dev) * 3.0  # spread the points across the near plane
    v_ref = ref.GaussianRasterizer(_settings(ref, cam, dev)).markVisible(x)
    v_our = RZ.GaussianRasterizer(_settings(RZ, cam, dev)).markVisible(x)
    assert v_our.dtype == torch.bool and torch.equal(v_our, v_ref)
    assert 0 < int(v_ref.sum()) < x.shape[0]


def test_precomputed_colours_equal_the_sh_colours(cuda_device):
    """colors_precomp set to the preprocess's own SH colours renders the same
    image, and its gradient is the colour gradient the SH backward consumes."""
    dev = cuda_device
    sc, ci = _case("tiny")
    cam = sc.cameras[ci]
    inp = _inputs(sc, dev, seed=14)
    rs = _settings(RZ, cam, dev)
    rast = RZ.GaussianRasterizer(rs)
    H, W = rs.image_height, rs.image_width
    weight = torch.rand((3, H, W), generator=torch.Generator().manual_seed(4)).to(dev)
    x = _leaves(inp)
    color, radii, _ = rast(x["means3D"], x["means2D"], x["opacities"], x["culling"], dc=x["dc"], shs=x["shs"],
                           scales=x["scales"], rotations=x["rotations"])
    rgb = color.grad_fn.saved_tensors[6]
    colors = rgb.detach().clone().requires_grad_(True)
    y = _leaves(inp)
    color2, radii2, _ = rast(y["means3D"], y["means2D"], y["opacities"], y["culling"], colors_precomp=colors,
                             scales=y["scales"], rotations=y["rotations"])
    assert torch.equal(radii2, radii) and torch.equal(color2, color)
    (color2 * weight).sum().backward()
    (color * weight).sum().backward()
    assert colors.grad is not None and colors.grad.abs().sum() > 0
    # the geometric gradients do not depend on where the colour came from,
    # except for the SH view-direction term that precomputed colours drop
    assert normwise_rel(y["opacities"].grad, x["opacities"].grad) <= GRAD_RTOL
    assert normwise_rel(y["scales"].grad, x["scales"].grad) <= GRAD_RTOL
