"""Drop-in replacement of the ``diff_gaussian_rasterization_f`` operator API.

Mirrors submodule/diff-gaussian-rasterization_f/diff_gaussian_rasterization_f/
__init__.py of the reference: the ``GaussianRasterizationSettings`` named
tuple (:647-659), ``GaussianRasterizer`` (:661-829) with
``preprocess_gaussians`` / ``render_gaussians``, the autograd functions
``_PreprocessGaussians`` (:75-173) and ``_RenderGaussians`` (:204-318), and a
``_C`` namespace exposing the native ops the Python layer calls directly
(``preprocess_gaussians[_backward]``, ``render_gaussians[_backward]``,
``get_local2j_ids_bool``) with the reference's positional signatures and
return tuples.  Everything runs on the sm_100a kernels of libblitzgs_b200.so;
there is no CPU path.

Gradient conventions are the reference's: the means2D gradient is with
respect to NDC-scaled screen position (dL/dpixel * W/2, H/2), the conic
off-diagonal gradient is half the derivative with respect to the stored entry,
and the alpha clamp at 0.99 is ignored in the backward.
"""
from types import SimpleNamespace
from typing import NamedTuple

import torch
import torch.nn as nn

from . import ops


class GaussianRasterizationSettings(NamedTuple):
    image_height: int
    image_width: int
    tanfovx: float
    tanfovy: float
    bg: torch.Tensor
    scale_modifier: float
    viewmatrix: torch.Tensor
    projmatrix: torch.Tensor
    sh_degree: int
    campos: torch.Tensor
    prefiltered: bool
    debug: bool


def _settings(scale_modifier, viewmatrix, projmatrix, tanfovx, tanfovy, H, W, degree, campos,
              prefiltered):
    return SimpleNamespace(scale_modifier=scale_modifier, viewmatrix=viewmatrix.contiguous(),
                           projmatrix=projmatrix.contiguous(), tanfovx=tanfovx, tanfovy=tanfovy,
                           image_height=H, image_width=W, sh_degree=degree,
                           campos=campos.contiguous(), prefiltered=prefiltered)


def _check_error_word(word, debug, prefiltered):
    if word is None:
        return
    if debug or prefiltered:
        v = int(word.item())
        if v & 1:
            raise RuntimeError("Point is filtered although prefiltered is set. This shouldn't happen!")


# ---------------------------------------------------------------------------
# Native-op namespace with the reference's _C signatures
# ---------------------------------------------------------------------------

def _preprocess_gaussians(means3D, scales, rotations, sh, opacity, scale_modifier, viewmatrix,
                          projmatrix, tan_fovx, tan_fovy, image_height, image_width, degree, campos,
                          prefiltered, debug, args=None):
    """Reference: PreprocessGaussiansCUDA (f/rasterize_points.cu:834-923)."""
    if means3D.ndimension() != 2 or means3D.size(1) != 3:
        raise RuntimeError("means3D must have dimensions (num_points, 3)")
    P = means3D.shape[0]
    st = _settings(scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height,
                   image_width, degree, campos, prefiltered)
    dev = means3D.device
    if P == 0 or sh.size(0) == 0:
        z = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt, device=dev)
        return (0, z(P, 2), z(P), z(P, dt=torch.int32), z(P, 6), z(P, 4), z(P, 3), z(P, 3, dt=torch.bool))
    layout = ops.sh_layout(shs=sh)
    word = torch.zeros(1, dtype=torch.int32, device=dev) if (prefiltered or debug) else None
    means2D, depths, radii, conic, rgb, cov3D, clamped = ops.preprocess_forward(
        means3D, scales, rotations, opacity.reshape(-1), layout, st, want_cov3D=True,
        want_clamped=True, error_word=word)
    _check_error_word(word, debug, prefiltered)
    if debug:
        torch.cuda.synchronize()
    return 0, means2D, depths, radii, cov3D, conic, rgb, clamped


def _preprocess_gaussians_backward(radii, cov3D, clamped, means3D, scales, rotations, sh,
                                   scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy,
                                   image_height, image_width, degree, campos, dL_dmeans2D,
                                   dL_dconic_opacity, dL_dcolors, R=0, debug=False, args=None):
    """Reference: PreprocessGaussiansBackwardCUDA (f/rasterize_points.cu:926-1029).

    cov3D and clamped are accepted for signature compatibility; the kernel
    recomputes both from the parameters (bit-identical to the forward's)."""
    st = _settings(scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height,
                   image_width, degree, campos, False)
    layout = ops.sh_layout(shs=sh)
    gm = dL_dmeans2D.contiguous()
    gc = dL_dconic_opacity.contiguous()
    gcol = dL_dcolors.contiguous()
    dmeans3D, dscales, drot, dop, dsh = ops.preprocess_backward(
        radii.contiguous(), means3D.contiguous(), scales.contiguous(), rotations.contiguous(), layout,
        st, gm, gc, gcol)
    if debug:
        torch.cuda.synchronize()
    return dmeans3D, dscales, drot, dsh, dop


def _pack_img_state(state):
    """ranges, final_T and n_contrib in one int32 buffer (the reference's imgBuffer role)."""
    return torch.cat([state.ranges.view(-1), state.final_T.view(torch.int32), state.n_contrib])


def _unpack_img_state(buf, H, W, R, point_list):
    gx, gy = ops.grid_dims(H, W)
    T = gx * gy
    HW = H * W
    ranges = buf[: 2 * T].view(T, 2)
    final_T = buf[2 * T: 2 * T + HW].view(torch.float32)
    n_contrib = buf[2 * T + HW: 2 * T + 2 * HW]
    return ops.RenderState(H, W, R, -1, point_list, ranges, final_T, n_contrib)


class _Timer:
    def __init__(self):
        self.a = torch.cuda.Event(enable_timing=True)
        self.b = torch.cuda.Event(enable_timing=True)

    def start(self):
        self.a.record()

    def stop(self):
        self.b.record()

    def ms(self):
        self.b.synchronize()
        return self.a.elapsed_time(self.b)


def _stats(args):
    if isinstance(args, dict):
        sc = args.get("stats_collector")
        if isinstance(sc, dict):
            return sc
    return None


def _render_gaussians(background, image_height, image_width, means2D, depths, radii, conic_opacity,
                      rgb, compute_locally, viewmatrix=None, campos=None, tan_fovx=None, tan_fovy=None,
                      all_map=None, render_geo=False, debug=False, args=None):
    """Reference: RenderGaussiansCUDA (r/rasterize_points.cu:274-361).

    Returns (num_rendered, color, n_render, n_consider, n_contrib, out_observe,
    out_all_map, out_plane_depth, geomBuffer, binningBuffer, imgBuffer); the
    three buffers hold this implementation's backward state."""
    if render_geo:
        raise NotImplementedError("render_geo (all-map / plane-depth rendering) is not on the training path")
    H, W = int(image_height), int(image_width)
    P = means2D.shape[0]
    dev = means2D.device
    sc = _stats(args)
    tm = _Timer() if sc is not None else None
    if tm:
        tm.start()
    color, n_render, n_consider, n_contrib, out_observe, state = ops.render_forward(
        means2D, depths, radii, conic_opacity, rgb, background, compute_locally, H, W)
    if tm:
        tm.stop()
        sc["_blitz_fwd_timer"] = tm
    out_all_map = torch.zeros((5, H, W), dtype=torch.float32, device=dev)
    out_plane_depth = torch.zeros((1, H, W), dtype=torch.float32, device=dev)
    geom = torch.empty((0,), dtype=torch.uint8, device=dev)
    img = _pack_img_state(state)
    if debug:
        torch.cuda.synchronize()
    return (state.R, color, n_render, n_consider, n_contrib, out_observe, out_all_map, out_plane_depth,
            geom, state.point_list, img)


def _render_gaussians_backward_record(background, R, binningBuffer, imageBuffer, compute_locally,
                                      dL_dout_color, means2D, conic_opacity, rgb, args=None):
    H, W = int(dL_dout_color.shape[1]), int(dL_dout_color.shape[2])
    state = _unpack_img_state(imageBuffer, H, W, R, binningBuffer)
    sc = _stats(args)
    tm = _Timer() if sc is not None else None
    if tm:
        tm.start()
    rec = ops.render_backward(state, means2D, conic_opacity, rgb, background, compute_locally,
                              dL_dout_color)
    if tm:
        tm.stop()
        sc["backward_render_time"] = tm.ms()
        fwd = sc.pop("_blitz_fwd_timer", None)
        if fwd is not None:
            sc["forward_render_time"] = fwd.ms()
    return rec


def _render_gaussians_backward(background, tan_fovx, tan_fovy, all_map_pixels, all_maps, R, geomBuffer,
                               binningBuffer, imageBuffer, compute_locally, dL_dout_color,
                               dL_dout_all_map, dL_dout_plane_depth, means2D, conic_opacity, rgb,
                               render_geo=False, debug=False, args=None):
    """Reference: RenderGaussiansBackwardCUDA (r/rasterize_points.cu:364-436).
    Returns (dL_dmeans2D [P,3], dL_dmeans2D_abs [P,3], dL_dconic_opacity [P,4],
    dL_dcolors [P,3], dL_dall_map [P,5])."""
    if render_geo:
        raise NotImplementedError("render_geo (all-map / plane-depth rendering) is not on the training path")
    rec = _render_gaussians_backward_record(background, R, binningBuffer, imageBuffer, compute_locally,
                                            dL_dout_color.contiguous(), means2D, conic_opacity, rgb, args)
    P = rec.shape[0]
    dmeans2D = rec[:, 0:3].contiguous()
    dmeans2D[:, 2] = 0
    dabs = rec[:, 4:7].contiguous()
    dall = torch.zeros((P, 5), dtype=torch.float32, device=rec.device)
    if debug:
        torch.cuda.synchronize()
    return dmeans2D, dabs, rec[:, 8:12].contiguous(), rec[:, 12:15].contiguous(), dall


def _get_local2j_ids_bool(image_height, image_width, mp_rank, mp_world_size, means2D, radii,
                          dist_global_strategy, args=None):
    """Reference: GetLocal2jIdsBoolCUDA (f/rasterize_points.cu:258-288)."""
    avoid = bool(args.get("avoid_pixel_all2all", False)) if isinstance(args, dict) else False
    return ops.local2j_ids_bool(image_height, image_width, mp_rank, mp_world_size, means2D, radii,
                                dist_global_strategy, avoid)


def _get_local2j_ids_bool_adjust_mode6(image_height, image_width, mp_rank, mp_world_size, means2D, radii,
                                       rectangles, args=None):
    """Reference: GetLocal2jIdsBoolAdjustMode6CUDA (f/rasterize_points.cu:337-368)."""
    avoid = bool(args.get("avoid_pixel_all2all", False)) if isinstance(args, dict) else False
    return ops.local2j_ids_bool_adjust_mode6(image_height, image_width, mp_rank, mp_world_size, means2D, radii,
                                             rectangles, avoid)


def _adam_update(param, param_grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps, N, M):
    """Reference: adamUpdate (f/rasterize_points.cu:807-833): in place, no return."""
    ops.adam_update(param, param_grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps, N, M)


def _full_sh(dc, sh, colors_precomp, P, dev):
    """SH layout of the full rasterizer's inputs: ``dc`` [P,1,3] and ``sh``
    [P,M,3] (the coefficients beyond DC), or ``sh`` alone holding all of
    them; with precomputed colours a zero DC stands in (its colour is not
    used)."""
    if colors_precomp is not None and colors_precomp.numel():
        return ops.sh_layout(shs=torch.zeros((P, 1, 3), dtype=torch.float32, device=dev)), 0
    if dc is None or dc.numel() == 0:
        return ops.sh_layout(shs=sh), None
    rest = sh if sh is not None and sh.numel() else torch.zeros((P, 0, 3), dtype=torch.float32, device=dev)
    return ops.sh_layout(dc=dc, rest=rest), None


def _full_forward(background, means3D, colors, opacity, scales, rotations, scale_modifier, cov3D_precomp,
                  viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height, image_width, dc, sh, degree, campos,
                  prefiltered, culling, debug, *, max_count=False, simp=False, blend=True):
    """Preprocess + exact-test binning + blend of the full rasterizer.
    Returns (color, radii, stats, state, ctx) with ``state`` the render state
    (tile lists, final T, contributor counts) and ``ctx`` = (settings, SH
    layout, means2D, conic_opacity, rgb, bg) for a backward or a depth pass."""
    if means3D.ndimension() != 2 or means3D.size(1) != 3:
        raise RuntimeError("means3D must have dimensions (num_points, 3)")
    if cov3D_precomp is not None and cov3D_precomp.numel():
        raise NotImplementedError("precomputed 3D covariances are not supported (scales and rotations only)")
    P = means3D.shape[0]
    dev = means3D.device
    H, W = int(image_height), int(image_width)
    layout, deg = _full_sh(dc, sh, colors, P, dev)
    st = _settings(scale_modifier, viewmatrix, projmatrix, tan_fovx, tan_fovy, H, W,
                   degree if deg is None else deg, campos, prefiltered)
    word = torch.zeros(1, dtype=torch.int32, device=dev) if (prefiltered or debug) else None
    cull = culling if culling is not None and culling.numel() else None
    m2, depths, radii, conic, rgb, _, _, rects = ops.preprocess_forward(
        means3D, scales, rotations, opacity.reshape(-1), layout, st, error_word=word, culling=cull, want_rects=True)
    _check_error_word(word, debug, prefiltered)
    if colors is not None and colors.numel():
        rgb = colors.reshape(P, 3).float().contiguous()
    bg = background.float().contiguous()
    color, state, stats = ops.rasterize_forward(m2, depths, radii, rects, conic, rgb, bg, H, W, max_count=max_count,
                                                simp=simp, blend=blend)
    if debug:
        torch.cuda.synchronize()
    return color, radii, stats, state, (st, layout, m2, conic, rgb, bg)


def _rasterize_gaussians_simp(background, means3D, colors, opacity, scales, rotations, scale_modifier,
                              cov3D_precomp, viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height, image_width,
                              dc, sh, degree, campos, prefiltered, culling, debug):
    """Reference: RasterizeGaussiansSimpCUDA (f/rasterize_points.cu:479-585).
    Returns (num_rendered, color, accum_weights_ptr, accum_weights_count,
    accum_max_count, radii, geomBuffer, binningBuffer, imgBuffer); the three
    buffers are empty (no backward follows)."""
    color, radii, stats, state, _ = _full_forward(
        background, means3D, colors, opacity, scales, rotations, scale_modifier, cov3D_precomp, viewmatrix,
        projmatrix, tan_fovx, tan_fovy, image_height, image_width, dc, sh, degree, campos, prefiltered, culling,
        debug, simp=True)
    e = torch.empty((0,), dtype=torch.uint8, device=means3D.device)
    return (state.R, color, stats["accum_weights"], stats["accum_count"], stats["max_count"], radii, e, e, e)


def _rasterize_gaussians_depth(background, means3D, colors, opacity, scales, rotations, scale_modifier,
                               cov3D_precomp, viewmatrix, projmatrix, tan_fovx, tan_fovy, image_height, image_width,
                               dc, sh, degree, campos, prefiltered, culling, debug):
    """Reference: RasterizeGaussiansDepthCUDA (f/rasterize_points.cu:588-700).
    Returns (num_rendered, color, out_pts, depth, accum_alpha, gidx,
    discriminants, radii, geomBuffer, binningBuffer, imgBuffer); the buffers
    are empty."""
    _, radii, _, state, (st, _, m2, conic, rgb, bg) = _full_forward(
        background, means3D, colors, opacity, scales, rotations, scale_modifier, cov3D_precomp, viewmatrix,
        projmatrix, tan_fovx, tan_fovy, image_height, image_width, dc, sh, degree, campos, prefiltered, culling,
        debug, blend=False)
    color, pts, depth, alpha, gidx, disc = ops.rasterize_depth(m2, conic, rgb, bg, state, means3D, scales,
                                                               rotations, st)
    e = torch.empty((0,), dtype=torch.uint8, device=means3D.device)
    return (state.R, color, pts, depth, alpha, gidx, disc, radii, e, e, e)


def _mark_visible(means3D, viewmatrix, projmatrix):
    """Reference: markVisible (f/rasterize_points.cu:785-804)."""
    return ops.mark_visible(means3D, viewmatrix, projmatrix)


_C = SimpleNamespace(
    rasterize_gaussians_simp=_rasterize_gaussians_simp,
    rasterize_gaussians_depth=_rasterize_gaussians_depth,
    mark_visible=_mark_visible,
    preprocess_gaussians=_preprocess_gaussians,
    preprocess_gaussians_backward=_preprocess_gaussians_backward,
    render_gaussians=_render_gaussians,
    render_gaussians_backward=_render_gaussians_backward,
    get_local2j_ids_bool=_get_local2j_ids_bool,
    get_local2j_ids_bool_adjust_mode6=_get_local2j_ids_bool_adjust_mode6,
    adamUpdate=_adam_update,
)


class SparseGaussianAdam(torch.optim.Adam):
    """The reference's SparseGaussianAdam (f/diff_gaussian_rasterization_f/
    __init__.py:830-863): one parameter tensor per group; ``step(visibility,
    N)`` updates only the Gaussians marked visible, with the bias corrections
    folded into the learning rate ``lr * sqrt(1 - 0.999^t) / (1 - 0.9^t)``.

    Also takes the sparse COO gradients of ``step.view_loss(sparse_grad=True)``:
    their rows are the Gaussians with radius > 0 -- the visibility the
    reference passes -- and only those rows are read and written."""

    def __init__(self, params, lr, eps):
        super().__init__(params=params, lr=lr, eps=eps)

    @torch.no_grad()
    def step(self, visibility=None, N=None, bsz=None):
        """``bsz``: divide the gradients by the batch size inside the update
        (the trainer's ``param.grad /= bsz``, train_internal.py:504-515,
        fused; the same float32 result) instead of beforehand."""
        scale = None
        if bsz is not None:
            import numpy as np
            scale = float(np.float32(1.0) / np.float32(bsz))  # PyTorch divides by a host scalar this way
        for group in self.param_groups:
            lr = group["lr"]
            eps = group["eps"]
            assert len(group["params"]) == 1, "more than one tensor in group"
            param = group["params"][0]
            if param.grad is None or param.grad.numel() == 0:
                continue
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(param, memory_format=torch.preserve_format)
            exp_avg, exp_avg_sq = state["exp_avg"], state["exp_avg_sq"]
            state["step"] += 1
            step = state["step"]
            lr_t = lr * (1 - 0.999 ** step) ** 0.5 / (1 - 0.9 ** step)
            n = N if N is not None else param.shape[0]
            M = param.numel() // n
            g = param.grad
            if g.is_sparse:
                g = g.coalesce()
                rows = g.indices()[0]
                ops.adam_update_rows(param, g.values().reshape(rows.numel(), M), exp_avg, exp_avg_sq, rows,
                                     float(lr_t), 0.9, 0.999, eps, n, M, grad_scale=1.0 if scale is None else scale)
            else:
                if scale is not None:
                    g = g * scale
                _C.adamUpdate(param, g, exp_avg, exp_avg_sq, visibility, float(lr_t), 0.9, 0.999, eps, n, M)


# ---------------------------------------------------------------------------
# Autograd functions and module (reference f/__init__.py:55-318, 647-829)
# ---------------------------------------------------------------------------

def preprocess_gaussians(means3D, scales, rotations, sh, opacities, raster_settings, cuda_args):
    return _PreprocessGaussians.apply(means3D, scales, rotations, sh, opacities, raster_settings, cuda_args)


class _PreprocessGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means3D, scales, rotations, sh, opacities, raster_settings, cuda_args):
        rs = raster_settings
        num_rendered, means2D, depths, radii, cov3D, conic_opacity, rgb, clamped = _C.preprocess_gaussians(
            means3D, scales, rotations, sh, opacities, rs.scale_modifier, rs.viewmatrix, rs.projmatrix,
            rs.tanfovx, rs.tanfovy, rs.image_height, rs.image_width, rs.sh_degree, rs.campos,
            rs.prefiltered, rs.debug, cuda_args)
        ctx.raster_settings = rs
        ctx.cuda_args = cuda_args
        ctx.num_rendered = num_rendered
        ctx.save_for_backward(means3D, scales, rotations, sh, radii)
        ctx.mark_non_differentiable(radii, depths)
        return means2D, rgb, conic_opacity, radii, depths

    @staticmethod
    def backward(ctx, grad_means2D, grad_rgb, grad_conic_opacity, grad_radii, grad_depths):
        rs = ctx.raster_settings
        means3D, scales, rotations, sh, radii = ctx.saved_tensors
        P = means3D.shape[0]
        dev = means3D.device
        if grad_means2D is None:
            grad_means2D = torch.zeros((P, 2), dtype=torch.float32, device=dev)
        if grad_rgb is None:
            grad_rgb = torch.zeros((P, 3), dtype=torch.float32, device=dev)
        if grad_conic_opacity is None:
            grad_conic_opacity = torch.zeros((P, 4), dtype=torch.float32, device=dev)
        st = _settings(rs.scale_modifier, rs.viewmatrix, rs.projmatrix, rs.tanfovx, rs.tanfovy,
                       rs.image_height, rs.image_width, rs.sh_degree, rs.campos, False)
        layout = ops.sh_layout(shs=sh)
        gm = grad_means2D if grad_means2D.stride(-1) == 1 else grad_means2D.contiguous()
        gc = grad_conic_opacity if (grad_conic_opacity.stride(-1) == 1 and grad_conic_opacity.stride(0) % 4 == 0
                                    and grad_conic_opacity.data_ptr() % 16 == 0) else grad_conic_opacity.contiguous()
        gcol = grad_rgb if grad_rgb.stride(-1) == 1 else grad_rgb.contiguous()
        dmeans3D, dscales, drot, dop, dsh = ops.preprocess_backward(
            radii, means3D, scales, rotations, layout, st, gm, gc, gcol)
        return dmeans3D, dscales, drot, dsh, dop, None, None


def render_gaussians(means2D, means2D_abs, conic_opacity, rgb, all_map, depths, radii, compute_locally,
                     extended_compute_locally, raster_settings, cuda_args):
    return _RenderGaussians.apply(means2D, means2D_abs, conic_opacity, rgb, all_map, depths, radii,
                                  compute_locally, extended_compute_locally, raster_settings, cuda_args)


class _RenderGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2D, means2D_abs, conic_opacity, rgb, all_maps, depths, radii, compute_locally,
                extended_compute_locally, raster_settings, cuda_args):
        rs = raster_settings
        avoid = bool(cuda_args.get("avoid_pixel_all2all", False)) if isinstance(cuda_args, dict) else False
        cl = extended_compute_locally if avoid else compute_locally
        (num_rendered, color, n_render, n_consider, n_contrib, out_observe, out_all_map, out_plane_depth,
         geom, binning, img) = _C.render_gaussians(
            rs.bg, rs.image_height, rs.image_width, means2D, depths, radii, conic_opacity, rgb, cl,
            rs.viewmatrix, rs.campos, rs.tanfovx, rs.tanfovy, all_maps, getattr(rs, "render_geo", False),
            rs.debug, cuda_args)
        ctx.raster_settings = rs
        ctx.cuda_args = cuda_args
        ctx.num_rendered = num_rendered
        ctx.means2D_abs_shape = tuple(means2D_abs.shape) if means2D_abs is not None else None
        ctx.save_for_backward(means2D, conic_opacity, rgb, binning, img, cl if cl is not None else compute_locally)
        ctx.mark_non_differentiable(n_render, n_consider, n_contrib)
        return color, n_render, n_consider, n_contrib, out_observe, out_all_map, out_plane_depth

    @staticmethod
    def backward(ctx, grad_color, grad_n_render, grad_n_consider, grad_n_contrib, grad_out_observe,
                 grad_out_all_map, grad_out_plane_depth):
        rs = ctx.raster_settings
        means2D, conic_opacity, rgb, binning, img, cl = ctx.saved_tensors
        if grad_color is None:
            grad_color = torch.zeros((3, rs.image_height, rs.image_width), dtype=torch.float32,
                                     device=means2D.device)
        rec = _render_gaussians_backward_record(rs.bg, ctx.num_rendered, binning, img, cl,
                                                grad_color.contiguous(), means2D, conic_opacity, rgb,
                                                ctx.cuda_args)
        g_means2D = rec[:, 0:2]
        g_abs = None
        if ctx.needs_input_grad[1] and ctx.means2D_abs_shape is not None:
            g_abs = rec[:, 4:4 + ctx.means2D_abs_shape[1]]
        g_conic = rec[:, 8:12]
        g_rgb = rec[:, 12:15]
        return g_means2D, g_abs, g_conic, g_rgb, None, None, None, None, None, None, None


def _empty(t):
    return torch.Tensor([]) if t is None else t


def rasterize_gaussians(means3D, means2D, dc, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                        flag_max_count, culling, raster_settings):
    return _RasterizeGaussians.apply(means3D, means2D, _empty(dc), _empty(sh), _empty(colors_precomp), opacities,
                                     _empty(scales), _empty(rotations), _empty(cov3Ds_precomp), flag_max_count,
                                     culling, raster_settings)


def _simp_or_depth_args(means3D, dc, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp, culling,
                        rs):
    return (rs.bg, means3D, _empty(colors_precomp), opacities, _empty(scales), _empty(rotations), rs.scale_modifier,
            _empty(cov3Ds_precomp), rs.viewmatrix, rs.projmatrix, rs.tanfovx, rs.tanfovy, rs.image_height,
            rs.image_width, _empty(dc), _empty(sh), rs.sh_degree, rs.campos, rs.prefiltered, culling, rs.debug)


@torch.no_grad()
def rasterize_gaussians_simp(means3D, means2D, dc, sh, colors_precomp, opacities, scales, rotations,
                             cov3Ds_precomp, culling, raster_settings):
    """Reference: _RasterizeGaussians.render_simp (f/__init__.py:477-521)."""
    out = _C.rasterize_gaussians_simp(*_simp_or_depth_args(means3D, dc, sh, colors_precomp, opacities, scales,
                                                           rotations, cov3Ds_precomp, culling, raster_settings))
    _, color, accum_w, accum_n, accum_max, radii = out[:6]
    return color, radii, accum_w, accum_n, accum_max


@torch.no_grad()
def rasterize_gaussians_depth(means3D, means2D, dc, sh, colors_precomp, opacities, scales, rotations,
                              cov3Ds_precomp, culling, raster_settings):
    """Reference: _RasterizeGaussians.render_depth (f/__init__.py:525-579)."""
    out = _C.rasterize_gaussians_depth(*_simp_or_depth_args(means3D, dc, sh, colors_precomp, opacities, scales,
                                                            rotations, cov3Ds_precomp, culling, raster_settings))
    _, color, pts, depth, alpha, gidx, disc = out[:7]
    return {"render": color, "out_pts": pts, "rendered_depth": depth, "discriminants": disc, "gidx": gidx,
            "accum_alpha": alpha}


class _RasterizeGaussians(torch.autograd.Function):
    """Reference: _RasterizeGaussians (f/diff_gaussian_rasterization_f/
    __init__.py:412-644).  The backward replays the blend over the same tile
    lists (csrc/blend.cu) and runs the preprocess backward; the means2D
    gradient keeps the reference's NDC scaling."""

    @staticmethod
    def forward(ctx, means3D, means2D, dc, sh, colors_precomp, opacities, scales, rotations, cov3Ds_precomp,
                flag_max_count, culling, raster_settings):
        rs = raster_settings
        color, radii, stats, state, (st, layout, m2, conic, rgb, bg) = _full_forward(
            rs.bg, means3D, colors_precomp, opacities, scales, rotations, rs.scale_modifier, cov3Ds_precomp,
            rs.viewmatrix, rs.projmatrix, rs.tanfovx, rs.tanfovy, rs.image_height, rs.image_width, dc, sh,
            rs.sh_degree, rs.campos, rs.prefiltered, culling, rs.debug, max_count=bool(flag_max_count))
        accum_max_count = stats.get("max_count")
        if accum_max_count is None:
            accum_max_count = torch.zeros((means3D.shape[0],), dtype=torch.float32, device=means3D.device)
        ctx.st, ctx.layout, ctx.state = st, layout, state
        ctx.precomp = colors_precomp.numel() > 0
        ctx.shapes = (means2D.shape, dc.shape, sh.shape, opacities.shape)
        ctx.save_for_backward(means3D, scales, rotations, radii, m2, conic, rgb, bg)
        ctx.mark_non_differentiable(radii, accum_max_count)
        return color, radii, accum_max_count

    @staticmethod
    def backward(ctx, grad_color, *_):
        means3D, scales, rotations, radii, m2, conic, rgb, bg = ctx.saved_tensors
        st, layout, state = ctx.st, ctx.layout, ctx.state
        P = means3D.shape[0]
        dev = means3D.device
        m2_shape, dc_shape, sh_shape, op_shape = ctx.shapes
        rec = ops.render_backward(state, m2, conic, rgb, bg, None, grad_color.contiguous())
        g_colors = rec[:, 12:15]
        g_precomp = None
        if ctx.precomp:
            g_precomp = g_colors.contiguous()
            g_colors = torch.zeros((P, 3), dtype=torch.float32, device=dev)
        dmeans3D = torch.empty((P, 3), dtype=torch.float32, device=dev)
        dscales = torch.empty((P, 3), dtype=torch.float32, device=dev)
        drot = torch.empty((P, 4), dtype=torch.float32, device=dev)
        dop = torch.empty((P, 1), dtype=torch.float32, device=dev)
        dc_t, _dcs, rest_t, _rs, M, _keep = layout
        dsh = torch.empty((P, M + 1, 3), dtype=torch.float32, device=dev)
        ops.preprocess_backward(radii, means3D, scales, rotations, layout, st, rec[:, 0:2], rec[:, 8:12], g_colors,
                                out=(dmeans3D, dscales, drot, dop, (dsh, (M + 1) * 3),
                                     (dsh.view(-1)[3:] if M > 0 else dsh, (M + 1) * 3)))
        g_means2D = torch.zeros(m2_shape, dtype=torch.float32, device=dev)
        g_means2D[:, :2] = rec[:, 0:2]
        g_dc = g_sh = None
        if not ctx.precomp:
            if len(dc_shape) and dc_shape[0] == P:
                g_dc = dsh[:, :1].reshape(dc_shape)
                g_sh = dsh[:, 1:].reshape(sh_shape) if len(sh_shape) and sh_shape[0] == P else None
            else:
                g_sh = dsh.reshape(sh_shape)
        return (dmeans3D, g_means2D, g_dc, g_sh, g_precomp, dop.reshape(op_shape), dscales, drot, None, None, None,
                None)


class GaussianRasterizer(nn.Module):
    def __init__(self, raster_settings):
        super().__init__()
        self.raster_settings = raster_settings

    def preprocess_gaussians(self, means3D, scales, rotations, shs, opacities, cuda_args=None):
        return preprocess_gaussians(means3D, scales, rotations, shs, opacities, self.raster_settings, cuda_args)

    def render_gaussians(self, means2D, means2D_abs, conic_opacity, rgb, all_map, depths, radii,
                         compute_locally, extended_compute_locally, cuda_args=None):
        return render_gaussians(means2D, means2D_abs, conic_opacity, rgb, all_map, depths, radii,
                                compute_locally, extended_compute_locally, self.raster_settings, cuda_args)

    def markVisible(self, positions):
        """bool [P]: Gaussians in front of the camera (view depth > 0.2;
        f/__init__.py:666-675)."""
        with torch.no_grad():
            rs = self.raster_settings
            return _C.mark_visible(positions, rs.viewmatrix, rs.projmatrix)

    def _inputs(self, shs, colors_precomp, scales, rotations, cov3D_precomp):
        """The reference's argument checks (f/__init__.py:695-720)."""
        if (shs is None and colors_precomp is None) or (shs is not None and colors_precomp is not None):
            raise Exception('Please provide excatly one of either SHs or precomputed colors!')
        if ((scales is None or rotations is None) and cov3D_precomp is None) or \
                ((scales is not None or rotations is not None) and cov3D_precomp is not None):
            raise Exception('Please provide exactly one of either scale/rotation pair or precomputed 3D covariance!')

    def forward(self, means3D, means2D, opacities, culling=None, dc=None, shs=None, colors_precomp=None,
                scales=None, rotations=None, cov3D_precomp=None, flag_max_count=False):
        """The reference's full (non-distributed) rasterizer
        (f/diff_gaussian_rasterization_f/__init__.py:691-729 ->
        _RasterizeGaussians :412-474): one camera, the whole image, each
        Gaussian binned over its float screen rectangle restricted to the
        tiles that pass the exact tile test.  Returns (color [3,H,W], radii
        int32 [P], accum_max_count float [P]); with ``flag_max_count`` every
        pixel adds 1 to the count of its Gaussian of largest blending weight.
        Gradients reach means3D, means2D (its first two columns: the
        NDC-scaled screen gradient), dc, shs or colors_precomp, opacities,
        scales and rotations.  ``cov3D_precomp`` is not supported."""
        self._inputs(shs, colors_precomp, scales, rotations, cov3D_precomp)
        return rasterize_gaussians(means3D, means2D, dc, shs, colors_precomp, opacities, scales, rotations,
                                   cov3D_precomp, flag_max_count, culling, self.raster_settings)

    def render_simp(self, means3D, means2D, opacities, culling=None, dc=None, shs=None, colors_precomp=None,
                    scales=None, rotations=None, cov3D_precomp=None):
        """Mini-splatting statistics pass (f/__init__.py:732-770, forward.cu:
        466-607): (color, radii, accum_weights_ptr float [P] = sum of alpha*T
        over the pixels each Gaussian blends into, accum_weights_count int32
        [P] = their number, accum_max_count float [P]).  No gradients."""
        self._inputs(shs, colors_precomp, scales, rotations, cov3D_precomp)
        return rasterize_gaussians_simp(means3D, means2D, dc, shs, colors_precomp, opacities, scales, rotations,
                                        cov3D_precomp, culling, self.raster_settings)

    def render_depth(self, means3D, means2D, opacities, culling=None, dc=None, shs=None, colors_precomp=None,
                     scales=None, rotations=None, cov3D_precomp=None):
        """Depth pass (f/__init__.py:773-810, forward.cu:614-845): a dict with
        "render" [3,H,W], "out_pts" [3,H,W], "rendered_depth" [1,H,W],
        "discriminants" [1,H,W], "gidx" int32 [1,H,W], "accum_alpha"
        [1,H,W].  No gradients."""
        self._inputs(shs, colors_precomp, scales, rotations, cov3D_precomp)
        return rasterize_gaussians_depth(means3D, means2D, dc, shs, colors_precomp, opacities, scales, rotations,
                                         cov3D_precomp, culling, self.raster_settings)
