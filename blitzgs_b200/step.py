"""Fused single-process training step: preprocess -> binning -> blend -> L1+SSIM
-> backward, per camera, on the sm_100a kernels.

This is the body of the reference's distributed_preprocess3dgs_and_all2all_final
+ render_final + batched_loss_computation + loss.backward() for the Gaussians
and tile rows a rank owns (gaussian_renderer/__init__.py:220-413, 664-854,
gaussian_renderer/loss_distribution.py:220-329), with three changes that keep
results identical:
  * SH coefficients are read from _features_dc / _features_rest in place (the
    reference concatenates them with torch.cat and splits them again in C++);
  * one autograd node per camera covers preprocess, render and loss, so no
    per-Gaussian intermediate is materialised for autograd and the render
    gradient record [P,16] feeds the preprocess backward directly;
  * the only host synchronisation is the two-number readback that sizes the
    binning buffers.
Parameter activations (exp, sigmoid, normalize) stay in PyTorch autograd,
exactly as GaussianModel's getters compute them.
"""
import torch
import torch.nn.functional as F

from . import ops

LAMBDA_DSSIM = 0.2


class _ViewLoss(torch.autograd.Function):
    """(xyz, scales, rots, opac, dc, rest) -> (l1_sum, ssim_sum) for one camera band."""

    @staticmethod
    def forward(ctx, xyz, scales, rots, opac, dc, rest, raster, gt, compute_locally, band):
        H, W = int(raster.image_height), int(raster.image_width)
        sh = ops.sh_layout(dc=dc, rest=rest)
        means2D, depths, radii, conic, rgb, _, _ = ops.preprocess_forward(
            xyz, scales, rots, opac.reshape(-1), sh, raster)
        color, n_render, n_consider, n_contrib, out_observe, state = ops.render_forward(
            means2D, depths, radii, conic, rgb, raster.bg, compute_locally, H, W)
        y0, y1 = band
        img_band = color[:, y0:y1, :]
        sums, partials = ops.loss_forward(img_band, gt)
        ctx.raster = raster
        ctx.band = band
        ctx.HW = (H, W)
        ctx.state = state
        ctx.cl = compute_locally
        ctx.save_for_backward(xyz, scales, rots, opac, dc, rest, means2D, conic, rgb, radii, gt, partials, img_band)
        ctx.mark_non_differentiable(radii, out_observe, n_render, n_consider, n_contrib)
        l1 = sums[0].to(torch.float32)
        ss = sums[1].to(torch.float32)
        return l1, ss, radii, out_observe, n_render, n_consider, n_contrib, color

    @staticmethod
    def backward(ctx, g_l1, g_ss, *_unused):
        xyz, scales, rots, opac, dc, rest, means2D, conic, rgb, radii, gt, partials, img_band = ctx.saved_tensors
        H, W = ctx.HW
        y0, y1 = ctx.band
        dev = xyz.device
        zero = torch.zeros((), device=dev)
        scale = torch.stack([g_l1 if g_l1 is not None else zero, g_ss if g_ss is not None else zero]).float()
        g_band = ops.loss_backward(img_band, gt, partials, scale)
        if y0 == 0 and y1 == H:
            dL_dpix = g_band
        else:
            dL_dpix = torch.zeros((3, H, W), dtype=torch.float32, device=dev)
            dL_dpix[:, y0:y1, :] = g_band
        rec = ops.render_backward(ctx.state, means2D, conic, rgb, ctx.raster.bg, ctx.cl, dL_dpix)
        sh = ops.sh_layout(dc=dc, rest=rest)
        P = xyz.shape[0]
        M = rest.shape[1]
        g_xyz = torch.empty_like(xyz)
        g_s = torch.empty_like(scales)
        g_q = torch.empty_like(rots)
        g_o = torch.empty((P, 1), dtype=torch.float32, device=dev)
        g_dc = torch.empty_like(dc)
        g_rest = torch.empty_like(rest)
        ops.preprocess_backward(radii, xyz, scales, rots, sh, ctx.raster, rec[:, 0:2], rec[:, 8:12], rec[:, 12:15],
                                out=(g_xyz, g_s, g_q, g_o, (g_dc, 3), (g_rest, max(M, 1) * 3)))
        return g_xyz, g_s, g_q, g_o.view_as(opac), g_dc, g_rest, None, None, None, None


def view_loss(model, raster, gt_band, compute_locally=None, band=None, lambda_dssim=LAMBDA_DSSIM,
              scale_reg_weight=10.0):
    """Loss of one camera exactly as batched_loss_computation forms it
    (loss_distribution.py:303-322): (1-l) L1/N3 + l (1 - SSIM/N3) +
    10 mean(min-axis scale of visible Gaussians), N3 = 3 H W.

    ``model`` = (xyz, _scaling, _rotation, _opacity, _features_dc, _features_rest)
    raw parameters; activations are applied here in PyTorch.
    Returns (loss, l1_sum, ssim_sum, radii, out_observe, color)."""
    xyz, s_raw, q_raw, o_raw, dc, rest = model
    H, W = int(raster.image_height), int(raster.image_width)
    band = band or (0, H)
    scales = torch.exp(s_raw)
    rots = F.normalize(q_raw)
    opac = torch.sigmoid(o_raw)
    l1, ss, radii, out_observe, _, _, _, color = _ViewLoss.apply(xyz, scales, rots, opac, dc, rest, raster, gt_band,
                                                                 compute_locally, band)
    n3 = H * W * 3
    loss = (1.0 - lambda_dssim) * (l1 / n3) + lambda_dssim * (1.0 - ss / n3)
    if scale_reg_weight:
        vis = (radii > 0).to(torch.float32)
        mins = scales.min(dim=1).values
        loss = loss + scale_reg_weight * (mins * vis).sum() / vis.sum().clamp(min=1.0)
    return loss, l1, ss, radii, out_observe, color
