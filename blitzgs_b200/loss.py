"""Fused L1 + SSIM loss over an image band (sm_100a kernels).

Drop-in for the reference's per-band loss
(gaussian_renderer/loss_distribution.py:220-263 final_system_loss_computation
with utils/loss_utils.py:83-124 pixelwise_l1_with_mask /
pixelwise_ssim_with_mask): the band [3,Hb,W] of the rendered image against
the uint8 ground-truth band (divided by 255 and clamped, as the reference
does), 11x11 Gaussian window (sigma 1.5) with zero padding at the band edges.
One forward kernel produces both sums and the per-pixel SSIM partial
derivatives; one backward kernel produces dL/dimage.
"""
import torch

from . import ops


class _BandLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img, gt):
        sums, partials = ops.loss_forward(img, gt)
        ctx.save_for_backward(img, gt, partials)
        return sums[0].to(torch.float32), sums[1].to(torch.float32)

    @staticmethod
    def backward(ctx, g_l1, g_ss):
        img, gt, partials = ctx.saved_tensors
        z = torch.zeros((), device=img.device)
        scale = torch.stack([g_l1 if g_l1 is not None else z, g_ss if g_ss is not None else z]).float()
        return ops.loss_backward(img, gt, partials, scale), None


def band_loss(img_band, gt_band):
    """(sum |img - gt|, sum SSIM map) over the band; differentiable in img."""
    return _BandLoss.apply(img_band.contiguous(), gt_band.contiguous())


def final_system_loss_computation(image, gt_band_u8, y0, y1, num_pixels):
    """(Ll1, ssim_loss) for tile-row band [y0, y1) of ``image`` [3,H,W], each
    normalised by num_pixels * 3 as the reference does (loss_distribution.py:253,257)."""
    l1, ss = band_loss(image[:, y0:y1, :], gt_band_u8)
    n3 = num_pixels * 3
    return l1 / n3, ss / n3
