"""Densification statistics of the training step.

The reference accumulates, after each camera's backward
(train_internal.py:340-371, scene/gaussian_model.py:792-794):

    max_radii2D[vis] = max(max_radii2D[vis], radii[vis])
    xyz_gradient_accum[vis] += ||dL/dmeans2D[vis, :2]||   (the viewspace gradient)
    denom[vis] += 1

with vis = radii > 0 of the camera's preprocess and dL/dmeans2D the gradient
of the preprocessed screen means (on N GPUs: summed over the ranks that
rendered the Gaussian).  The fused steps never materialise a means2D tensor
for autograd; their render-backward record holds that gradient, so they call
these functions with the record's rows instead (``step.view_loss(...,
densify=stats)``, ``dist_step.batch_loss(..., densify=stats)``).

Plain PyTorch on whatever device the tensors live on: a gather-free
index_add over the visible rows and one elementwise maximum per camera.
"""
import torch


class DensificationStats:
    """The three per-Gaussian buffers the reference keeps on GaussianModel:
    xyz_gradient_accum [P,1], denom [P,1] and max_radii2D [P] (float32)."""

    def __init__(self, P, device, dtype=torch.float32):
        self.xyz_gradient_accum = torch.zeros((P, 1), dtype=dtype, device=device)
        self.denom = torch.zeros((P, 1), dtype=dtype, device=device)
        self.max_radii2D = torch.zeros((P,), dtype=dtype, device=device)

    def reset(self):
        self.xyz_gradient_accum.zero_()
        self.denom.zero_()
        self.max_radii2D.zero_()

    def average_grad(self):
        """xyz_gradient_accum / denom with the NaNs of never-visible Gaussians
        (0/0) set to 0: the value the reference's densify_and_prune
        thresholds (scene/gaussian_model.py:695-697)."""
        g = self.xyz_gradient_accum / self.denom
        g[g.isnan()] = 0.0
        return g


def update_max_radii(stats, radii):
    """max_radii2D = max(max_radii2D, radii) where radii > 0.  Radii are
    never negative and the buffer starts at 0, so a plain elementwise maximum
    equals the reference's masked update."""
    torch.maximum(stats.max_radii2D, radii.to(stats.max_radii2D.dtype), out=stats.max_radii2D)


def accumulate_grad(stats, rows, grad_means2D):
    """xyz_gradient_accum[rows] += ||grad_means2D[:, :2]||, denom[rows] += 1.
    ``rows``: int64 [n] Gaussian indices, unique (a camera's visible list);
    ``grad_means2D``: [n, >=2], row i the gradient of Gaussian rows[i]."""
    if rows.numel() == 0:
        return
    g = grad_means2D[:, :2].to(stats.xyz_gradient_accum.dtype)
    norm = torch.norm(g, dim=-1, keepdim=True)
    stats.xyz_gradient_accum.index_add_(0, rows, norm)
    stats.denom.index_add_(0, rows, torch.ones_like(norm))
