"""Run the REFERENCE rasterizer's stock training path on a GPU (test helper).

TEST INFRASTRUCTURE ONLY.  The reference's diff_gaussian_rasterization_f / _r
CUDA modules, built unmodified from the reference sources by
oracle/build_ref.py into oracle/_ref/ (git-ignored; it travels to the GPU box
with the working tree), are driven through the reference's own Python
autograd wrappers and loss helpers, exactly as one rank of its trainer at
world size 1 drives them:

  GaussianModel getters (scene/gaussian_model.py:248-276): exp, normalize,
    sigmoid, cat(dc, rest)
  GaussianRasterizer.preprocess_gaussians  (f/__init__.py:677-689)
  GaussianRasterizer.render_gaussians      (f/__init__.py:812-829)
  loss_utils.pixelwise_l1/ssim_with_mask   (utils/loss_utils.py:83-124)
  the loss of batched_loss_computation     (gaussian_renderer/loss_distribution.py:303-322):
    0.8 L1/N3 + 0.2 (1 - SSIM/N3) + 10 mean(min-axis scale of the visible Gaussians)
  loss.backward() down to the raw parameters.

"Visible" is render_final's visibility_filter (gaussian_renderer/__init__.py:832):
radius > 0 among the Gaussians the exchange delivered to the rank, i.e. those
_C.get_local2j_ids_bool routes to it (workload_division.py:682-704, at world
size 1 the whole tile range [0, T)).

The render state the reference keeps for its backward (the sorted per-tile
lists, tile ranges, final transmittance and per-pixel contributor counts)
is decoded from the autograd node's saved buffers with the layout of
r/cuda_rasterizer/rasterizer_impl.cu (ImageState / BinningState).
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def available():
    return all(os.path.exists(os.path.join(REF_DIR, p, "_C.so"))
               for p in ("diff_gaussian_rasterization_f", "diff_gaussian_rasterization_r")) and \
        os.path.exists(os.path.join(REF_DIR, "ref_loss_utils.py"))


def _modules():
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import diff_gaussian_rasterization_f as ref
    import ref_loss_utils as LU
    return ref, LU


def cuda_args(ws=1, rank=0):
    return {"mode": "train", "world_size": str(ws), "global_rank": str(rank), "local_rank": str(rank),
            "mp_world_size": str(ws), "mp_rank": str(rank), "log_folder": "/tmp", "log_interval": "1000000",
            "iteration": "1", "avoid_pixel_all2all": False, "stats_collector": {}}


def settings(cam, dev, sh_degree=3):
    ref, _ = _modules()
    return ref.GaussianRasterizationSettings(
        image_height=int(cam.image_height), image_width=int(cam.image_width), tanfovx=cam.tanfovx,
        tanfovy=cam.tanfovy, bg=torch.zeros(3, device=dev), scale_modifier=1.0,
        viewmatrix=cam.world_view_transform.to(dev), projmatrix=cam.full_proj_transform.to(dev),
        sh_degree=sh_degree, campos=cam.camera_center.to(dev), prefiltered=False, debug=False)


def _decode_state(node, H, W):
    """point_list, ranges, final_T, n_contrib from the render node's saved
    binning / image buffers (r/cuda_rasterizer/rasterizer_impl.cu:176-184:
    128-byte aligned consecutive arrays final_T f32[N], n_contrib u32[N],
    n_contrib2loss u32[N], ranges uint2[T]; the binning buffer starts with
    point_list u32[R])."""
    saved = node.saved_tensors
    binning_buf, img_buf = saved[6], saved[7]
    N = H * W
    T = ((W + 15) // 16) * ((H + 15) // 16)
    al = lambda x: (x + 127) // 128 * 128  # noqa: E731
    o1 = al(4 * N)
    o3 = al(al(o1 + 4 * N) + 4 * N)
    final_T = img_buf[: 4 * N].view(torch.float32).clone()
    n_contrib = img_buf[o1:o1 + 4 * N].view(torch.int32).clone()
    ranges = img_buf[o3:o3 + 8 * T].view(torch.int32).reshape(T, 2).clone()
    R = int(ranges[:, 1].max().item()) if T else 0
    point_list = binning_buf[: 4 * R].view(torch.int32).clone()
    return point_list, ranges, final_T, n_contrib


def preprocess(model, cam, dev):
    """Reference preprocess of raw parameters (no autograd): (means2D, rgb,
    conic_opacity, radii, depths)."""
    ref, _ = _modules()
    xyz, s_raw, q_raw, o_raw, dc, rest = [t.to(dev) for t in model]
    with torch.no_grad():
        rast = ref.GaussianRasterizer(settings(cam, dev))
        return rast.preprocess_gaussians(xyz, torch.exp(s_raw), torch.nn.functional.normalize(q_raw),
                                         torch.cat((dc, rest), 1), torch.sigmoid(o_raw), cuda_args())


def train_view(model, cam, gt_u8, dev, reg_weight=10.0, lambda_dssim=0.2):
    """One camera of the reference's training step from raw parameters.

    Returns a dict of forward outputs, the decoded render state, the loss
    and the gradients of the six raw parameter tensors (g_xyz, g_scaling,
    g_rotation, g_opacity, g_features_dc, g_features_rest)."""
    ref, LU = _modules()
    params = [t.to(dev).detach().requires_grad_(True) for t in model]
    xyz, s_raw, q_raw, o_raw, dc, rest = params
    H, W = int(cam.image_height), int(cam.image_width)
    scales = torch.exp(s_raw)
    rots = torch.nn.functional.normalize(q_raw)
    shs = torch.cat((dc, rest), dim=1)
    opac = torch.sigmoid(o_raw)
    rast = ref.GaussianRasterizer(settings(cam, dev))
    ca = cuda_args()
    means2D, rgb, conic, radii, depths = rast.preprocess_gaussians(xyz, scales, rots, shs, opac, ca)
    gx, gy = (W + 15) // 16, (H + 15) // 16
    cl = torch.ones((gy, gx), dtype=torch.bool, device=dev)
    abs_pts = torch.zeros((xyz.shape[0], 3), device=dev) + 0
    all_map = torch.zeros((xyz.shape[0], 5), device=dev)
    color, n_render, n_consider, n_contrib_t, out_observe, _, _ = rast.render_gaussians(
        means2D, abs_pts, conic, rgb, all_map, depths, radii, cl, None, ca)
    point_list, ranges, final_T, n_contrib = _decode_state(color.grad_fn, H, W)
    gt = torch.clamp(gt_u8.to(dev) / 255.0, 0.0, 1.0)
    ones = torch.ones((H, W), dtype=torch.bool, device=dev)
    n3 = H * W * 3
    Ll1 = LU.pixelwise_l1_with_mask(color, gt, ones).sum() / n3
    ss = LU.pixelwise_ssim_with_mask(color, gt, ones).sum() / n3
    loss = (1.0 - lambda_dssim) * Ll1 + lambda_dssim * (1.0 - ss)
    T = gx * gy
    routed = ref._C.get_local2j_ids_bool(H, W, 0, 1, means2D.detach(), radii,
                                         torch.tensor([0, T], dtype=torch.int32, device=dev), ca)[:, 0]
    vis = (radii > 0) & routed
    if reg_weight and vis.sum() > 0:
        loss = loss + reg_weight * torch.sort(scales[vis], dim=-1)[0][..., 0].mean()
    loss.backward()
    out = dict(radii=radii, means2D=means2D.detach(), depths=depths, conic_opacity=conic.detach(),
               rgb=rgb.detach(), image=color.detach(), n_render=n_render, n_consider=n_consider,
               n_contrib_tile=n_contrib_t, out_observe=out_observe, point_list=point_list, ranges=ranges,
               final_T=final_T, n_contrib=n_contrib, loss=float(loss.item()),
               grads=[p.grad.detach() for p in params])
    return out


def as_np(t):
    return t.detach().cpu().numpy() if torch.is_tensor(t) else np.asarray(t)
