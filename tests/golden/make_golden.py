"""Generate the golden vectors in this directory by running the REFERENCE
rasterizer (BlitzGS's diff_gaussian_rasterization_f / _r CUDA modules, built
from the reference sources by oracle/build_ref.py into oracle/_ref/) on a
GPU, through the reference's own Python autograd wrappers, and the reference
loss helpers (utils/loss_utils.py).

Run on a B200:  python tests/golden/make_golden.py --out <dir>
(default: this directory) and commit the .npz files here.  Inputs are NOT stored: the tests regenerate
them from the same seeds with blitzgs_b200.scene (CPU torch.Generator, bit
identical everywhere); an input checksum is stored to detect drift.

Cases
  tiny   BASELINE config 1: 16,384 Gaussians, one 256x256 camera.  Stores the
         bit-exact outputs (radii, means2D, depths, per-tile sorted lists and
         ranges, n_contrib), the image, tile statistics, observation counts,
         the routing mask for a 4-way row split, loss sums, and every
         gradient row (rasterizer intermediates and activated parameters,
         float32) with its norm and sum.
  small  2,048 Gaussians, ragged 184x120 image, with edge cases planted: 5 %
         opacity below 1/255 (extent falls back to 3.33), points behind the
         near plane, points beyond the 1.3 tan(fov) clamp.  Stores every
         forward output and every gradient (rasterizer intermediates and
         parameter gradients), plus a render restricted to a band of tile rows.
"""
import argparse
import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))

from blitzgs_b200 import scene as S  # noqa: E402


def input_checksum(sc):
    h = hashlib.sha256()
    for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest):
        h.update(t.contiguous().numpy().tobytes())
    for c in sc.cameras:
        for t in (c.world_view_transform, c.full_proj_transform, c.camera_center):
            h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def small_scene(seed=1, P=2048, H=120, W=184):
    """Tiny scene with planted edge cases (deterministic)."""
    sc = S.tiny(seed=seed, P=P, H=H, W=W)
    g = torch.Generator().manual_seed(seed + 77)
    n = P // 20
    idx = torch.randperm(P, generator=g)
    sc.opacity[idx[:n]] = -7.0                                   # alpha < 1/255
    sc.xyz[idx[n:n + 16]] = torch.tensor([0.0, 0.0, -3.5])       # behind the camera
    sc.xyz[idx[n + 16:n + 48], 0] = 2.9                           # far off to the side (clamp path)
    sc.scaling[idx[n + 48:n + 64]] = -1.5                         # a few large splats
    return sc


def cuda_args(ws=1, rank=0):
    return {"mode": "train", "world_size": str(ws), "global_rank": str(rank), "local_rank": str(rank),
            "mp_world_size": str(ws), "mp_rank": str(rank), "log_folder": "/tmp", "log_interval": "1000000",
            "iteration": "1", "avoid_pixel_all2all": False, "stats_collector": {}}


def decode_img_buffer(img_buf, H, W, n_tiles):
    """ImageState layout of the reference (r/cuda_rasterizer/rasterizer_impl.cu:176-184,
    rasterizer_impl.h obtain(): 128-byte aligned consecutive arrays)."""
    N = H * W
    b = img_buf.cpu().numpy().view(np.uint8)
    al = lambda x: (x + 127) // 128 * 128
    o0 = 0
    o1 = al(o0 + 4 * N)
    o2 = al(o1 + 4 * N)
    o3 = al(o2 + 4 * N)
    final_T = b[o0:o0 + 4 * N].view(np.float32).copy()
    n_contrib = b[o1:o1 + 4 * N].view(np.uint32).copy()
    ranges = b[o3:o3 + 8 * n_tiles].view(np.uint32).reshape(n_tiles, 2).copy()
    return final_T, n_contrib, ranges


def run_reference(sc, cam, gt, compute_locally=None, want_grads=True):
    import diff_gaussian_rasterization_f as ref
    import ref_loss_utils as LU
    dev = "cuda"
    xyz = sc.xyz.to(dev).requires_grad_(True)
    s_raw = sc.scaling.to(dev)
    q_raw = sc.rotation.to(dev)
    o_raw = sc.opacity.to(dev)
    scales = torch.exp(s_raw).detach().requires_grad_(True)
    rots = torch.nn.functional.normalize(q_raw).detach().requires_grad_(True)
    shs = torch.cat((sc.features_dc, sc.features_rest), 1).to(dev).requires_grad_(True)
    ops_ = torch.sigmoid(o_raw).detach().requires_grad_(True)
    H, W = cam.image_height, cam.image_width
    rs = ref.GaussianRasterizationSettings(
        image_height=H, image_width=W, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy,
        bg=torch.zeros(3, device=dev), scale_modifier=1.0, viewmatrix=cam.world_view_transform.to(dev),
        projmatrix=cam.full_proj_transform.to(dev), sh_degree=3, campos=cam.camera_center.to(dev),
        prefiltered=False, debug=False)
    rast = ref.GaussianRasterizer(rs)
    ca = cuda_args()
    means2D, rgb, conic, radii, depths = rast.preprocess_gaussians(xyz, scales, rots, shs, ops_, ca)
    means2D.retain_grad()
    rgb.retain_grad()
    conic.retain_grad()
    gx, gy = (W + 15) // 16, (H + 15) // 16
    cl = torch.ones((gy, gx), dtype=torch.bool, device=dev) if compute_locally is None else compute_locally.to(dev)
    abs_pts = torch.zeros((xyz.shape[0], 3), device=dev, requires_grad=True) + 0
    abs_pts.retain_grad()
    all_map = torch.zeros((xyz.shape[0], 5), device=dev)
    color, n_render, n_consider, n_contrib_t, out_observe, _, _ = rast.render_gaussians(
        means2D, abs_pts, conic, rgb, all_map, depths, radii, cl, None, ca)
    # reference render state (saved tensors of the autograd node)
    node = color.grad_fn
    saved = node.saved_tensors
    binning_buf, img_buf = saved[6], saved[7]
    R = node.num_rendered if hasattr(node, "num_rendered") else None
    final_T, n_contrib, ranges = decode_img_buffer(img_buf, H, W, gx * gy)
    R = int(ranges[:, 1].max()) if ranges.size else 0
    point_list = binning_buf.cpu().numpy().view(np.uint8)[: 4 * R].view(np.uint32).copy()
    gt_f = torch.clamp(gt.to(dev) / 255.0, 0.0, 1.0)
    ones = torch.ones((H, W), dtype=torch.bool, device=dev)
    l1_map = LU.pixelwise_l1_with_mask(color, gt_f, ones)
    ssim_map = LU.pixelwise_ssim_with_mask(color, gt_f, ones)
    n3 = H * W * 3
    Ll1 = l1_map.sum() / n3
    ss = ssim_map.sum() / n3
    loss = 0.8 * Ll1 + 0.2 * (1.0 - ss)
    out = dict(
        radii=radii.cpu().numpy(), means2D=means2D.detach().cpu().numpy(), depths=depths.cpu().numpy(),
        conic_opacity=conic.detach().cpu().numpy(), rgb=rgb.detach().cpu().numpy(),
        point_list=point_list, ranges=ranges, final_T=final_T, n_contrib=n_contrib,
        image=color.detach().cpu().numpy(), n_render=n_render.cpu().numpy(), n_consider=n_consider.cpu().numpy(),
        n_contrib_tile=n_contrib_t.cpu().numpy(), out_observe=out_observe.cpu().numpy(),
        l1_sum=np.float64(l1_map.sum().item()), ssim_sum=np.float64(ssim_map.sum().item()),
        loss=np.float64(loss.item()))
    if want_grads:
        loss.backward()
        out.update(
            g_means2D=means2D.grad.cpu().numpy(), g_conic_opacity=conic.grad.cpu().numpy(),
            g_rgb=rgb.grad.cpu().numpy(), g_means2D_abs=abs_pts.grad.cpu().numpy(),
            g_means3D=xyz.grad.cpu().numpy(), g_scales=scales.grad.cpu().numpy(),
            g_rotations=rots.grad.cpu().numpy(), g_shs=shs.grad.cpu().numpy(),
            g_opacities=ops_.grad.cpu().numpy())
    return out


def route_reference(means2D, radii, H, W, division_rows):
    import diff_gaussian_rasterization_f as ref
    gx = (W + 15) // 16
    dist = torch.tensor(division_rows, dtype=torch.int32, device="cuda") * gx
    m = ref._C.get_local2j_ids_bool(H, W, 0, len(division_rows) - 1, torch.as_tensor(means2D).cuda(),
                                    torch.as_tensor(radii).cuda(), dist, cuda_args())
    return m.cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    ap.add_argument("--only", choices=["tiny", "small"], default=None)
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    torch.backends.cudnn.deterministic = True

    if a.only != "small":
        make_tiny(a.out)
    if a.only != "tiny":
        make_small(a.out)


def make_tiny(out):
    # --- tiny (config 1) ---
    sc = S.tiny()
    cam = sc.cameras[0]
    gt = S.target_image(0, cam.image_height, cam.image_width)
    o = run_reference(sc, cam, gt)
    route = route_reference(o["means2D"], o["radii"], cam.image_height, cam.image_width, [0, 4, 8, 12, 16])
    keep = ["radii", "means2D", "depths", "point_list", "ranges", "n_contrib", "image", "n_render",
            "n_consider", "n_contrib_tile", "out_observe", "l1_sum", "ssim_sum", "loss"]
    d = {k: o[k] for k in keep}
    d["n_contrib"] = d["n_contrib"].astype(np.uint16)
    d["route_packed"] = np.packbits(route.astype(np.uint8), axis=None)
    d["route_shape"] = np.array(route.shape)
    for k in ("g_means3D", "g_scales", "g_rotations", "g_shs", "g_opacities", "g_means2D", "g_conic_opacity",
              "g_rgb"):
        g = o[k].astype(np.float64)
        d[k + "_l2"] = np.sqrt((g * g).sum())
        d[k + "_sum"] = g.sum()
        d[k] = o[k].astype(np.float32)
    d["input_sha256"] = np.array(input_checksum(sc))
    np.savez_compressed(os.path.join(out, "golden_tiny.npz"), **d)
    print("tiny: R", len(o["point_list"]), "visible", int((o["radii"] > 0).sum()), "loss", o["loss"])


def make_small(out):
    # --- small with edge cases, full outputs + band render ---
    sc = small_scene()
    cam = sc.cameras[0]
    gt = S.target_image(1, cam.image_height, cam.image_width)
    o = run_reference(sc, cam, gt)
    H, W = cam.image_height, cam.image_width
    gx, gy = (W + 15) // 16, (H + 15) // 16
    band = torch.zeros((gy, gx), dtype=torch.bool)
    band[2:5] = True
    ob = run_reference(sc, cam, gt, compute_locally=band)
    d = dict(o)
    for k, v in ob.items():
        d["band_" + k] = v
    d["band_rows"] = np.array([2, 5])
    d["input_sha256"] = np.array(input_checksum(sc))
    np.savez_compressed(os.path.join(out, "golden_small.npz"), **d)
    print("small: R", len(o["point_list"]), "visible", int((o["radii"] > 0).sum()), "loss", o["loss"])


if __name__ == "__main__":
    main()
