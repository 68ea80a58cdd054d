"""Generate golden_full.npz by running the REFERENCE's full rasterizer
(diff_gaussian_rasterization_f: GaussianRasterizer.forward with
flag_max_count, render_simp and markVisible -> _C.rasterize_gaussians,
_C.rasterize_gaussians_simp, _C.mark_visible), built unmodified from the
reference sources by oracle/build_ref.py into oracle/_ref/, on a GPU.

Run on a B200:  python tests/golden/make_golden_full.py --out <dir>
(default: this directory) and commit golden_full.npz here.  Inputs are not
stored: the tests rebuild them from the same seeds (blitzgs_b200.scene, CPU
torch.Generator); an input checksum detects drift.

Case: 8,192 Gaussians (config-1 distribution, seed 4), one ragged 184x200
camera at an angle, a 10 % culling mask, background (0.1, 0.25, 0.4).
Stored: radii; the preprocess state the binning reads (means2D, depths,
rects, conic_opacity, rgb; zero rows where radius is 0), decoded from the
forward's geometry buffer (f/cuda_rasterizer/rasterizer_impl.cu:271-287);
the valid per-tile lists and ranges, n_contrib and final T decoded from the
binning / image buffers; the image; accum_max_count; render_simp's
accum_weights_ptr / accum_weights_count; markVisible of the points scaled by
3; and, from a second forward with seeded precomputed colours, that image
and the gradients of means3D, means2D, opacities, scales, rotations and
colors_precomp for loss = sum(weight * image), weight seeded.  (The
reference's backward of this path is only run with precomputed colours:
with SH colours it stores the DC gradient through the null dL_ddc pointer
that Rasterizer::backward passes, f/cuda_rasterizer/rasterizer_impl.cu:
933-955 and backward.cu:45-50.)
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

BG = (0.1, 0.25, 0.4)


def full_scene():
    """The golden case's scene, camera, culling mask and loss weight (CPU)."""
    sc = S.tiny(seed=4, P=8192, H=200, W=184)
    cam = S.look_at_camera([2.2, -0.9, -1.9], [0.05, 0.0, 0.0], [0, -1, 0], 184, 200, 1.05, uid=1)
    g = torch.Generator().manual_seed(404)
    culling = torch.rand(sc.xyz.shape[0], generator=g) < 0.1
    weight = torch.rand((3, 200, 184), generator=g)
    colors = torch.rand((sc.xyz.shape[0], 3), generator=g)
    return sc, cam, culling, weight, colors


def input_checksum(sc, cam, culling, weight, colors):
    h = hashlib.sha256()
    for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest, cam.world_view_transform,
              cam.full_proj_transform, cam.camera_center, culling, weight, colors):
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def activated_inputs(sc, dev):
    return dict(means3D=sc.xyz.to(dev), scales=torch.exp(sc.scaling).to(dev),
                rotations=torch.nn.functional.normalize(sc.rotation).to(dev),
                opacities=torch.sigmoid(sc.opacity).to(dev), dc=sc.features_dc.to(dev).contiguous(),
                shs=sc.features_rest.to(dev).contiguous())


def settings(pkg, cam, dev):
    return pkg.GaussianRasterizationSettings(
        image_height=int(cam.image_height), image_width=int(cam.image_width), tanfovx=cam.tanfovx,
        tanfovy=cam.tanfovy, bg=torch.tensor(BG, device=dev), scale_modifier=1.0,
        viewmatrix=cam.world_view_transform.to(dev), projmatrix=cam.full_proj_transform.to(dev), sh_degree=3,
        campos=cam.camera_center.to(dev), prefiltered=False, debug=False)


def _decode(color, P, H, W):
    """Geometry, binning and image buffers of the reference forward
    (rasterizer_impl.cu:271-331): 128-byte aligned consecutive arrays."""
    saved = color.grad_fn.saved_tensors
    geom, binning, img = saved[8], saved[9], saved[10]
    al = lambda x: (x + 127) // 128 * 128  # noqa: E731
    o_depth = 0
    o_clamped = al(4 * P)
    o_radii = al(o_clamped + 3 * P)
    o_rects = al(o_radii + 4 * P)
    o_m2 = al(o_rects + 8 * P)
    o_cov = al(o_m2 + 8 * P)
    o_conic = al(o_cov + 24 * P)
    o_rgb = al(o_conic + 16 * P)
    f = lambda o, n, c: geom[o:o + 4 * n * c].view(torch.float32).reshape(n, c) if c > 1 else \
        geom[o:o + 4 * n].view(torch.float32)  # noqa: E731
    state = dict(depths=f(o_depth, P, 1), rects=f(o_rects, P, 2), means2D=f(o_m2, P, 2), conic_opacity=f(o_conic, P, 4),
                 rgb=f(o_rgb, P, 3))
    N = H * W
    T = ((W + 15) // 16) * ((H + 15) // 16)
    o1 = al(4 * N)
    o2 = al(o1 + 4 * N)
    state["final_T"] = img[: 4 * N].view(torch.float32)
    state["n_contrib"] = img[o1:o1 + 4 * N].view(torch.int32)
    state["ranges"] = img[o2:o2 + 8 * T].view(torch.int32).reshape(T, 2)
    R = int(state["ranges"][:, 1].max().item()) if T else 0
    state["point_list"] = binning[: 4 * R].view(torch.int32)
    return {k: v.detach().cpu().clone() for k, v in state.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    args = ap.parse_args()
    import diff_gaussian_rasterization_f as ref
    dev = torch.device("cuda", 0)
    sc, cam, culling, weight, colors = full_scene()
    H, W = int(cam.image_height), int(cam.image_width)
    P = sc.xyz.shape[0]
    inp = activated_inputs(sc, dev)
    cull = culling.to(dev)
    rast = ref.GaussianRasterizer(settings(ref, cam, dev))
    # SH colours: forward state only (no backward, see above)
    x = {k: v.clone().requires_grad_(True) for k, v in inp.items()}
    color, radii, amc = rast(x["means3D"], torch.zeros_like(inp["means3D"], requires_grad=True), x["opacities"],
                             cull, dc=x["dc"], shs=x["shs"], scales=x["scales"], rotations=x["rotations"],
                             flag_max_count=True)
    state = _decode(color, P, H, W)
    color = color.detach().clone()
    del x
    # precomputed colours: forward and backward
    y = {k: inp[k].clone().requires_grad_(True) for k in ("means3D", "opacities", "scales", "rotations")}
    y["means2D"] = torch.zeros_like(inp["means3D"], requires_grad=True)
    y["colors_precomp"] = colors.to(dev).requires_grad_(True)
    color_pc, _, _ = rast(y["means3D"], y["means2D"], y["opacities"], cull, colors_precomp=y["colors_precomp"],
                          scales=y["scales"], rotations=y["rotations"])
    (color_pc * weight.to(dev)).sum().backward()
    with torch.no_grad():
        _, _, acc_w, acc_n, _ = rast.render_simp(inp["means3D"], torch.zeros_like(inp["means3D"]), inp["opacities"],
                                                 cull, dc=inp["dc"], shs=inp["shs"], scales=inp["scales"],
                                                 rotations=inp["rotations"])
        vis = rast.markVisible(inp["means3D"] * 3.0)
    torch.cuda.synchronize()
    keep = (radii > 0).cpu()
    out = {"checksum": np.array(input_checksum(sc, cam, culling, weight, colors)), "radii": radii.detach().cpu().numpy(),
           "image": color.cpu().numpy(), "image_precomp": color_pc.detach().cpu().numpy(),
           "accum_max_count": amc.detach().cpu().numpy(),
           "accum_weights_ptr": acc_w.cpu().numpy(), "accum_weights_count": acc_n.cpu().numpy(),
           "mark_visible": vis.cpu().numpy()}
    for k in ("depths", "rects", "means2D", "conic_opacity", "rgb"):
        v = state[k].clone()
        v[~keep] = 0
        out[k] = v.numpy()
    for k in ("final_T", "n_contrib", "ranges", "point_list"):
        out[k] = state[k].numpy()
    for k in ("means3D", "means2D", "opacities", "scales", "rotations", "colors_precomp"):
        out["grad_" + k] = y[k].grad.cpu().numpy()
    path = os.path.join(args.out, "golden_full.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes; R =", len(out["point_list"]),
          "visible =", int(keep.sum()))


if __name__ == "__main__":
    main()
