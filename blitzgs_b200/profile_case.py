"""Run a few training views of a synthetic BASELINE config, for profilers.

  python -m blitzgs_b200.profile_case --config city --P 2000000 --views 2

Each view is one full forward + backward (preprocess, binning, blend, L1+SSIM
and their backwards).  With --P the scene keeps the config's distribution
but fewer Gaussians, so an ncu capture stays small while its inputs remain
larger than L2.
"""
import argparse
import sys

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="city")
    ap.add_argument("--P", type=int, default=None)
    ap.add_argument("--views", type=int, default=2)
    a = ap.parse_args(argv)
    from . import scene as S, step as ST
    kw = {"P": a.P} if a.P else {}
    sc = S.CONFIGS[a.config](seed=0, **kw)
    dev = torch.device("cuda", 0)
    model = [t.to(dev).requires_grad_(True) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                      sc.features_dc, sc.features_rest)]
    for v in range(a.views):
        cam = sc.cameras[v % len(sc.cameras)].to(dev)
        gt = S.target_image(v, cam.image_height, cam.image_width).to(dev)
        rs = S.raster_settings(cam, device=dev)
        for p in model:
            p.grad = None
        loss, *_ = ST.view_loss(model, rs, gt)
        loss.backward()
    torch.cuda.synchronize()
    print(f"profile_case ok: {a.config} P={sc.P} views={a.views} loss={loss.item():.6f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
