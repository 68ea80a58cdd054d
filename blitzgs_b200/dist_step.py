"""Distributed training step over N GPUs (one process per GPU, NCCL).

Per step, for a batch of cameras split into tile-row bands by
``start_strategy_final``:
  forward   every rank preprocesses its spatial shard for every camera,
            routes each visible Gaussian to the ranks whose bands its tile
            rect overlaps (the reference's get_local2j_ids semantics), and
            ONE all_to_all_single moves a 12-float record per (Gaussian,
            camera, destination); each rank renders its bands and computes
            the band loss (L1 + SSIM + the min-scale regulariser over the
            received visible Gaussians, loss_distribution.py:303-322);
  backward  band loss / render backward on the receivers, ONE reverse
            all_to_all_single of 12-float gradient records, scatter-add
            into per-camera accumulators on the owners, preprocess backward
            accumulated into the shard's parameter gradients.
These two all-to-alls and the tiny size all-gather are the only collectives
(the reference additionally all-gathers sizes with a blocking .cpu() and
runs a second all-to-all for radii/depths).
"""
import torch
import torch.nn.functional as F

from . import distributed as D
from . import ops

# forward record: conic00 conic01 conic11 opacity | x y | r g b | depth radius(bits) minscale
_FWD_C = 12
# gradient record: conic00 conic01 conic11 opacity | x y | r g b | |x| |y| minscale
_BWD_C = 12


def _records(m2, depths, radii, conic, rgb, minscale):
    return torch.cat([conic, m2, rgb, depths[:, None], radii.view(torch.float32)[:, None], minscale[:, None]], 1)


class _DistributedBatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xyz, scales, rots, opac, dc, rest, setup):
        rasters, gts, strategies, group, lambda_dssim, reg_w = setup
        n_cams = len(rasters)
        rank = torch.distributed.get_rank(group)
        ws = torch.distributed.get_world_size(group)
        sh = ops.sh_layout(dc=dc, rest=rest)
        minscale = scales.min(dim=1).values
        records, radii_local, send_ids = [], [], []
        for k, rs in enumerate(rasters):
            m2, d, r, co, rgb, _, _ = ops.preprocess_forward(xyz, scales, rots, opac.reshape(-1), sh, rs)
            radii_local.append(r)
            records.append(_records(m2, d, r, co, rgb, minscale))
            ids_local, _ = strategies[k].get_local2j_ids(m2, r, rs, {"avoid_pixel_all2all": False})
            per = [torch.empty((0,), dtype=torch.int64, device=xyz.device) for _ in range(ws)]
            for lid, g in enumerate(strategies[k].gpu_ids):
                per[g] = ids_local[lid]
            send_ids.append(per)
        plan = D.plan_exchange(send_ids, n_cams, group)
        recv = D.exchange_forward(records, plan, group)

        loss_sum = torch.zeros((), dtype=torch.float32, device=xyz.device)
        saved = {}
        for k in range(n_cams):
            st = strategies[k]
            if rank not in st.gpu_ids:
                continue
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            rec = recv.get(k)
            if rec is None:
                rec = torch.zeros((0, _FWD_C), dtype=torch.float32, device=xyz.device)
            conic = rec[:, 0:4].contiguous()
            m2 = rec[:, 4:6].contiguous()
            rgb = rec[:, 6:9].contiguous()
            depth = rec[:, 9].contiguous()
            radii = rec[:, 10].contiguous().view(torch.int32)
            mins = rec[:, 11]
            y0t, y1t = st.row_range(rank)
            cl = st.get_compute_locally(device=xyz.device)
            color, _, _, _, _, state = ops.render_forward(m2, depth, radii, conic, rgb, rs.bg, cl, H, W)
            y0, y1 = y0t * D.TILE, min(H, y1t * D.TILE)
            band = color[:, y0:y1, :]
            gt = gts[k]
            sums, partials = ops.loss_forward(band, gt)
            n3 = H * W * 3
            vis = (radii > 0).to(torch.float32)
            nvis = vis.sum()
            reg = (mins * vis).sum() / nvis.clamp(min=1.0)
            lk = ((1.0 - lambda_dssim) * (sums[0] / n3) + lambda_dssim * (1.0 - sums[1] / n3)).to(torch.float32)
            lk = lk + reg_w * reg
            loss_sum = loss_sum + lk
            saved[k] = (state, m2, conic, rgb, cl, band, gt, partials, vis, nvis, (y0, y1), n3)
        ctx.setup = setup
        ctx.plan = plan
        ctx.saved = saved
        ctx.radii_local = radii_local
        ctx.save_for_backward(xyz, scales, rots, opac, dc, rest)
        return loss_sum

    @staticmethod
    def backward(ctx, g_loss):
        rasters, gts, strategies, group, lambda_dssim, reg_w = ctx.setup
        xyz, scales, rots, opac, dc, rest = ctx.saved_tensors
        n_cams = len(rasters)
        dev = xyz.device
        grads = {}
        for k, (state, m2, conic, rgb, cl, band, gt, partials, vis, nvis, (y0, y1), n3) in ctx.saved.items():
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            scale = torch.stack([g_loss * (1.0 - lambda_dssim) / n3, -g_loss * lambda_dssim / n3]).float()
            g_band = ops.loss_backward(band, gt, partials, scale)
            dpix = torch.zeros((3, H, W), dtype=torch.float32, device=dev)
            dpix[:, y0:y1] = g_band
            rec16 = ops.render_backward(state, m2, conic, rgb, rs.bg, cl, dpix)
            g = torch.empty((m2.shape[0], _BWD_C), dtype=torch.float32, device=dev)
            g[:, 0:4] = rec16[:, 8:12]
            g[:, 4:6] = rec16[:, 0:2]
            g[:, 6:9] = rec16[:, 12:15]
            g[:, 9:11] = rec16[:, 4:6]
            g[:, 11] = g_loss * reg_w * vis / nvis.clamp(min=1.0)
            grads[k] = g
        P = xyz.shape[0]
        acc = D.exchange_backward(grads, ctx.plan, P, n_cams, _BWD_C, group, device=dev)
        sh = ops.sh_layout(dc=dc, rest=rest)
        M = rest.shape[1]
        g_xyz = torch.zeros_like(xyz)
        g_s = torch.zeros_like(scales)
        g_q = torch.zeros_like(rots)
        g_o = torch.zeros((P, 1), dtype=torch.float32, device=dev)
        g_dc = torch.zeros_like(dc)
        g_rest = torch.zeros_like(rest)
        g_min = torch.zeros((P,), dtype=torch.float32, device=dev)
        for k in range(n_cams):
            a = acc[k]
            ops.preprocess_backward(ctx.radii_local[k], xyz, scales, rots, sh, rasters[k], a[:, 4:6], a[:, 0:4],
                                    a[:, 6:9], out=(g_xyz, g_s, g_q, g_o, (g_dc, 3), (g_rest, max(M, 1) * 3)),
                                    accumulate=True)
            g_min += a[:, 11]
        # minscale = scales.min(dim=1): gradient goes to the arg-min axis
        am = scales.argmin(dim=1)
        g_s.scatter_add_(1, am[:, None], g_min[:, None])
        return g_xyz, g_s, g_q, g_o.view_as(opac), g_dc, g_rest, None


def batch_loss(shard_model, rasters, gts, strategies, group=None, lambda_dssim=0.2, reg_w=10.0):
    """Sum over the cameras this rank renders of the reference's per-camera
    loss.  Every rank must call ``.backward()`` on the result (the backward
    exchange is a collective), also when it renders nothing.
    ``shard_model`` = raw (xyz, _scaling, _rotation, _opacity, _features_dc,
    _features_rest) of this rank's shard; ``gts[k]`` is this rank's uint8
    ground-truth band of camera k (rows of its tile band) or None."""
    xyz, s_raw, q_raw, o_raw, dc, rest = shard_model
    scales = torch.exp(s_raw)
    rots = F.normalize(q_raw)
    opac = torch.sigmoid(o_raw)
    return _DistributedBatch.apply(xyz, scales, rots, opac, dc, rest,
                                   (rasters, gts, strategies, group, lambda_dssim, reg_w))
