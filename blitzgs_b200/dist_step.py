"""Distributed training step over N GPUs (one process per GPU, NCCL).

Per step, for a batch of cameras split into tile-row bands by
``start_strategy_final``:
  forward   every rank runs the fused raw preprocess (activations in the
            kernel) of its spatial shard for every camera, routes each
            listed Gaussian (radius > 0) to the ranks whose bands its tile
            rect overlaps (the reference's get_local2j_ids semantics), and
            ONE all_to_all_single moves a 12-float record per (Gaussian,
            camera, destination); each rank renders its bands and computes
            the band loss (L1 + SSIM + the min-scale regulariser over the
            received visible Gaussians, loss_distribution.py:303-322);
  backward  band loss / render backward on the receivers, ONE reverse
            all_to_all_single of 12-float gradient records, one scatter-add
            into compact per-camera rows on the owners (aligned with each
            camera's visible list), and the listed preprocess backward
            accumulated into the shard's raw-parameter gradients.
These two all-to-alls and the tiny size all-gather are the only collectives
(the reference additionally all-gathers sizes with a blocking .cpu() and
runs a second all-to-all for radii/depths).  Host synchronisations per step:
the visible-list lengths, the routed-pair count, and the size all-gather.
"""
import torch

from . import distributed as D
from . import ops

# forward record: conic00 conic01 conic11 opacity | x y | r g b | depth radius(bits) minscale
_FWD_C = 12
# gradient record: conic00 conic01 conic11 opacity | x y | r g b | |x| |y| minscale
_BWD_C = 12


class _DistributedBatch(torch.autograd.Function):
    """One autograd node for the whole batch: raw parameters of this rank's
    shard in, summed band losses out.  Per camera only the shard's listed
    Gaussians (radius > 0, from the fused raw preprocess) are routed, packed
    and sent; the backward receives their gradient records into compact
    per-camera rows and runs the listed preprocess backward on them."""

    @staticmethod
    def forward(ctx, xyz, s_raw, q_raw, o_raw, dc, rest, setup):
        rasters, gts, strategies, group, lambda_dssim, reg_w = setup
        n_cams = len(rasters)
        rank = torch.distributed.get_rank(group)
        ws = torch.distributed.get_world_size(group)
        dev = xyz.device
        sh = ops.sh_layout(dc=dc, rest=rest)
        # 1. preprocess every camera (no host sync in between)
        pre = []
        for rs in rasters:
            m2, d, r, co, rgb, _, vlist, vcount, _, _, _ = ops.preprocess_forward_raw(
                xyz, s_raw, q_raw, o_raw.reshape(-1), sh, rs, None, want_reg=False, want_list=True)
            pre.append((m2, d, r, co, rgb, vlist, vcount))
        counts = torch.cat([p[6] for p in pre]).cpu().tolist() if n_cams else []
        # 2. pack the listed Gaussians' records and route them (one nonzero for the batch)
        recs, masks, ids_all = [], [], []
        for k, (m2, d, r, co, rgb, vlist, vcount) in enumerate(pre):
            ids = vlist[:counts[k]].to(torch.int64)
            ids_all.append(ids)
            m2c, rc = m2.index_select(0, ids), r.index_select(0, ids)
            smin = torch.exp(s_raw.index_select(0, ids)).min(dim=1).values
            recs.append(torch.cat([co.index_select(0, ids), m2c, rgb.index_select(0, ids), d.index_select(0, ids)[:, None],
                                   rc.view(torch.float32)[:, None], smin[:, None]], 1))
            st = strategies[k]
            dist_global = torch.tensor(st.division_pos, dtype=torch.int32, device=dev) * D.CONTEXT.TILE_X
            mk = ops.local2j_ids_bool(rs_h(rasters[k]), rs_w(rasters[k]), st.rank, st.world_size, m2c, rc,
                                      dist_global, False)
            # columns are the camera's renderers; widen to all ranks
            full = torch.zeros((mk.shape[0], ws), dtype=torch.bool, device=dev)
            full[:, torch.tensor(st.gpu_ids, device=dev)] = mk
            masks.append(full)
        offs = [0]
        for c in counts:
            offs.append(offs[-1] + c)
        records = torch.cat(recs, 0) if recs else torch.zeros((0, _FWD_C), device=dev)
        mask = torch.cat(masks, 0) if masks else torch.zeros((0, ws), dtype=torch.bool, device=dev)
        cam_of_row = torch.repeat_interleave(torch.arange(n_cams, device=dev), torch.tensor(counts, device=dev))
        nz = mask.nonzero()
        rows, dst = nz[:, 0], nz[:, 1]
        key = dst * n_cams + cam_of_row.index_select(0, rows)
        order = torch.sort(key, stable=True).indices
        send_rows = rows.index_select(0, order)
        sizes = torch.bincount(key, minlength=ws * n_cams).cpu().tolist()
        # send_ids[k][j]: compact positions of camera k's records for rank j
        send_ids = [[None] * ws for _ in range(n_cams)]
        pos = 0
        for j in range(ws):
            for k in range(n_cams):
                c = sizes[j * n_cams + k]
                send_ids[k][j] = send_rows[pos:pos + c] - offs[k]
                pos += c
        plan = D.plan_exchange(send_ids, n_cams, group)
        send = records.index_select(0, send_rows)
        recv_buf = torch.empty((sum(plan.recv_splits), _FWD_C), dtype=torch.float32, device=dev)
        torch.distributed.all_to_all_single(recv_buf, send, plan.recv_splits, plan.send_splits, group=group)
        recv = {}
        for k, parts in plan.recv_offsets.items():
            tot = sum(c for _, _, c in parts)
            if tot:
                recv[k] = torch.cat([recv_buf[s:s + c] for _, s, c in parts if c], 0)

        # 3. render and score the bands this rank owns
        loss_sum = torch.zeros((), dtype=torch.float32, device=dev)
        saved = {}
        for k in range(n_cams):
            st = strategies[k]
            if rank not in st.gpu_ids:
                continue
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            rec = recv.get(k)
            if rec is None:
                rec = torch.zeros((0, _FWD_C), dtype=torch.float32, device=dev)
            conic = rec[:, 0:4].contiguous()
            m2 = rec[:, 4:6].contiguous()
            rgb = rec[:, 6:9].contiguous()
            depth = rec[:, 9].contiguous()
            radii = rec[:, 10].contiguous().view(torch.int32)
            mins = rec[:, 11]
            y0t, y1t = st.row_range(rank)
            cl = st.get_compute_locally(device=dev)
            color, _, _, _, _, state = ops.render_forward(m2, depth, radii, conic, rgb, rs.bg, cl, H, W)
            y0, y1 = y0t * D.TILE, min(H, y1t * D.TILE)
            band = color[:, y0:y1, :]
            sums, partials = ops.loss_forward(band, gts[k])
            n3 = H * W * 3
            vis = (radii > 0).to(torch.float32)
            nvis = vis.sum()
            reg = (mins * vis).sum() / nvis.clamp(min=1.0)
            lk = ((1.0 - lambda_dssim) * (sums[0] / n3) + lambda_dssim * (1.0 - sums[1] / n3)).to(torch.float32)
            loss_sum = loss_sum + lk + reg_w * reg
            saved[k] = (state, m2, conic, rgb, cl, band, gts[k], partials, vis, nvis, (y0, y1), n3)
        ctx.setup = setup
        ctx.plan = plan
        ctx.saved = saved
        ctx.pre = [(p[0], p[2], p[5], p[6]) for p in pre]  # means2D, radii, vis_list, vis_count
        ctx.counts, ctx.offs = counts, offs
        ctx.send_rows = send_rows
        ctx.ids_all = ids_all
        ctx.save_for_backward(xyz, s_raw, q_raw, o_raw, dc, rest)
        return loss_sum

    @staticmethod
    def backward(ctx, g_loss):
        rasters, gts, strategies, group, lambda_dssim, reg_w = ctx.setup
        xyz, s_raw, q_raw, o_raw, dc, rest = ctx.saved_tensors
        n_cams = len(rasters)
        dev = xyz.device
        plan = ctx.plan
        # receiver: render backward of the owned bands -> 12-float gradient records
        send = torch.zeros((sum(plan.recv_splits), _BWD_C), dtype=torch.float32, device=dev)
        for k, (state, m2, conic, rgb, cl, band, gt, partials, vis, nvis, (y0, y1), n3) in ctx.saved.items():
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            scale = torch.stack([g_loss * (1.0 - lambda_dssim) / n3, -g_loss * lambda_dssim / n3]).float()
            g_band = ops.loss_backward(band, gt, partials, scale)
            dpix = torch.zeros((3, H, W), dtype=torch.float32, device=dev)
            dpix[:, y0:y1] = g_band
            rec16 = ops.render_backward(state, m2, conic, rgb, rs.bg, cl, dpix)
            g = torch.cat([rec16[:, 8:12], rec16[:, 0:2], rec16[:, 12:15], rec16[:, 4:6],
                           (g_loss * reg_w * vis / nvis.clamp(min=1.0))[:, None]], 1)
            pos = 0
            for _, s, c in plan.recv_offsets[k]:
                if c:
                    send[s:s + c] = g[pos:pos + c]
                    pos += c
        recv = torch.empty((sum(plan.send_splits), _BWD_C), dtype=torch.float32, device=dev)
        torch.distributed.all_to_all_single(recv, send, plan.send_splits, plan.recv_splits, group=group)
        # owner: one scatter-add into compact per-camera rows (aligned with the visible lists)
        acc = torch.zeros((ctx.offs[-1], _BWD_C), dtype=torch.float32, device=dev)
        acc.index_add_(0, ctx.send_rows, recv)
        sh = ops.sh_layout(dc=dc, rest=rest)
        M = rest.shape[1]
        g_xyz, g_s, g_q, g_o, g_dc, g_rest = (torch.zeros_like(t) for t in (xyz, s_raw, q_raw, o_raw, dc, rest))
        for k in range(n_cams):
            m2, r, vlist, vcount = ctx.pre[k]
            a = acc[ctx.offs[k]:ctx.offs[k + 1]]
            if ctx.counts[k] == 0:
                continue
            ops.preprocess_backward_raw(r, m2, xyz, s_raw, q_raw, o_raw.reshape(-1), sh, rasters[k],
                                        a[:, 4:6], a[:, 0:4], a[:, 6:9],
                                        (g_xyz, g_s, g_q, g_o, (g_dc, 3), (g_rest, max(M, 1) * 3)),
                                        vis_list=vlist, vis_count=vcount, accumulate=True,
                                        rows=ops.ROWS_UPSTREAM_BY_SLOT)
            # min-scale regulariser: to the smallest axis of exp(_scaling), chained through exp
            ids = ctx.ids_all[k]
            s_act = torch.exp(s_raw.detach().index_select(0, ids))
            mn, am = s_act.min(dim=1)
            g_s.index_put_((ids, am), a[:, 11] * mn, accumulate=True)
        return g_xyz, g_s, g_q, g_o, g_dc, g_rest, None


def rs_h(rs):
    return int(rs.image_height)


def rs_w(rs):
    return int(rs.image_width)


def batch_loss(shard_model, rasters, gts, strategies, group=None, lambda_dssim=0.2, reg_w=10.0):
    """Sum over the cameras this rank renders of the reference's per-camera
    loss.  Every rank must call ``.backward()`` on the result (the backward
    exchange is a collective), also when it renders nothing.
    ``shard_model`` = raw (xyz, _scaling, _rotation, _opacity, _features_dc,
    _features_rest) of this rank's shard; ``gts[k]`` is this rank's uint8
    ground-truth band of camera k (rows of its tile band) or None."""
    xyz, s_raw, q_raw, o_raw, dc, rest = shard_model
    return _DistributedBatch.apply(xyz, s_raw, q_raw, o_raw, dc, rest,
                                   (rasters, gts, strategies, group, lambda_dssim, reg_w))
