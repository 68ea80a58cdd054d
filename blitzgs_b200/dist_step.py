"""Distributed training step over N GPUs (one process per GPU, NCCL).

Per step, for a batch of cameras split into tile-row bands by
``start_strategy_final``:
  forward   every rank runs the fused raw preprocess (activations in the
            kernel) of its spatial shard for every camera; the same kernel
            writes each listed Gaussian's (radius > 0) 12-float exchange
            record and the ranks whose bands its tile rect overlaps (the
            reference's get_local2j_ids semantics); one all-gather of the
            per-destination counts sizes the exchange, a pack kernel fills
            the send buffer, and ONE all_to_all_single moves a record per
            (Gaussian, camera, destination); each rank unpacks every
            camera's received records with one kernel (which also sums the
            min-scale regulariser), renders its bands and forms the band
            loss on the device (L1 + SSIM + the regulariser over the
            received visible Gaussians, loss_distribution.py:303-322);
  backward  band loss / render backward on the receivers, the gradient
            records written straight into the send buffer by one kernel per
            camera, ONE reverse all_to_all_single of 12-float gradient
            records, one scatter-add into compact per-camera rows on the
            owners (aligned with each camera's visible list), and the listed
            preprocess backward accumulated into the shard's raw-parameter
            gradients.
These two all-to-alls and the tiny size all-gather are the only collectives
(the reference additionally all-gathers sizes with a blocking .cpu() and
runs a second all-to-all for radii/depths).  Host synchronisations per step:
the count all-gather, and one readback of every rendered camera's binning
totals.
"""
import torch

from . import densify as DZ
from . import distributed as D
from . import ops
from torch.autograd.graph import get_gradient_edge

from .step import _GRADS, _zero_fill_async, _zero_fill_wait

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
        rasters, gts, strategies, group, lambda_dssim, reg_w, densify = setup
        n_cams = len(rasters)
        rank = torch.distributed.get_rank(group)
        ws = torch.distributed.get_world_size(group)
        dev = xyz.device
        sh = ops.sh_layout(dc=dc, rest=rest)
        # 1. preprocess every camera in one call; the kernels also write each
        #    listed Gaussian's exchange record, its destination ranks and the
        #    per-destination counts (no host synchronisation in between).  The
        #    visible lists are in ascending index order.
        P = xyz.shape[0]
        gx = D.CONTEXT.TILE_X
        table, tnp = _pinned_table(n_cams, ws)  # tile interval [lo, hi) of every rank, per camera
        for k, st in enumerate(strategies):
            for r_local, g in enumerate(st.gpu_ids):
                tnp[k, 0, g] = st.division_pos[r_local] * gx
                tnp[k, 1, g] = st.division_pos[r_local + 1] * gx
        table_dev = table[:n_cams].to(dev, non_blocking=True)
        cnt = torch.zeros((n_cams, 1 + ws), dtype=torch.int32, device=dev)  # list length | rows per rank
        # one allocation per buffer kind for the whole batch; camera k's rows start at k*Pc
        Pc = (max(P, 1) + 3) // 4 * 4
        b_m2 = torch.empty((n_cams, Pc, 2), dtype=torch.float32, device=dev)
        b_depth = torch.empty((n_cams, Pc), dtype=torch.float32, device=dev)
        b_radii = torch.empty((n_cams, Pc), dtype=torch.int32, device=dev)
        b_co = torch.empty((n_cams, Pc, 4), dtype=torch.float32, device=dev)
        b_rgb = torch.empty((n_cams, Pc, 3), dtype=torch.float32, device=dev)
        b_list = torch.empty((n_cams, Pc), dtype=torch.int32, device=dev)
        b_mask = torch.empty((n_cams, Pc), dtype=torch.int32, device=dev)
        b_rec = torch.empty((n_cams, Pc, _FWD_C), dtype=torch.float32, device=dev)
        cams = _camera_arrays(rasters)
        ops.preprocess_forward_raw_batch(xyz, s_raw, q_raw, o_raw.reshape(-1), sh, rasters, cams, Pc,
                                         (b_m2, b_depth, b_radii, b_co, b_rgb, b_list), cnt,
                                         exchange=(table_dev, b_rec, b_mask))
        if densify is not None:
            for k in range(n_cams):
                DZ.update_max_radii(densify, b_radii[k, :P])
        # 2. one all-gather of every rank's counts: the only host synchronisation
        #    before the render (it sizes the all-to-all on every rank)
        gdev = dev if torch.distributed.get_backend(group) == "nccl" else torch.device("cpu")
        allc = torch.empty((ws * n_cams, 1 + ws), dtype=torch.int32, device=gdev)
        torch.distributed.all_gather_into_tensor(allc, cnt.to(gdev), group=group)
        allc = allc.view(ws, n_cams, 1 + ws).cpu().tolist()
        counts, plan, offs, dest_off = D.exchange_layout(allc, rank, ws, n_cams)
        n_send = sum(plan.send_splits)
        send = torch.empty((max(n_send, 1), _FWD_C), dtype=torch.float32, device=dev)
        send_row = torch.empty((max(n_send, 1),), dtype=torch.int32, device=dev)
        ops.exchange_pack_batch(counts, Pc, b_rec, b_mask, dest_off, offs[:-1], send, send_row)
        recv_buf = torch.empty((sum(plan.recv_splits), _FWD_C), dtype=torch.float32, device=dev)
        torch.distributed.all_to_all_single(recv_buf, send[:n_send], plan.recv_splits, plan.send_splits, group=group)
        # 3. render and score the bands this rank owns.  Per camera: unpack
        #    the received records (and the regulariser sums) in one kernel,
        #    count tile instances; then one readback of every camera's totals
        #    sizes all the binning buffers at once.
        mine = [k for k in range(n_cams) if rank in strategies[k].gpu_ids]
        nm = len(mine)
        totals = torch.zeros((max(nm, 1), 2), dtype=torch.int64, device=dev)
        regs = torch.zeros((max(nm, 1), 2), dtype=torch.float64, device=dev)
        staged = []
        for i, k in enumerate(mine):
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            segs = [(s, c) for _, s, c in plan.recv_offsets.get(k, []) if c]
            conic, m2, rgb, depth, radii = ops.exchange_unpack(recv_buf, segs, regs[i])
            cl = _band_mask(strategies[k], rank, dev)
            counts_k = torch.empty((max(m2.shape[0], 1),), dtype=torch.int32, device=dev)
            ops.render_count(m2, radii, cl, H, W, counts_k, totals[i])
            staged.append((k, segs, conic, m2, rgb, depth, radii, cl, counts_k))
        # one camera with known buffer sizes (the usual case at one view per
        # GPU): render_forward issues its binning before it reads the totals
        # back (and checks the scan status words); otherwise one readback of
        # every camera's totals first
        spec = nm == 1 and ops.render_caps_known(dev, int(rasters[mine[0]].image_height),
                                                 int(rasters[mine[0]].image_width))
        tot_host = [None] * nm
        if not spec:
            status = ops.queue_scan_status(dev)
            tot_host = totals.cpu().tolist() if nm else []
            if not nm:
                torch.cuda.current_stream(dev).synchronize()
            ops.check_scan_status(status)
        losses = []
        saved = {}
        for i, (k, segs, conic, m2, rgb, depth, radii, cl, counts_k) in enumerate(staged):
            rs = rasters[k]
            H, W = int(rs.image_height), int(rs.image_width)
            color, _, _, _, _, state = ops.render_forward(m2, depth, radii, conic, rgb, rs.bg, cl, H, W,
                                                          counts=counts_k, totals=totals[i],
                                                          totals_host=tot_host[i], caps_update=True)
            y0t, y1t = strategies[k].row_range(rank)
            y0, y1 = y0t * D.TILE, min(H, y1t * D.TILE)
            band = color[:, y0:y1, :]
            sums, partials = ops.loss_forward(band, gts[k])
            n3 = H * W * 3
            out = ops.loss_combine(sums, regs[i], lambda_dssim, n3, reg_w)
            losses.append(out[0])
            saved[k] = (state, m2, conic, rgb, cl, band, gts[k], partials, radii, out, (y0, y1), n3, segs)
        if losses:
            loss_sum = losses[0] if len(losses) == 1 else torch.stack(losses).sum()
        else:
            loss_sum = torch.zeros((), dtype=torch.float32, device=dev)
        ctx.setup = setup
        ctx.plan = plan
        ctx.saved = saved
        ctx.pre = (b_m2, b_radii, b_list, cnt, Pc, cams)
        ctx.counts, ctx.offs = counts, offs
        ctx.send_rows = send_row[:n_send].to(torch.int64)
        params = (xyz, s_raw, q_raw, o_raw, dc, rest)
        ctx.params = params if all(t.is_leaf and t.requires_grad for t in params) else None
        ctx.nodes = [get_gradient_edge(t).node for t in params] if ctx.params is not None else None
        ctx.save_for_backward(xyz, s_raw, q_raw, o_raw, dc, rest)
        return loss_sum

    @staticmethod
    def backward(ctx, g_loss):
        rasters, gts, strategies, group, lambda_dssim, reg_w, densify = ctx.setup
        xyz, s_raw, q_raw, o_raw, dc, rest = ctx.saved_tensors
        n_cams = len(rasters)
        dev = xyz.device
        plan = ctx.plan
        # the shard's dense gradients are zero except at listed rows: written in
        # place into .grad (only the rows written before are zeroed again), or
        # zero-filled on a side stream while the render backward (issue
        # bound) runs
        inplace = _GRADS.targets(ctx.params, ctx.nodes) if ctx.params is not None else None
        if inplace is not None:
            grads = [e["t"] for e in inplace[0]]
        else:
            grads = [torch.empty_like(t) for t in (xyz, s_raw, q_raw, o_raw, dc, rest)]
            _zero_fill_async(grads)
        try:
            # receiver: render backward of the owned bands -> 12-float gradient records
            send = torch.zeros((sum(plan.recv_splits), _BWD_C), dtype=torch.float32, device=dev)
            for k, (state, m2, conic, rgb, cl, band, gt, partials, radii, out, (y0, y1), n3, segs) in \
                    ctx.saved.items():
                rs = rasters[k]
                H, W = int(rs.image_height), int(rs.image_width)
                scales = ops.loss_combine_backward(g_loss, None, None, out, lambda_dssim, n3, reg_w)
                g_band = ops.loss_backward(band, gt, partials, scales[0:2])
                if y0 == 0 and y1 == H:
                    dpix = g_band
                else:
                    dpix = torch.zeros((3, H, W), dtype=torch.float32, device=dev)
                    dpix[:, y0:y1] = g_band
                rec16 = ops.render_backward(state, m2, conic, rgb, rs.bg, cl, dpix)
                ops.grad_records_pack(rec16, radii, scales[2:3], segs, send)
            recv = torch.empty((sum(plan.send_splits), _BWD_C), dtype=torch.float32, device=dev)
            torch.distributed.all_to_all_single(recv, send, plan.send_splits, plan.recv_splits, group=group)
            # owner: one scatter-add into compact per-camera rows (aligned with the visible lists)
            acc = torch.zeros((max(ctx.offs[-1], 1), _BWD_C), dtype=torch.float32, device=dev)
            acc.index_add_(0, ctx.send_rows, recv)
            sh = ops.sh_layout(dc=dc, rest=rest)
            M = rest.shape[1]
            g_xyz, g_s, g_q, g_o, g_dc, g_rest = grads
        finally:
            # every exit orders this stream after the fill before the grads are used or freed
            if inplace is None:
                _zero_fill_wait()
        b_m2, b_radii, b_list, cnt, Pc, cams = ctx.pre
        if densify is not None:
            for k in range(n_cams):
                if ctx.counts[k]:
                    # viewspace gradient of the owner's screen means: summed over the receivers
                    DZ.accumulate_grad(densify, b_list[k, :ctx.counts[k]].to(torch.int64),
                                       acc[ctx.offs[k]:ctx.offs[k + 1], 4:6])
        ops.preprocess_backward_raw_batch(b_radii, b_m2, b_list, cnt, Pc, xyz, s_raw, q_raw, o_raw.reshape(-1), sh,
                                          rasters, cams, acc, ctx.offs[:-1],
                                          (g_xyz, g_s, g_q, g_o, (g_dc, 3), (g_rest, max(M, 1) * 3)))
        if inplace is not None:
            rows = [b_list[k, :ctx.counts[k]] for k in range(n_cams) if ctx.counts[k]]
            rows = torch.cat(rows) if rows else torch.zeros((0,), dtype=torch.int32, device=dev)
            _GRADS.written(ctx.params, inplace[0], (rows, rows.numel()), fresh=not inplace[1])
            return None, None, None, None, None, None, None
        return g_xyz, g_s, g_q, g_o, g_dc, g_rest, None


_TABLE = {}
_MASKS = {}


def _band_mask(strategy, rank, dev):
    """The rank's compute_locally tile mask of a camera (rows of its band),
    cached per (device, band): bands repeat from step to step."""
    y0, y1 = strategy.row_range(rank)
    key = (dev.index, y0, y1, D.CONTEXT.TILE_Y, D.CONTEXT.TILE_X)
    m = _MASKS.get(key)
    if m is None:
        if len(_MASKS) > 4096:
            _MASKS.clear()
        m = _MASKS[key] = strategy.get_compute_locally(device=dev)
    return m


_CAMS = {}


def _camera_arrays(rasters):
    """(viewmatrices [n,16], projmatrices [n,16], campos [n,3]) of the batch,
    cached per batch of camera tensors: the key holds the tensors themselves
    (so their ids cannot be reused while cached) and their version counters
    (an in-place change of a matrix misses the cache)."""
    key = tuple((id(t), t._version) for r in rasters for t in (r.viewmatrix, r.projmatrix, r.campos))
    hit = _CAMS.get(key)
    if hit is not None:
        return hit[1]
    views = torch.stack([r.viewmatrix.reshape(16) for r in rasters])
    projs = torch.stack([r.projmatrix.reshape(16) for r in rasters])
    campos = torch.stack([r.campos.reshape(3) for r in rasters])
    out = (views.float().contiguous(), projs.float().contiguous(), campos.float().contiguous())
    if len(_CAMS) > 256:
        _CAMS.clear()
    _CAMS[key] = ([t for r in rasters for t in (r.viewmatrix, r.projmatrix, r.campos)], out)
    return out


def _pinned_table(n_cams, ws):
    """Reused pinned host buffer [n_cams, 2, ws] of per-rank tile intervals
    (zeros: a rank that renders none of a camera).  Reuse is safe: every step
    synchronises with the host (the count all-gather) after its copy."""
    t = _TABLE.get(ws)
    if t is None or t[0].shape[0] < n_cams:
        buf = torch.zeros((max(n_cams, 8), 2, ws), dtype=torch.int32).pin_memory()
        t = _TABLE[ws] = (buf, buf.numpy())  # numpy view: element writes cost far less than tensor indexing
    t[1][:n_cams] = 0
    return t


def batch_loss(shard_model, rasters, gts, strategies, group=None, lambda_dssim=0.2, reg_w=10.0, densify=None):
    """Sum over the cameras this rank renders of the reference's per-camera
    loss.  Every rank must call ``.backward()`` on the result (the backward
    exchange is a collective), also when it renders nothing.
    ``shard_model`` = raw (xyz, _scaling, _rotation, _opacity, _features_dc,
    _features_rest) of this rank's shard; ``gts[k]`` is this rank's uint8
    ground-truth band of camera k (rows of its tile band) or None.
    ``densify`` (a densify.DensificationStats over the shard) receives the
    densification statistics of every camera of the batch."""
    xyz, s_raw, q_raw, o_raw, dc, rest = shard_model
    return _DistributedBatch.apply(xyz, s_raw, q_raw, o_raw, dc, rest,
                                   (rasters, gts, strategies, group, lambda_dssim, reg_w, densify))
