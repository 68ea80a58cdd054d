"""The multi-GPU step's orchestration on gloo ranks (CPU): blitzgs_b200.dist_step
forward and backward, the workload division, the exchange layout and both
all-to-alls, the scatter-back, the in-place gradient buffers and the
densification statistics, at world sizes 1-8.

The native kernels are replaced by CPU stand-ins with a simple model of
their contracts (one 12-float record per listed Gaussian and destination,
records unpacked in receive order, one-pixel splats, a linear band loss, a
per-row gradient record), in arithmetic that is exact in float32.  What runs
for real is the host code between them, so the test checks that every
Gaussian a camera's band needs reaches the rank that renders it and that its
gradient comes back to the right row of the right shard: the loss and every
Gaussian's gradient at N ranks must equal the one-rank run."""
import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, W = 96, 64  # 6 x 4 tiles
P_TOTAL = 600


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# ---------------------------------------------------------------------------
# CPU stand-ins of the native ops dist_step calls
# ---------------------------------------------------------------------------

def _project(xyz, k):
    """Camera k's screen position of each Gaussian: x = X W, y = (Y + k/16) H."""
    return xyz[:, 0] * W, (xyz[:, 1] + k / 16.0) * H


def _fake_preprocess_batch(xyz, s_raw, q_raw, o_raw, sh, rasters, cams, Pc, out, cnt, exchange=None):
    m2, depth, radii, conic, rgb, vlist = out
    table, rec, mask = exchange
    dc = sh[0].reshape(-1, 3)
    P = xyz.shape[0]
    if P == 0:
        return
    gx = (W + 15) // 16
    for k, r in enumerate(rasters):
        x, y = _project(xyz.detach(), r.k)
        listed = (x >= 0) & (x < W) & (y >= 0) & (y < H) & (o_raw.detach() > -1.5)
        ids = listed.nonzero(as_tuple=True)[0]
        L = ids.numel()
        radii[k, :P] = listed.to(torch.int32)
        m2[k, :P, 0], m2[k, :P, 1] = x, y
        vlist[k, :L] = ids.to(torch.int32)
        ty = torch.floor(y[ids] / 16).to(torch.int64)
        r0, r1 = (ty - 1).clamp(min=0), (ty + 2).clamp(max=(H + 15) // 16)
        bits = torch.zeros(L, dtype=torch.int32)
        for j in range(table.shape[-1]):
            lo, hi = int(table[k, 0, j]), int(table[k, 1, j])
            bits |= (((r0 * gx) < hi) & (lo < (r1 * gx))).to(torch.int32) << j
        mask[k, :L] = bits
        rec[k, :L] = 0
        rec[k, :L, 3] = o_raw.detach()[ids]
        rec[k, :L, 4], rec[k, :L, 5] = x[ids], y[ids]
        rec[k, :L, 6:9] = dc.detach()[ids]
        rec[k, :L, 9] = xyz.detach()[ids, 2]
        rec[k, :L, 10] = torch.ones(L, dtype=torch.int32).view(torch.float32)
        rec[k, :L, 11] = s_raw.detach()[ids].min(dim=1).values
        cnt[k, 0] = L
        for j in range(table.shape[-1]):
            cnt[k, 1 + j] = int(((bits >> j) & 1).sum())


def _fake_pack_batch(counts, Pc, rec, mask, dest_off, row_base, send, send_row):
    for k, L in enumerate(counts):
        for j in range(len(dest_off[k])):
            rows = ((mask[k, :L] >> j) & 1).nonzero(as_tuple=True)[0]
            o = dest_off[k][j]
            send[o:o + rows.numel()] = rec[k, rows]
            send_row[o:o + rows.numel()] = (row_base[k] + rows).to(torch.int32)


def _fake_unpack(recv, segs, reg):
    rows = torch.cat([recv[s:s + c] for s, c in segs]) if segs else torch.zeros((0, 12))
    radii = rows[:, 10].contiguous().view(torch.int32)
    vis = radii > 0
    reg[0] += rows[vis, 11].double().sum()
    reg[1] += float(vis.sum())
    return rows[:, 0:4], rows[:, 4:6], rows[:, 6:9], rows[:, 9], radii


def _pixels(m2):
    return torch.floor(m2[:, 1]).long().clamp(0, H - 1), torch.floor(m2[:, 0]).long().clamp(0, W - 1)


def _fake_render_forward(m2, depth, radii, conic, rgb, bg, cl, H_, W_, counts=None, totals=None,
                         totals_host=None, caps_update=False):
    color = torch.zeros((3, H, W), dtype=torch.float32)
    py, px = _pixels(m2)
    inside = cl[py // 16, px // 16]
    for n in inside.nonzero(as_tuple=True)[0].tolist():
        color[:, py[n], px[n]] += rgb[n]
    return color, None, None, None, None, (py, px, inside)


def _fake_render_backward(state, m2, conic, rgb, bg, cl, dpix):
    py, px, inside = state
    rec16 = torch.zeros((m2.shape[0], 16), dtype=torch.float32)
    d = dpix[:, py, px].t() * inside[:, None]
    rec16[:, 12:15] = d
    rec16[:, 0], rec16[:, 1] = d.sum(1), 2 * d.sum(1)
    rec16[:, 4:6] = rec16[:, 0:2].abs()
    return rec16


def _fake_grad_pack(rec16, radii, reg_scale, segs, send):
    n = 0
    for s, c in segs:
        r = rec16[n:n + c]
        send[s:s + c, 0:4] = r[:, 8:12]
        send[s:s + c, 4:6] = r[:, 0:2]
        send[s:s + c, 6:9] = r[:, 12:15]
        send[s:s + c, 9:11] = r[:, 4:6]
        send[s:s + c, 11] = torch.where(radii[n:n + c] > 0, reg_scale[0], torch.zeros(()))
        n += c


def _fake_loss_forward(band, gt):
    return torch.stack([(band.double() * gt.double()).sum(), torch.zeros((), dtype=torch.float64)]), None


def _fake_loss_combine(sums, reg, lambda_dssim, n3, reg_w):
    cnt = max(float(reg[1]), 1.0)
    loss = float(sums[0]) + reg_w * float(reg[0]) / cnt
    return torch.tensor([loss, float(sums[0]), 0.0, float(reg[0]), cnt], dtype=torch.float32)


def _fake_loss_combine_backward(g_loss, g_l1, g_ss, out, lambda_dssim, n3, reg_w):
    g = float(g_loss)
    return torch.tensor([g, 0.0, g * reg_w / float(out[4])], dtype=torch.float32)


def _fake_loss_backward(band, gt, partials, scales):
    return (scales[0] * gt.float()).contiguous()


def _fake_preprocess_backward_batch(radii, m2, vlist, cnt, Pc, xyz, s_raw, q_raw, o_raw, sh, rasters, cams, acc,
                                    row0, out):
    g_xyz, g_s, g_q, g_o, (g_dc, _), _ = out
    for k in range(len(rasters)):
        L = int(cnt[k, 0])
        if L == 0:
            continue
        rows = acc[row0[k]:row0[k] + L]
        ids = vlist[k, :L].long()
        g_dc.view(-1, 3).index_add_(0, ids, rows[:, 6:9])
        g_xyz[:, 0].index_add_(0, ids, rows[:, 4] * W)
        g_xyz[:, 1].index_add_(0, ids, rows[:, 5] * H)
        arg = s_raw.detach()[ids].argmin(dim=1)
        g_s.view(-1).index_add_(0, ids * 3 + arg, rows[:, 11])


def _install_fakes():
    from blitzgs_b200 import ops
    torch.Tensor.pin_memory = lambda self: self  # no CUDA here: pinned buffers are plain host memory
    ops.preprocess_forward_raw_batch = _fake_preprocess_batch
    ops.exchange_pack_batch = _fake_pack_batch
    ops.exchange_unpack = _fake_unpack
    ops.render_count = lambda m2, radii, cl, H_, W_, counts, totals: totals.copy_(
        torch.tensor([m2.shape[0], m2.shape[0]]))
    ops.render_caps_known = lambda dev, H_, W_: False
    ops.queue_scan_status = lambda dev: None
    ops.check_scan_status = lambda status: None
    ops.render_forward = _fake_render_forward
    ops.render_backward = _fake_render_backward
    ops.grad_records_pack = _fake_grad_pack
    ops.loss_forward = _fake_loss_forward
    ops.loss_combine = _fake_loss_combine
    ops.loss_combine_backward = _fake_loss_combine_backward
    ops.loss_backward = _fake_loss_backward
    ops.preprocess_backward_raw_batch = _fake_preprocess_backward_batch
    ops.zero_fill_async = lambda ts: [t.zero_() for t in ts]
    ops.zero_fill_wait = lambda: None
    ops.zero_rows = lambda ts, rows, n: [t.view(t.shape[0], -1).index_fill_(0, rows[:n].long(), 0.0) for t in ts]


# ---------------------------------------------------------------------------
# one rank
# ---------------------------------------------------------------------------

def _scene():
    g = torch.Generator().manual_seed(7)
    xyz = torch.rand(P_TOTAL, 3, generator=g)
    # values on a 1/8 grid: every sum the stand-ins form is exact in float32
    s_raw = torch.floor(torch.rand(P_TOTAL, 3, generator=g) * 16) / 8 - 1
    q_raw = torch.rand(P_TOTAL, 4, generator=g)
    o_raw = torch.floor(torch.rand(P_TOTAL, 1, generator=g) * 32) / 8 - 2
    dc = torch.floor(torch.rand(P_TOTAL, 1, 3, generator=g) * 16) / 8
    rest = torch.zeros(P_TOTAL, 15, 3)
    return xyz, s_raw, q_raw, o_raw, dc, rest


def _worker(rank, ws, n_cams, reg_w, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        _install_fakes()
        from blitzgs_b200 import distributed as D
        from blitzgs_b200 import dist_step as DS
        D.init_context(rank, ws, H, W, group=None, bsz=n_cams)
        scene = _scene()
        lo_hi = [(int(c[0]), int(c[-1]) + 1) for c in torch.tensor_split(torch.arange(P_TOTAL), ws)]
        lo, hi = lo_hi[rank]
        model = [t[lo:hi].clone().requires_grad_(True) for t in scene]
        cams = [SimpleNamespace(uid=k) for k in range(n_cams)]
        rasters = [SimpleNamespace(k=k, image_height=H, image_width=W, viewmatrix=torch.eye(4) * (k + 1),
                                   projmatrix=torch.eye(4), campos=torch.zeros(3), bg=torch.zeros(3), sh_degree=3,
                                   scale_modifier=1.0, tanfovx=1.0, tanfovy=1.0) for k in range(n_cams)]
        g = torch.Generator().manual_seed(11)
        gt_full = [torch.randint(0, 4, (3, H, W), generator=g, dtype=torch.uint8) for _ in range(n_cams)]
        history = D.DivisionStrategyHistoryFinal(cams, ws, rank)
        from blitzgs_b200.densify import DensificationStats
        stats = DensificationStats(hi - lo, "cpu")
        results = []
        for step in range(3):
            strategies, _ = D.start_strategy_final(cams, history)
            gts = []
            for k, st in enumerate(strategies):
                rr = st.row_range(rank)
                gts.append(None if rr is None else gt_full[k][:, rr[0] * 16:min(H, rr[1] * 16)])
            if step < 2:
                for p in model:
                    p.grad = None  # fresh buffers in step 0, reused (earlier rows zeroed) in step 1
            # step 2 accumulates into the gradients of step 1
            loss = DS.batch_loss(model, rasters, gts, strategies, reg_w=reg_w, densify=stats)
            loss.backward()
            # numpy copies: they travel through the queue by value (a shared
            # tensor would vanish with this process)
            results.append((float(loss.detach()), [p.grad.numpy().copy() for p in model]))
        dens = [t.numpy().copy() for t in (stats.max_radii2D, stats.xyz_gradient_accum, stats.denom)]
        q.put((rank, "ok", lo, hi, (results, dens)))
    except BaseException as ex:  # report to the parent
        import traceback
        q.put((rank, repr(ex) + traceback.format_exc(), 0, 0, None))
    finally:
        dist.destroy_process_group()


def _run(ws, n_cams, reg_w):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, n_cams, reg_w, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] == "ok", r[1]
    # per step: total loss over ranks, each gradient tensor assembled over the
    # shards; and the densification statistics assembled likewise
    steps = []
    for s in range(3):
        loss = sum(r[4][0][s][0] for r in res)
        grads = [torch.zeros_like(t) for t in _scene()]
        for r in res:
            for gt, g in zip(grads, r[4][0][s][1]):
                gt[r[2]:r[3]] = torch.from_numpy(g)
        steps.append((loss, grads))
    dens = [torch.zeros(P_TOTAL), torch.zeros(P_TOTAL, 1), torch.zeros(P_TOTAL, 1)]
    for r in res:
        for d, v in zip(dens, r[4][1]):
            d[r[2]:r[3]] = torch.from_numpy(v)
    return steps, dens


_SINGLE = {}


@pytest.mark.parametrize("ws,n_cams,reg_w", [
    (2, 2, 10.0),   # one whole view per rank
    (3, 3, 10.0),
    (8, 8, 10.0),
    (2, 4, 10.0),   # two whole views per rank
    (4, 2, 0.0),    # each view split into two tile-row bands
])
def test_multi_rank_step_equals_one_rank(ws, n_cams, reg_w):
    key = (n_cams, reg_w)
    if key not in _SINGLE:
        _SINGLE[key] = _run(1, n_cams, reg_w)
    want, want_dens = _SINGLE[key]
    got, got_dens = _run(ws, n_cams, reg_w)
    for s in range(3):
        assert got[s][0] == pytest.approx(want[s][0], rel=1e-6), (s, got[s][0], want[s][0])
        for name, a, b in zip(("xyz", "scaling", "rotation", "opacity", "dc", "rest"), got[s][1], want[s][1]):
            assert torch.allclose(a, b, rtol=1e-6, atol=1e-6), (s, name, (a - b).abs().max())
    # the step saw work: gradients reach the colours and positions, and step 2 accumulated
    assert float(want[0][1][4].abs().sum()) > 0 and float(want[0][1][0].abs().sum()) > 0
    assert torch.allclose(want[2][1][4], 2 * want[1][1][4])
    # densification statistics over the three steps: max_radii2D, the summed
    # norm of each Gaussian's viewspace gradient (on N ranks the owner's sum
    # over the receivers) and the visibility count
    for name, a, b in zip(("max_radii2D", "xyz_gradient_accum", "denom"), got_dens, want_dens):
        assert torch.allclose(a, b, rtol=1e-6, atol=1e-6), (name, (a - b).abs().max())
    assert 0 < float(want_dens[2].max()) <= 3 * n_cams  # at most once per camera and step
    assert float(want_dens[1].sum()) > 0
