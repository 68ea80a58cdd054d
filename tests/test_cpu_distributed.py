"""Multi-rank host logic on CPU: the exchange layout of the multi-GPU step
(blitzgs_b200.distributed.exchange_layout with the count all-gather, the
all-to-alls and the scatter-back, on gloo ranks; the GPU pack kernel is
restated on the CPU and checked against the same rule on a GPU) and the
workload-division policy (pure host code, checked against a restatement of
gaussian_renderer/workload_division.py:785-873)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blitzgs_b200 import distributed as D


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


N_CAMS = 3
# Gaussians per rank (contiguous z-order shards: global id = shard offset +
# local index); rank 3 holds an empty shard
SHARD = [40, 47, 33, 0, 29, 51, 18, 36]


def _rank_data(rank, ws):
    """One rank's output of the batched preprocess, restated on the CPU: per
    camera its visible list (ascending local index), each listed Gaussian's
    12-float record (global id, camera, source rank, ...) and destination
    mask, and the count row [list length, rows per rank]."""
    P = SHARD[rank]
    base = sum(SHARD[:rank])
    g = torch.Generator().manual_seed(100 + rank)
    cams = []
    for k in range(N_CAMS):
        listed = (torch.rand(P, generator=g) < 0.7).nonzero(as_tuple=True)[0]
        L = len(listed)
        rec = torch.zeros(L, 12)
        rec[:, 0] = (base + listed).float()
        rec[:, 1] = float(k)
        rec[:, 2] = float(rank)
        rec[:, 3:] = torch.rand(L, 9, generator=g)
        mask = torch.zeros(L, dtype=torch.int64)
        for j in range(ws):
            m = torch.rand(L, generator=g) < (0.2 + 0.1 * (j % 7))
            if k == 2 and j == 1:
                m[:] = False  # a camera sends nothing to rank 1
            mask |= m.to(torch.int64) << j
        cnt = [L] + [int(((mask >> j) & 1).sum()) for j in range(ws)]
        cams.append((listed, rec, mask, cnt))
    return cams


def _pack(cams, dest_off, n_send, ws):
    """CPU statement of blitz_exchange_pack_batch: camera k's rows routed to
    rank j, in list order, from dest_off[k][j]; send_row = offs[k] + slot."""
    send = torch.zeros(n_send, 12)
    send_row = torch.full((n_send,), -1, dtype=torch.int64)
    row0 = 0
    for k, (listed, rec, mask, cnt) in enumerate(cams):
        for j in range(ws):
            rows = ((mask >> j) & 1).nonzero(as_tuple=True)[0]
            o = dest_off[k][j]
            send[o:o + len(rows)] = rec[rows]
            send_row[o:o + len(rows)] = row0 + rows
        row0 += len(listed)
    return send, send_row


def _worker(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        cams = _rank_data(rank, ws)
        # the count all-gather and layout of dist_step, on gloo
        cnt = torch.tensor([c[3] for c in cams], dtype=torch.int32)
        allc = torch.empty((ws * N_CAMS, 1 + ws), dtype=torch.int32)
        dist.all_gather_into_tensor(allc, cnt)
        allc = allc.view(ws, N_CAMS, 1 + ws).tolist()
        counts, plan, offs, dest_off = D.exchange_layout(allc, rank, ws, N_CAMS)
        assert counts == [c[3][0] for c in cams]
        n_send = sum(plan.send_splits)
        send, send_row = _pack(cams, dest_off, n_send, ws)
        assert bool((send_row >= 0).all()), "every send row is written exactly once"
        recv = torch.empty((sum(plan.recv_splits), 12))
        dist.all_to_all_single(recv, send, plan.recv_splits, plan.send_splits)
        # receiver: camera k = its runs in recv_offsets order; the rows are exactly the
        # Gaussians routed here, in ascending global id (source rank, then local index)
        everyone = [_rank_data(i, ws) for i in range(ws)]
        for k in range(N_CAMS):
            segs = [(s_, c) for _, s_, c in plan.recv_offsets[k] if c]
            got = torch.cat([recv[s_:s_ + c] for s_, c in segs]) if segs else torch.zeros(0, 12)
            exp = []
            for i in range(ws):
                listed, rec, mask, _ = everyone[i][k]
                exp.append(rec[((mask >> rank) & 1).bool()])
            exp = torch.cat(exp)
            assert torch.equal(got, exp), (rank, k)
            ids = got[:, 0]
            assert bool((ids[1:] > ids[:-1]).all()), "receive order is ascending global id"
            assert (k in plan.my_cams) == (len(got) > 0)
        # backward: the gradient rows go back along the same layout and are summed
        # into the owner's compact per-camera rows (offs[k] + slot) through send_row
        g_send = recv[:, :3] * 2 + 1 + rank
        g_recv = torch.empty((n_send, 3))
        dist.all_to_all_single(g_recv, g_send, plan.send_splits, plan.recv_splits)
        acc = torch.zeros((offs[-1], 3))
        acc.index_add_(0, send_row, g_recv)
        for k, (listed, rec, mask, _) in enumerate(cams):
            e = torch.zeros(len(listed), 3)
            for j in range(ws):
                sel = ((mask >> j) & 1).bool()
                e[sel] += rec[sel, :3] * 2 + 1 + j
            assert torch.allclose(acc[offs[k]:offs[k + 1]], e), (rank, k)
        q.put((rank, "ok"))
    except BaseException as ex:  # report to the parent
        import traceback
        q.put((rank, repr(ex) + traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2, 3, 4, 8])
def test_exchange_layout_round_trip_gloo(ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(res) == [(r, "ok") for r in range(ws)], res


def _ref_division(heur, n_rows, ws, coeff):
    pref = torch.cumsum(heur, 0)
    thr = torch.arange(1, ws) * (pref[-1] / ws)
    pos = [0] + torch.searchsorted(pref, thr, right=True).tolist() + [len(heur)]
    for i in range(1, len(pos) - 1):
        if pos[i] % n_rows + coeff >= n_rows:
            pos[i] = pos[i] // n_rows * n_rows + n_rows
        elif pos[i] % n_rows - coeff <= 0:
            pos[i] = pos[i] // n_rows * n_rows
    return pos


class _Cam:
    def __init__(self, uid):
        self.uid = uid


@pytest.mark.parametrize("ws,bsz", [(1, 1), (2, 2), (4, 4), (8, 8), (4, 2), (8, 3)])
def test_start_strategy_matches_reference_policy(ws, bsz):
    D.init_context(0, ws, 864, 1152, bsz=bsz, border_divpos_coeff=1.0, local_sampling=False)
    cams = [_Cam(i) for i in range(bsz)]
    hist = D.DivisionStrategyHistoryFinal(cams, ws, 0)
    strategies, tasks = D.start_strategy_final(cams, hist)
    pos = _ref_division(torch.ones(54 * bsz), 54, ws, 1.0)
    # every rank's tasks are exactly the division's intersections with each camera
    for g in range(ws):
        exp = []
        for idx in range(bsz):
            off = idx * 54
            l, r = pos[g], pos[g + 1]
            if r <= off or off + 54 <= l:
                continue
            exp.append((idx, max(l, off) - off, min(r, off + 54) - off))
        assert tasks[g] == exp
    for st in strategies:
        assert st.division_pos[0] == 0 and st.division_pos[-1] == 54
    if bsz == ws:
        # an even split at view boundaries: one whole view per rank (never rebalanced at <=1080p)
        assert all(len(t) == 1 and t[0][1:] == (0, 54) for t in tasks)


def test_division_pos_heuristic_and_asserts():
    D.init_context(0, 2, 864, 1152)
    h = torch.tensor([1.0, 1.0, 1.0, 5.0, 1.0, 1.0])
    assert D.division_pos_heuristic(h, 6, 2, right=True) == [0, 3, 6]
    with pytest.raises(AssertionError):
        D.DivisionStrategyFinal(None, 2, [0, 1], [0, 30, 20], [(0, 30), (30, 20)])


def test_finish_strategy_skips_rebalance_at_1080p_or_less():
    D.init_context(0, 2, 864, 1152, bsz=2, adjust_strategy_warmp_iterations=-1)
    D.CONTEXT.DEFAULT_GROUP = None
    cams = [_Cam(0), _Cam(1)]
    hist = D.DivisionStrategyHistoryFinal(cams, 2, 0)
    st, _ = D.start_strategy_final(cams, hist)
    stats = [{"forward_render_time": 3.0, "backward_render_time": 4.0, "forward_loss_time": 1.0}, {}]
    D.finish_strategy_final(cams, hist, st, stats, gather_fn=lambda v: [[9.0, -1.0], [-1.0, 9.0]])
    assert torch.equal(hist.accum_heuristic[0], torch.ones(54))  # bsz >= ws at 1152x864: no update
    assert len(hist.history) == 1


def test_zorder_shards_partition():
    g = torch.Generator().manual_seed(0)
    xyz = torch.rand(1000, 3, generator=g)
    sh = D.zorder_shards(xyz, 4)
    allids = torch.cat(sh)
    assert torch.equal(torch.sort(allids).values, torch.arange(1000))
    assert [len(s) for s in sh] == [250, 250, 250, 250]
    # spatial locality: shard bounding boxes are much smaller than the scene's
    vol = [(xyz[s].max(0).values - xyz[s].min(0).values).prod().item() for s in sh]
    assert max(vol) < 0.8


def test_division_positions_round_like_torch():
    """The numpy split equals the torch formulation (float32 cumsum
    accumulated in double, float32 share and thresholds, searchsorted) on
    random and tied heuristics."""
    import numpy as np
    import torch
    from blitzgs_b200 import distributed as D

    def torch_split(h, ws, right):
        prefix = torch.cumsum(h, dim=0)
        per = prefix[-1] / ws
        th = torch.arange(1, ws, dtype=prefix.dtype) * per
        return [0] + torch.searchsorted(prefix, th, right=right).tolist() + [h.shape[0]]

    g = np.random.default_rng(3)
    for trial in range(300):
        n = int(g.integers(8, 600))
        ws = int(g.integers(2, 9))
        h = (g.random(n) * g.choice([1.0, 1e3, 1e-3])).astype(np.float32)
        if trial % 3 == 0:
            h[:] = 1.0  # ties on the thresholds
        t = torch.from_numpy(h)
        for right in (False, True):
            assert D.division_pos_heuristic(t, n, ws, right=right) == torch_split(t, ws, right)
