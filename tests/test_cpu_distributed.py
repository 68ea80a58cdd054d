"""Multi-rank host logic on CPU: the packed exchange (gloo, world_size 2) and the
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


def _rank_data(rank, ws):
    """Deterministic shard records and routes of one rank."""
    P = 40 + 7 * rank
    g = torch.Generator().manual_seed(100 + rank)
    recs = []
    for k in range(N_CAMS):
        gid = torch.arange(P, dtype=torch.float32) + 1000 * rank
        recs.append(torch.stack([gid, torch.full((P,), float(k)), torch.full((P,), float(rank)),
                                 torch.rand(P, generator=g)], 1))
    send = []
    for k in range(N_CAMS):
        per = []
        for j in range(ws):
            m = torch.rand(P, generator=g) < (0.3 + 0.2 * j)
            if k == 2 and j == 1:
                m[:] = False  # a camera sends nothing to rank 1
            per.append(m.nonzero(as_tuple=True)[0])
        send.append(per)
    return P, recs, send


def _worker(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        P, recs, send = _rank_data(rank, ws)
        plan = D.plan_exchange(send, N_CAMS)
        out = D.exchange_forward(recs, plan)
        # expected: concatenation over source ranks (in order) of their rows routed here
        for k in range(N_CAMS):
            exp = []
            for i in range(ws):
                Pi, ri, si = _rank_data(i, ws)
                if len(si[k][rank]):
                    exp.append(ri[k][si[k][rank]])
            if exp:
                assert torch.equal(out[k], torch.cat(exp, 0)), (rank, k)
            else:
                assert k not in out
        # backward: gradient = f(record); owner accumulates over destinations
        grads = {k: v[:, :3] * 2 + 1 for k, v in out.items()}
        acc = D.exchange_backward(grads, plan, P, N_CAMS, 3)
        for k in range(N_CAMS):
            e = torch.zeros(P, 3)
            for j in range(ws):
                ids = send[k][j]
                e.index_add_(0, ids, recs[k][ids][:, :3] * 2 + 1)
            assert torch.allclose(acc[k], e), (rank, k)
        q.put((rank, "ok"))
    except BaseException as ex:  # report to the parent
        q.put((rank, repr(ex)))
    finally:
        dist.destroy_process_group()


def test_exchange_round_trip_gloo_ws2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(res) == [(0, "ok"), (1, "ok")], res


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
