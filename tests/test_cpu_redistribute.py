"""Redistribution of the shards after densification (blitzgs_b200.redistribute)
on gloo CPU ranks: the round-robin mode against a restatement of the
reference's all2all_gaussian_state (scene/gaussian_model.py:1044-1052,
1075-1076), the z-order mode's invariants, Adam moments travelling with their
rows, and the redistribution trigger."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blitzgs_b200 import densify as DZ
from blitzgs_b200 import redistribute as RD


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


_SIZES = [300, 90, 170]


def _shard(rank):
    """Rank-local rows: positions, and a feature row whose column 0 is the
    row's global id; sizes differ per rank (a densified, unbalanced state)."""
    n = _SIZES[rank]
    g = torch.Generator().manual_seed(40 + rank)
    xyz = torch.rand(n, 3, generator=g) * torch.tensor([100.0, 60.0, 8.0])
    feat = torch.rand(n, 4, generator=g)
    feat[:, 0] = torch.arange(n, dtype=torch.float32) + 1000 * rank
    return xyz, feat


def _model(rank):
    xyz, feat = _shard(rank)
    params = [torch.nn.Parameter(xyz.clone()), torch.nn.Parameter(feat.clone())]
    opt = torch.optim.Adam([{"params": [p], "lr": 1e-3} for p in params])
    for p in params:  # moments tied to their rows: exp_avg = 2 * row, exp_avg_sq = 3 * row
        opt.state[p] = {"step": torch.tensor(4.0), "exp_avg": p.detach() * 2, "exp_avg_sq": p.detach() * 3}
    return params, opt


def _worker(rank, ws, port, mode, q, sizes=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    if sizes is not None:
        _SIZES[:] = sizes
    try:
        params, opt = _model(rank)
        stats = DZ.DensificationStats(params[0].shape[0], "cpu")
        stats.denom += 1
        new = RD.redistribute(params, opt, mode=mode, force=True, densify=stats)
        xyz, feat = new
        assert isinstance(xyz, torch.nn.Parameter) and opt.param_groups[0]["params"][0] is xyz
        for p in new:
            st = opt.state[p]
            assert torch.equal(st["exp_avg"], p.detach() * 2) and torch.equal(st["exp_avg_sq"], p.detach() * 3)
            assert float(st["step"]) == 4.0
        assert stats.denom.shape[0] == xyz.shape[0] and not stats.denom.any()
        if mode == "round_robin":
            # reference: rows i % ws == j go to rank j; received = sources in rank order
            exp_x, exp_f = [], []
            for i in range(ws):
                xi, fi = _shard(i)
                sel = torch.arange(xi.shape[0]) % ws == rank
                exp_x.append(xi[sel])
                exp_f.append(fi[sel])
            assert torch.equal(xyz.detach(), torch.cat(exp_x)) and torch.equal(feat.detach(), torch.cat(exp_f))
            q.put((rank, "ok", None))
        else:
            lo, span = RD.global_bbox(xyz, None)
            keys = RD.morton_keys_in(xyz, lo, span)
            assert torch.all(keys[1:] >= keys[:-1])  # each shard stays in z-order
            kmin = keys.min() if keys.numel() else torch.tensor(2 ** 62)
            kmax = keys.max() if keys.numel() else torch.tensor(-1)
            q.put((rank, "ok", (int(kmin), int(kmax), feat[:, 0].long().tolist())))
    except Exception:
        q.put((rank, traceback.format_exc(), None))
    finally:
        dist.destroy_process_group()


def _run(ws, mode, sizes=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, mode, q, sizes)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for r, status, _ in res:
        assert status == "ok", status
    return res


@pytest.mark.parametrize("ws", [2, 3])
def test_round_robin_matches_reference_all2all(ws):
    _run(ws, "round_robin")


@pytest.mark.parametrize("ws,sizes", [(2, None), (3, None), (3, [300, 0, 170])])
def test_zorder_keeps_rows_orders_ranges_and_balances(ws, sizes):
    res = _run(ws, "zorder", sizes)
    if sizes is not None:
        _SIZES[:] = sizes
    ids = sorted(i for _, _, (_, _, rows) in res for i in rows)
    expected = sorted(int(i) for r in range(ws) for i in _shard(r)[1][:, 0].long().tolist())
    assert ids == expected  # every row arrives exactly once
    total = len(ids)
    for r in range(ws - 1):
        assert res[r][2][1] <= res[r + 1][2][0]  # contiguous z-order ranges, in rank order
    for _, _, (_, _, rows) in res:
        assert abs(len(rows) - total / ws) <= 0.05 * total / ws


def _trigger_worker(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        out = (RD.need_redistribute([100, 120][rank], threshold=1.5),
               RD.need_redistribute([100, 160][rank], threshold=1.5),
               RD.need_redistribute([100, 100][rank], force=True))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_trigger_is_the_reference_threshold():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_trigger_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for _, out in res:
        assert out == (False, True, True)


def _missing_moment_worker(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        params, opt = _model(rank)
        if rank == 1:  # this rank has not stepped its optimizer: no moments yet
            for p in params:
                opt.state.pop(p)
        try:
            RD.redistribute(params, opt, mode="round_robin", force=True)
            q.put((rank, "no error"))
        except RuntimeError as e:
            q.put((rank, "raised" if "different Adam moments" in str(e) else repr(e)))
    finally:
        dist.destroy_process_group()


def test_ranks_with_different_moments_fail_together():
    """A rank without Adam moments (not stepped yet) would make fewer
    exchanges than the others; every rank raises before the first one."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_missing_moment_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(res) == [(0, "raised"), (1, "raised")]
