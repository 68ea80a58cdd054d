"""Redistribution of the Gaussians across ranks after densification.

The reference (scene/gaussian_model.py:1044-1133) checks after densification
whether the ranks' Gaussian counts drifted apart (min * threshold < max, or
a forced round; need_redistribute_gaussians, :1078-1088) and then moves
every row of every parameter *and* its Adam moments (exp_avg, exp_avg_sq)
to its destination rank with one all-to-all per tensor
(all2all_gaussian_state :1044-1052, all2all_tensors_in_optimizer
:1054-1073), rebuilds the optimizer's parameters and resets the
densification statistics (redistribute_gaussians :1090-1133).  Its
destination is round-robin: local row i goes to rank i % world_size
(get_destination_1, :1075-1076).

Here the same machinery serves the spatial sharding the fused distributed
step uses (each rank owns a contiguous z-order range of the scene, which
keeps the Gaussians a camera sees on few ranks and their rows together in
memory):

  * ``mode="zorder"``: Morton keys over the global bounding box (one
    all-reduce), splitters from an all-gather of evenly spaced samples of
    every rank's sorted keys weighted by its count, destination = the
    key's bucket; every rank sorts what it receives by key, so each shard
    stays in z-order;
  * ``mode="round_robin"``: the reference's destinations and order.

Collectives: one all-gather of counts, (z-order: one all-reduce and one
all-gather of samples,) one all-gather of the send-size matrix, and one
all_to_all_single per tensor.  Works with NCCL on device tensors and with
gloo on CPU tensors.
"""
import torch
import torch.distributed as dist

from .distributed import _spread_bits


def _counts(n_local, group, device):
    ws = dist.get_world_size(group)
    c = torch.tensor([n_local], dtype=torch.int64, device=device)
    out = [torch.zeros_like(c) for _ in range(ws)]
    dist.all_gather(out, c, group=group)
    return [int(x) for x in torch.cat(out).tolist()]


def need_redistribute(n_local, group=None, threshold=1.5, force=False, device="cpu"):
    """The reference's trigger: True when forced or when min(counts) *
    threshold < max(counts) over the ranks (every rank gets the same
    answer; a single rank never redistributes)."""
    if dist.get_world_size(group) == 1:
        return False
    if force:
        return True
    c = _counts(n_local, group, device)
    return min(c) * threshold < max(c)


def global_bbox(xyz, group=None):
    """(lo, span) float64 [3] of all ranks' positions (one all-reduce of
    [-min, max]); empty shards contribute nothing."""
    x = xyz.detach().to(torch.float64)
    if x.shape[0]:
        mm = torch.cat([-x.min(0).values, x.max(0).values])
    else:
        mm = torch.full((6,), float("-inf"), dtype=torch.float64, device=x.device)
    dist.all_reduce(mm, op=dist.ReduceOp.MAX, group=group)
    lo = -mm[:3]
    span = (mm[3:] - lo).clamp(min=1e-12)
    return lo, span


def morton_keys_in(xyz, lo, span):
    """63-bit z-order keys of positions quantised to 21 bits per axis over
    the given box (the single-process zorder_shards uses the points' own
    box)."""
    x = xyz.detach().to(torch.float64)
    q = ((x - lo) / span * (2 ** 21 - 1)).round().clamp(0, 2 ** 21 - 1).to(torch.int64)
    return _spread_bits(q[:, 0]) | (_spread_bits(q[:, 1]) << 1) | (_spread_bits(q[:, 2]) << 2)


def zorder_destinations(keys, group=None, samples=1024):
    """Destination rank of every local key: ws equal-count ranges of the
    global key order, located from an all-gather of ``samples`` evenly
    spaced keys of every rank (each standing for count/samples keys)."""
    ws = dist.get_world_size(group)
    dev = keys.device
    n = keys.shape[0]
    sk = torch.sort(keys).values
    if n:
        pos = (torch.arange(samples, device=dev, dtype=torch.float64) + 0.5) * (n / samples)
        smp = sk[pos.long().clamp(max=n - 1)]
    else:
        smp = torch.zeros(samples, dtype=torch.int64, device=dev)
    counts = _counts(n, group, dev)
    allsmp = [torch.zeros_like(smp) for _ in range(ws)]
    dist.all_gather(allsmp, smp.contiguous(), group=group)
    vals, wts = [], []
    for r in range(ws):
        if counts[r]:
            vals.append(allsmp[r])
            wts.append(torch.full((samples,), counts[r] / samples, dtype=torch.float64, device=dev))
    if not vals:
        return torch.zeros(0, dtype=torch.int64, device=dev)
    v = torch.cat(vals)
    w = torch.cat(wts)
    o = torch.argsort(v, stable=True)
    v, cw = v[o], torch.cumsum(w[o], 0)
    total = float(sum(counts))
    # splitter j: the first sample key whose cumulative weight reaches j/ws of the total
    targets = torch.tensor([total * j / ws for j in range(1, ws)], dtype=torch.float64, device=dev)
    idx = torch.searchsorted(cw, targets).clamp(max=v.numel() - 1)
    splitters = v[idx]
    return torch.searchsorted(splitters, keys, right=True)


def round_robin_destinations(n_local, world_size, device="cpu"):
    """The reference's get_destination_1: local row i -> rank i % world_size."""
    return torch.arange(n_local, device=device) % world_size


def exchange_rows(tensors, dest, group=None):
    """Move row i of every tensor to rank dest[i] (one all_to_all_single per
    tensor).  Rows arrive ordered by source rank, then by their order at the
    source.  Returns the received tensors."""
    ws = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = dest.device
    send = torch.bincount(dest, minlength=ws).to(torch.int64)
    mat = [torch.zeros_like(send) for _ in range(ws)]
    dist.all_gather(mat, send, group=group)
    send_splits = [int(x) for x in send.tolist()]
    recv_splits = [int(mat[i][rank]) for i in range(ws)]
    order = torch.argsort(dest, stable=True)
    out = []
    for t in tensors:
        src = t.detach()[order].contiguous()
        recv = torch.empty((sum(recv_splits),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_to_all_single(recv, src, recv_splits, send_splits, group=group)
        out.append(recv)
    return out


def redistribute(params, optimizer=None, group=None, mode="zorder", threshold=1.5, force=False,
                 densify=None, samples=1024):
    """Rebalance a model shard across the ranks.

    ``params``: the shard's parameter tensors, all with one row per Gaussian,
    the first being the positions [n, 3] (the reference's order: xyz,
    features_dc, features_rest, opacity, scaling, rotation).  ``optimizer``
    (one parameter per group, as the reference's Adam and
    SparseGaussianAdam): its exp_avg / exp_avg_sq travel with their rows and
    its groups are rebuilt around the new parameters.  ``densify`` (a
    densify.DensificationStats) is re-created for the new shard size, zeroed
    as the reference resets its statistics.

    Returns the new parameters (nn.Parameters when the inputs were), or the
    inputs unchanged when no redistribution is needed."""
    xyz = params[0]
    dev = xyz.device
    n = xyz.shape[0]
    if not need_redistribute(n, group, threshold, force, device=dev):
        return list(params)
    ws = dist.get_world_size(group)
    if mode == "zorder":
        lo, span = global_bbox(xyz, group)
        dest = zorder_destinations(morton_keys_in(xyz, lo, span), group, samples)
    elif mode == "round_robin":
        dest = round_robin_destinations(n, ws, dev)
    else:
        raise ValueError(f"unknown redistribution mode {mode!r}")
    states = []
    if optimizer is not None:
        for p in params:
            st = optimizer.state.get(p, {})
            states.append([k for k in ("exp_avg", "exp_avg_sq") if k in st])
        # every rank must move the same moments, or the exchanges below pair
        # different tensors (or wait for ever): agree first, fail together
        have = torch.tensor([[k in keys for k in ("exp_avg", "exp_avg_sq")] for keys in states],
                            dtype=torch.int32, device=dev).reshape(-1)
        lo_have, hi_have = have.clone(), have.clone()
        dist.all_reduce(lo_have, op=dist.ReduceOp.MIN, group=group)
        dist.all_reduce(hi_have, op=dist.ReduceOp.MAX, group=group)
        if not torch.equal(lo_have, hi_have):
            raise RuntimeError("redistribute: the ranks hold different Adam moments (a rank has not stepped "
                               "its optimizer yet); step every rank, or redistribute before any step")
    moving = list(params)
    for p, keys in zip(params, states):
        moving += [optimizer.state[p][k] for k in keys]
    moved = exchange_rows(moving, dest, group)
    if mode == "zorder":
        # keep the shard in z-order: sort what arrived by key
        order = torch.argsort(morton_keys_in(moved[0], lo, span), stable=True)
        moved = [t[order].contiguous() for t in moved]
    new_params = []
    for p, t in zip(params, moved[:len(params)]):
        new_params.append(torch.nn.Parameter(t, requires_grad=p.requires_grad)
                          if isinstance(p, torch.nn.Parameter) else t)
    if optimizer is not None:
        k = len(params)
        for p, np_, keys in zip(params, new_params, states):
            st = optimizer.state.pop(p, None)
            for key in keys:
                st[key] = moved[k]
                k += 1
            for grp in optimizer.param_groups:
                if len(grp["params"]) == 1 and grp["params"][0] is p:
                    grp["params"][0] = np_
            if st is not None:
                optimizer.state[np_] = st
    if densify is not None:
        m = new_params[0].shape[0]
        densify.xyz_gradient_accum = torch.zeros((m, 1), dtype=densify.xyz_gradient_accum.dtype, device=dev)
        densify.denom = torch.zeros((m, 1), dtype=densify.denom.dtype, device=dev)
        densify.max_radii2D = torch.zeros((m,), dtype=densify.max_radii2D.dtype, device=dev)
    return new_params
