"""Multi-GPU plumbing: workload division, spatial sharding, and the one
exchange per direction.

Workload division mirrors the reference's "final" policy
(gaussian_renderer/workload_division.py:66-82, 645-937):
``division_pos_heuristic``, ``DivisionStrategyFinal``,
``DivisionStrategyHistoryFinal``, ``start_strategy_final`` and
``finish_strategy_final`` keep the reference's names, arguments, assertions
and results.  The reference reads process globals from utils.general_utils
(GLOBAL_RANK, DEFAULT_GROUP, TILE_X/Y, IMG_H/W, args); here they live in
``CONTEXT`` (set once with ``init_context``).

Gaussian sharding is spatial: Morton (z-order) keys of the means, equal-count
contiguous chunks (the reference shards round-robin; parity is therefore
compared on global Gaussian ids, never on shard-local indices).

The exchange replaces all_to_all_communication_final
(gaussian_renderer/__init__.py:22-189) -- per (destination, camera)
index_select + cat, a blocking size all_gather and two NCCL all-to-alls
forward plus the autograd all-to-all backward -- with one packed
all_to_all_single per direction: a 12-float record per (Gaussian, camera,
destination) forward, a 12-float gradient record back, scatter-added into the
owner's per-camera gradient accumulators.  Received records are ordered by
source rank, then by the sender's local index, as in the reference.  The
functions here are device-agnostic torch.distributed code (NCCL on GPUs,
gloo on CPU in the tests).
"""
from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np
import torch
import torch.distributed as dist

TILE = 16

# ---------------------------------------------------------------------------
# process context (the reference's utils.general_utils globals)
# ---------------------------------------------------------------------------

CONTEXT = SimpleNamespace(GLOBAL_RANK=0, WORLD_SIZE=1, DEFAULT_GROUP=None, TILE_X=1, TILE_Y=1, IMG_H=0, IMG_W=0,
                          args=SimpleNamespace(bsz=1, border_divpos_coeff=1.0, local_sampling=False,
                                               heuristic_decay=0.0, adjust_strategy_warmp_iterations=-1,
                                               no_heuristics_update=False),
                          cur_iter=0)


def init_context(rank, world_size, image_height, image_width, group=None, **args):
    CONTEXT.GLOBAL_RANK = rank
    CONTEXT.WORLD_SIZE = world_size
    CONTEXT.DEFAULT_GROUP = group
    CONTEXT.IMG_H, CONTEXT.IMG_W = image_height, image_width
    CONTEXT.TILE_X = (image_width + TILE - 1) // TILE
    CONTEXT.TILE_Y = (image_height + TILE - 1) // TILE
    for k, v in args.items():
        setattr(CONTEXT.args, k, v)
    return CONTEXT


def _group_size():
    g = CONTEXT.DEFAULT_GROUP
    if g is None:
        return CONTEXT.WORLD_SIZE
    return dist.get_world_size(g)


# ---------------------------------------------------------------------------
# workload division (reference workload_division.py)
# ---------------------------------------------------------------------------

def division_pos_heuristic(heuristic, tile_num, world_size, right=False):
    """Split the prefix sum of per-tile-row costs into world_size equal parts
    (workload_division.py:66-82).  Runs on the host copy of the heuristic,
    in numpy with PyTorch's float32 rounding: torch.cumsum of float32 on the
    CPU accumulates in double and rounds each prefix to float32, which
    cumsum in float64 followed by one cast reproduces; the share and the
    thresholds are float32 operations as in torch (a few torch calls cost
    ~0.1 ms per step, this ~0.01)."""
    assert heuristic.shape[0] == tile_num, "the length of heuristics should be the same as the number of tiles."
    h = heuristic.detach().to("cpu").numpy() if isinstance(heuristic, torch.Tensor) else np.asarray(heuristic)
    if h.dtype != np.float32:
        # other dtypes: the torch formulation itself
        t = torch.from_numpy(np.ascontiguousarray(h))
        prefix = torch.cumsum(t, dim=0)
        per = prefix[-1] / world_size
        thresholds = torch.arange(1, world_size, dtype=prefix.dtype) * per
        idx = torch.searchsorted(prefix, thresholds, right=right)
        return [0] + idx.tolist() + [tile_num]
    prefix = np.cumsum(h, dtype=np.float64).astype(np.float32)
    per = np.float32(prefix[-1]) / np.float32(world_size)
    thresholds = np.arange(1, world_size, dtype=np.float32) * per
    idx = np.searchsorted(prefix, thresholds, side="right" if right else "left")
    return [0] + [int(i) for i in idx] + [tile_num]


class DivisionStrategyFinal:
    """Row split of one camera over the ranks rendering it (workload_division.py:645-736)."""

    def __init__(self, camera, world_size, gpu_ids, division_pos, gpu_for_this_camera_tilelr):
        assert world_size > 0, "The world_size must be greater than 0."
        assert len(gpu_ids) == world_size, "The number of gpu_ids must be equal to the world_size."
        assert len(division_pos) == world_size + 1, "The number of division_pos must be equal to the world_size+1."
        assert division_pos[0] == 0, "The first element of division_pos must be 0."
        assert division_pos[-1] == CONTEXT.TILE_Y, \
            "The last element of division_pos must be equal to the total number of tiles."
        for i in range(1, len(division_pos)):
            assert division_pos[i] > division_pos[i - 1], "The division_pos must be in ascending order."
        for idx in range(len(gpu_for_this_camera_tilelr)):
            assert (gpu_for_this_camera_tilelr[idx][0] == division_pos[idx]
                    and gpu_for_this_camera_tilelr[idx][1] == division_pos[idx + 1]), \
                "The division_pos must be consistent with gpu_for_this_camera_tilelr."
        self.camera = camera
        self.world_size = world_size
        self.gpu_ids = gpu_ids
        self.rank = gpu_ids.index(CONTEXT.GLOBAL_RANK) if CONTEXT.GLOBAL_RANK in gpu_ids else -1
        self.division_pos = division_pos

    def get_local2j_ids(self, means2D, radii, raster_settings, cuda_args):
        from . import ops
        dist_global = torch.tensor(self.division_pos, dtype=torch.int32, device=means2D.device) * CONTEXT.TILE_X
        avoid = bool(cuda_args.get("avoid_pixel_all2all", False)) if isinstance(cuda_args, dict) else False
        mask = ops.local2j_ids_bool(raster_settings.image_height, raster_settings.image_width, self.rank,
                                    self.world_size, means2D, radii, dist_global, avoid)
        return [mask[:, rk].nonzero(as_tuple=True)[0] for rk in range(self.world_size)], mask

    def row_range(self, rank=None):
        rank = CONTEXT.GLOBAL_RANK if rank is None else rank
        if rank not in self.gpu_ids:
            return None
        r = self.gpu_ids.index(rank)
        return self.division_pos[r], self.division_pos[r + 1]

    def get_compute_locally(self, device="cuda"):
        rr = self.row_range()
        if rr is None:
            return None
        cl = torch.zeros((CONTEXT.TILE_Y, CONTEXT.TILE_X), dtype=torch.bool, device=device)
        cl[rr[0]:rr[1]] = True
        return cl

    def get_compute_locally_all(self, device="cuda"):
        if CONTEXT.GLOBAL_RANK not in self.gpu_ids:
            return None
        return torch.ones((CONTEXT.TILE_Y, CONTEXT.TILE_X), dtype=torch.bool, device=device)

    def get_extended_compute_locally(self):
        return None


class DivisionStrategyHistoryFinal:
    """Per-camera accumulated tile-row heuristic (workload_division.py:739-782)."""

    def __init__(self, dataset, world_size, rank):
        self.world_size = world_size
        self.rank = rank
        self.accum_heuristic = {}
        cams = dataset.cameras if hasattr(dataset, "cameras") else dataset
        for camera in cams:
            self.accum_heuristic[camera.uid] = torch.ones((CONTEXT.TILE_Y,), dtype=torch.float32)
        self.history = []

    def store_stats(self, batched_cameras, gpu_camera_running_time, batched_strategies):
        info = []
        all_cam = [0 for _ in batched_cameras]
        all_gpu = [0 for _ in range(self.world_size)]
        for cid, camera in enumerate(batched_cameras):
            each = []
            for g in batched_strategies[cid].gpu_ids:
                all_cam[cid] += gpu_camera_running_time[g][cid]
                all_gpu[g] += gpu_camera_running_time[g][cid]
                each.append(gpu_camera_running_time[g][cid])
            info.append({"camera_id": camera.uid, "gpu_ids": batched_strategies[cid].gpu_ids,
                         "division_pos": batched_strategies[cid].division_pos, "each_gpu_running_time": each})
        self.history.append({"iteration": CONTEXT.cur_iter, "all_gpu_running_time": all_gpu,
                             "all_camera_running_time": all_cam, "batched_camera_info": info})

    def to_json(self):
        return self.history


def start_strategy_final(batched_cameras, strategy_history):
    """Row split of the batch's concatenated tile rows (workload_division.py:785-873)."""
    args = CONTEXT.args
    ws = _group_size()
    n_rows = CONTEXT.TILE_Y
    total = n_rows * len(batched_cameras)
    if args.local_sampling:
        strategies = []
        tasks = [[] for _ in range(ws)]
        per_gpu = args.bsz // CONTEXT.WORLD_SIZE
        for idx, camera in enumerate(batched_cameras):
            g = idx // per_gpu
            tasks[g].append((idx, 0, n_rows))
            strategies.append(DivisionStrategyFinal(camera, 1, [g], [0, n_rows], [(0, n_rows)]))
        return strategies, tasks
    catted = np.concatenate([strategy_history.accum_heuristic[c.uid].detach().to("cpu").numpy()
                             for c in batched_cameras])
    pos = division_pos_heuristic(catted, total, ws, right=True)
    coeff = args.border_divpos_coeff
    for i in range(1, len(pos) - 1):
        if pos[i] % n_rows + coeff >= n_rows:
            pos[i] = pos[i] // n_rows * n_rows + n_rows
        elif pos[i] % n_rows - coeff <= 0:
            pos[i] = pos[i] // n_rows * n_rows
    for i in range(0, len(pos) - 1):
        assert pos[i] + coeff < pos[i + 1], "Each part between division_pos must be large enough."
    strategies = []
    tasks = [[] for _ in range(ws)]
    for idx, camera in enumerate(batched_cameras):
        off = idx * n_rows
        gids, tilelr = [], []
        for g in range(ws):
            l, r = pos[g], pos[g + 1]
            if r <= off or off + n_rows <= l:
                continue
            gids.append(g)
            lo, hi = max(l, off) - off, min(r, off + n_rows) - off
            tilelr.append((lo, hi))
            tasks[g].append((idx, lo, hi))
        strategies.append(DivisionStrategyFinal(camera, len(gids), gids, [0] + [t[1] for t in tilelr], tilelr))
    return strategies, tasks


def finish_strategy_final(batched_cameras, strategy_history, batched_strategies, batched_statistic_collector,
                          gather_fn=None):
    """Update the per-camera heuristic from measured render/loss times
    (workload_division.py:876-937).  ``gather_fn(list_of_floats) -> [ws][n]``
    all-gathers the per-camera times (defaults to the process group)."""
    times = []
    missing = False
    for idx, st in enumerate(batched_strategies):
        if CONTEXT.GLOBAL_RANK not in st.gpu_ids:
            times.append(-1.0)
            continue
        stats = batched_statistic_collector[idx]
        if any(k not in stats for k in ("forward_render_time", "backward_render_time", "forward_loss_time")):
            missing = True
        times.append(stats.get("forward_render_time", 0.0) + stats.get("backward_render_time", 0.0)
                     + stats.get("forward_loss_time", 0.0) * 2)
    gathered = (gather_fn or _allgather_floats)(times)
    strategy_history.store_stats(batched_cameras, gathered, batched_strategies)
    args = CONTEXT.args
    ws = _group_size()
    if (missing or CONTEXT.cur_iter <= args.adjust_strategy_warmp_iterations or ws == 1
            or args.no_heuristics_update
            or (args.bsz >= ws and (CONTEXT.IMG_H <= 1080 or CONTEXT.IMG_W <= 1920))
            or (CONTEXT.IMG_H <= 600 or CONTEXT.IMG_W <= 1000)):
        return
    for cid, (camera, st) in enumerate(zip(batched_cameras, batched_strategies)):
        new = torch.zeros((CONTEXT.TILE_Y,), dtype=torch.float32)
        for lid, g in enumerate(st.gpu_ids):
            l, r = st.division_pos[lid], st.division_pos[lid + 1]
            new[l:r] = gathered[g][cid] / (r - l)
        if args.heuristic_decay == 0:
            strategy_history.accum_heuristic[camera.uid] = new
        else:
            strategy_history.accum_heuristic[camera.uid] = (
                strategy_history.accum_heuristic[camera.uid] * args.heuristic_decay + new * (1 - args.heuristic_decay))


def _allgather_floats(vals):
    ws = _group_size()
    if ws == 1:
        return [list(vals)]
    backend = dist.get_backend(CONTEXT.DEFAULT_GROUP)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor(vals, dtype=torch.float32, device=dev)
    out = torch.empty((ws * len(vals),), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(out, t, group=CONTEXT.DEFAULT_GROUP)
    out = out.view(ws, len(vals))
    return out.cpu().tolist()


# ---------------------------------------------------------------------------
# spatial sharding
# ---------------------------------------------------------------------------

def _spread_bits(v):
    v = v & 0x1FFFFF
    v = (v | (v << 32)) & 0x1F00000000FFFF
    v = (v | (v << 16)) & 0x1F0000FF0000FF
    v = (v | (v << 8)) & 0x100F00F00F00F00F
    v = (v | (v << 4)) & 0x10C30C30C30C30C3
    v = (v | (v << 2)) & 0x1249249249249249
    return v


def morton_keys(xyz):
    """63-bit z-order keys of positions quantised to 21 bits per axis over their bounding box."""
    x = xyz.detach().to("cpu", torch.float64)
    lo = x.min(0).values
    span = (x.max(0).values - lo).clamp(min=1e-12)
    q = ((x - lo) / span * (2 ** 21 - 1)).round().to(torch.int64)
    return _spread_bits(q[:, 0]) | (_spread_bits(q[:, 1]) << 1) | (_spread_bits(q[:, 2]) << 2)


def zorder_shards(xyz, world_size):
    """Global Gaussian ids owned by each rank: z-order sorted, equal-count chunks."""
    order = torch.argsort(morton_keys(xyz), stable=True)
    return [c.clone() for c in torch.tensor_split(order, world_size)]


# ---------------------------------------------------------------------------
# exchange
# ---------------------------------------------------------------------------

@dataclass
class ExchangePlan:
    """Send/receive bookkeeping of one step (kept for the backward exchange)."""
    size: list                # size[src][dst][cam] record counts, identical on every rank
    my_cams: list             # cameras this rank renders, in batch order
    recv_offsets: dict = field(default_factory=dict)  # cam -> [(src, start, count) in recv buffer]
    send_splits: list = field(default_factory=list)
    recv_splits: list = field(default_factory=list)


def plan_from_sizes(size, n_cams, rank, ws):
    """Splits and receive offsets from size[src][dst][cam] (the same matrix on
    every rank).  The send buffer holds, per destination in rank order, that
    destination's rows camera by camera; the receive buffer holds, per
    source in rank order, the rows that source sent, camera by camera."""
    my_cams = [k for k in range(n_cams) if any(size[i][rank][k] for i in range(ws))]
    plan = ExchangePlan(size=size, my_cams=my_cams)
    plan.send_splits = [sum(size[rank][j]) for j in range(ws)]
    plan.recv_splits = [sum(size[i][rank]) for i in range(ws)]
    off = 0
    per_cam = {k: [] for k in range(n_cams)}
    for i in range(ws):
        for k in range(n_cams):
            c = size[i][rank][k]
            per_cam[k].append((i, off, c))
            off += c
    plan.recv_offsets = per_cam
    return plan


def send_offsets(size, rank, ws, n_cams):
    """dest_off[k][j]: first send-buffer row of camera k's records for rank j
    (the layout plan_from_sizes describes)."""
    base = [0]
    for j in range(ws):
        base.append(base[-1] + sum(size[rank][j]))
    out = []
    for k in range(n_cams):
        out.append([base[j] + sum(size[rank][j][:k]) for j in range(ws)])
    return out


def exchange_layout(allc, rank, ws, n_cams):
    """Everything one step's exchange needs, from the all-gathered counts
    ``allc[src][cam] = [list length, rows for rank 0, ..., rows for rank
    ws-1]`` (identical on every rank): (counts, plan, offs, dest_off) with
    counts[k] this rank's list length of camera k, offs the compact-row
    offsets of the cameras' lists (offs[k] + slot is the row of camera k's
    slot-th listed Gaussian in the backward's accumulator), and dest_off the
    send offsets of send_offsets()."""
    counts = [int(allc[rank][k][0]) for k in range(n_cams)]
    size = [[[int(allc[i][k][1 + j]) for k in range(n_cams)] for j in range(ws)] for i in range(ws)]
    plan = plan_from_sizes(size, n_cams, rank, ws)
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    return counts, plan, offs, send_offsets(size, rank, ws, n_cams)
