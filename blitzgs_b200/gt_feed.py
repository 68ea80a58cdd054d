"""Ground-truth feed of a training batch: each rank gets the uint8 rows of
every camera band it renders (reference gaussian_renderer/loss_distribution.py:9-217).

Tasks are the ``gpuid2tasks`` of ``start_strategy_final``: rank g renders
tile rows [t_l, t_r) of camera c for every (c, t_l, t_r) in gpuid2tasks[g],
in camera order; a rank's tasks cover a contiguous range of cameras, and only
its first and last camera can be partial.

``load_camera_from_cpu_to_all_gpu`` (loss_distribution.py:83-217):
  * default: every rank copies, for each camera of its range, rows
    [first task's top, H) of its first camera, full images in between and
    [0, last task's bottom) of its last camera from the camera's host copy
    (``original_image_backup``) into ``camera.original_image`` on its GPU;
  * ``distributed_storage`` (only the node's first rank holds the images):
    that rank loads the union of the bands of all ranks of the node once and
    sends every other rank its band of each task point to point (one
    batch_isend_irecv); it keeps its own tasks' bands;
  * ``local_sampling``: every rank loads its own range (its tasks are whole
    cameras) and nothing moves between ranks.
``load_camera_from_cpu_to_all_gpu_for_eval`` (loss_distribution.py:21-80)
gives every rank of the node the whole image of every camera (a broadcast
from the rank that holds it; the reference scatters identical copies).

Host copies go through pinned staging buffers with non-blocking copies.
"""
import torch
import torch.distributed as dist

BLOCK_Y = 16


def coverage_y(tile_l, tile_r, image_height, block_y=BLOCK_Y):
    """Pixel rows [y0, y1) of tile rows [tile_l, tile_r) (get_coverage_y_min_max)."""
    return tile_l * block_y, min(tile_r * block_y, image_height)


def _rank(group):
    return dist.get_rank(group) if dist.is_initialized() else 0


def _to_device(host_rows, device):
    """Copy a host uint8 slice to ``device`` through a pinned staging buffer."""
    dev = torch.device(device)
    if dev.type == "cpu":
        return host_rows.contiguous().clone()
    staged = torch.empty(host_rows.shape, dtype=host_rows.dtype, pin_memory=True)
    staged.copy_(host_rows)
    out = torch.empty(host_rows.shape, dtype=host_rows.dtype, device=dev)
    out.copy_(staged, non_blocking=True)
    return out


def _load_range(batched_cameras, first, last, image_height, device):
    """Rows of cameras first[0]..last[0] a contiguous task range covers, onto
    ``device``; returns {camera: (y0, y1)}."""
    cov = {}
    top = coverage_y(first[1], first[2], image_height)[0]
    bottom = coverage_y(last[1], last[2], image_height)[1]
    for c in range(first[0], last[0] + 1):
        y0 = top if c == first[0] else 0
        y1 = bottom if c == last[0] else image_height
        cam = batched_cameras[c]
        cam.original_image = _to_device(cam.original_image_backup[:, y0:y1, :], device)
        cov[c] = (y0, y1)
    return cov


def load_camera_from_cpu_to_all_gpu(batched_cameras, batched_strategies, gpuid2tasks, *, device="cuda",
                                    group=None, distributed_storage=False, local_sampling=False,
                                    node_ranks=None, image_height=None):
    """Set ``camera.original_image`` on every rank to the uint8 rows of the
    bands it renders (see the module docstring).  ``node_ranks``: the ranks
    sharing the first rank's host copy in ``distributed_storage`` mode
    (default: every rank of ``group``, one node)."""
    del batched_strategies  # the tasks carry the bands, as in the reference
    rank = _rank(group)
    H = int(image_height if image_height is not None else batched_cameras[0].image_height)
    if not distributed_storage or local_sampling:
        tasks = gpuid2tasks[rank]
        if tasks:
            _load_range(batched_cameras, tasks[0], tasks[-1], H, device)
        return
    if node_ranks is None:
        node_ranks = list(range(dist.get_world_size(group)))
    first_rank = node_ranks[0]
    ops = []
    if rank == first_rank:
        busy = [r for r in node_ranks if gpuid2tasks[r]]
        if not busy:
            return
        cov = _load_range(batched_cameras, gpuid2tasks[busy[0]][0], gpuid2tasks[busy[-1]][-1], H, device)
        for r in node_ranks:
            if r == rank:
                continue
            for c, tl, tr in gpuid2tasks[r]:
                y0, y1 = coverage_y(tl, tr, H)
                base = cov[c][0]
                band = batched_cameras[c].original_image[:, y0 - base:y1 - base, :].contiguous()
                ops.append(dist.P2POp(dist.isend, band, r, group=group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for c, tl, tr in gpuid2tasks[rank]:
            y0, y1 = coverage_y(tl, tr, H)
            base = cov[c][0]
            batched_cameras[c].original_image = batched_cameras[c].original_image[:, y0 - base:y1 - base, :].contiguous()
    else:
        bufs = []
        W = None
        for c, tl, tr in gpuid2tasks[rank]:
            y0, y1 = coverage_y(tl, tr, H)
            W = int(batched_cameras[c].image_width)
            buf = torch.zeros((3, y1 - y0, W), dtype=torch.uint8, device=device)
            bufs.append((c, buf))
            ops.append(dist.P2POp(dist.irecv, buf, first_rank, group=group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for c, buf in bufs:
            batched_cameras[c].original_image = buf


def load_camera_from_cpu_to_all_gpu_for_eval(batched_cameras, batched_strategies, gpuid2tasks, *, device="cuda",
                                             group=None, distributed_storage=False, local_sampling=False,
                                             bsz=None, node_ranks=None):
    """Every rank gets the whole uint8 image of every camera.  With
    ``distributed_storage`` the holder broadcasts it: the node's first rank,
    or with ``local_sampling`` the rank whose cameras they are (camera i on
    rank i // (bsz / world size))."""
    del batched_strategies, gpuid2tasks
    if not distributed_storage:
        for cam in batched_cameras:
            cam.original_image = _to_device(cam.original_image_backup, device)
        return
    ws = dist.get_world_size(group)
    if node_ranks is None:
        node_ranks = list(range(ws))
    rank = _rank(group)
    for idx, cam in enumerate(batched_cameras):
        src = idx // (bsz // ws) if local_sampling else node_ranks[0]
        if rank == src:
            cam.original_image = _to_device(cam.original_image_backup, device)
        else:
            cam.original_image = torch.zeros((3, int(cam.image_height), int(cam.image_width)), dtype=torch.uint8,
                                             device=device)
        dist.broadcast(cam.original_image, src=src, group=group)
