"""Ground-truth band feed (blitzgs_b200.gt_feed) on gloo CPU ranks: every rank
ends up with exactly the uint8 rows of the bands its tasks name
(gaussian_renderer/loss_distribution.py:83-217), in the default,
distributed-storage and local-sampling modes, and the eval feed gives every
rank whole images (loss_distribution.py:21-80)."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blitzgs_b200 import gt_feed as G

H, W, WS = 64, 24, 3
# rank g renders tile rows [t_l, t_r) of camera c for (c, t_l, t_r) in TASKS[g]
TASKS = [[(0, 0, 4), (1, 0, 1)], [(1, 1, 4), (2, 0, 2)], [(2, 2, 4)]]
LOCAL_TASKS = [[(0, 0, 4)], [(1, 0, 4)], [(2, 0, 4)]]
# the rank holding the images renders nothing itself
IDLE_HOLDER_TASKS = [[], [(0, 0, 4), (1, 0, 3)], [(1, 3, 4), (2, 0, 4)]]


class _Cam:
    def __init__(self, k, has_copy):
        g = torch.Generator().manual_seed(70 + k)
        self.image_height, self.image_width = H, W
        self.full = torch.randint(0, 256, (3, H, W), generator=g, dtype=torch.uint8)
        self.original_image_backup = self.full.clone() if has_copy else None
        self.original_image = None


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WS)
    try:
        if mode == "eval_dist":
            cams = [_Cam(k, rank == 0) for k in range(3)]
            G.load_camera_from_cpu_to_all_gpu_for_eval(cams, None, None, device="cpu", distributed_storage=True)
            for c in cams:
                assert torch.equal(c.original_image, c.full)
            q.put((rank, "ok"))
            return
        if mode == "eval_local":
            # camera i held by rank i // (bsz / ws), bsz = 3
            cams = [_Cam(k, k == rank) for k in range(3)]
            G.load_camera_from_cpu_to_all_gpu_for_eval(cams, None, None, device="cpu", distributed_storage=True,
                                                       local_sampling=True, bsz=3)
            for c in cams:
                assert torch.equal(c.original_image, c.full)
            q.put((rank, "ok"))
            return
        tasks = {"local": LOCAL_TASKS, "dist_idle_holder": IDLE_HOLDER_TASKS}.get(mode, TASKS)
        # distributed storage: only the first rank of the node holds the images
        cams = [_Cam(k, not mode.startswith("dist") or rank == 0) for k in range(3)]
        G.load_camera_from_cpu_to_all_gpu(cams, None, tasks, device="cpu", distributed_storage=(mode != "default"),
                                          local_sampling=(mode == "local"))
        for c, tl, tr in tasks[rank]:
            y0, y1 = G.coverage_y(tl, tr, H)
            got = cams[c].original_image
            assert got is not None and got.dtype == torch.uint8 and torch.equal(got, cams[c].full[:, y0:y1, :]), \
                (c, tl, tr, None if got is None else tuple(got.shape))
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["default", "dist", "dist_idle_holder", "local", "eval_dist", "eval_local"])
def test_gt_bands_reach_their_ranks(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(WS)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs])
    for p in procs:
        p.join(timeout=60)
    for r, status in res:
        assert status == "ok", status


def test_coverage_rows():
    assert G.coverage_y(0, 4, 64) == (0, 64)
    assert G.coverage_y(2, 5, 70) == (32, 70)  # the last tile row is clipped to the image
