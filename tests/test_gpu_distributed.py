"""N-GPU step vs the single-GPU step on the same seeded scene (needs >= 2 GPUs).

Two NCCL ranks, each owning a z-order shard; the batch's cameras are split
into tile-row bands by start_strategy_final.  Gradients are gathered by
global Gaussian id and compared with the single-GPU result of the same band
layout (tolerance: 1e-4 relative, normwise, per parameter tensor)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WS = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _scene():
    from blitzgs_b200 import scene as S
    sc = S.tiny(seed=31, P=30000, H=192, W=256)
    # a second camera from another side
    c2 = S.look_at_camera([2.5, -0.5, -1.5], [0, 0, 0], [0, -1, 0], 256, 192, 1.0, uid=1)
    sc.cameras.append(c2)
    return sc


def _single_gpu_reference(sc, cam_ids, bands, dev):
    """Per-camera band losses computed on one GPU exactly as the ranks do."""
    from blitzgs_b200 import scene as S, step as ST
    model = [t.to(dev).requires_grad_(True) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                      sc.features_dc, sc.features_rest)]
    total = 0
    for k, c in enumerate(cam_ids):
        cam = sc.cameras[c].to(dev)
        gt = S.target_image(c, cam.image_height, cam.image_width).to(dev)
        rs = S.raster_settings(cam, device=dev)
        H, W = cam.image_height, cam.image_width
        for (r0, r1) in bands[k]:
            cl = torch.zeros(((H + 15) // 16, (W + 15) // 16), dtype=torch.bool, device=dev)
            cl[r0:r1] = True
            y0, y1 = r0 * 16, min(H, r1 * 16)
            loss, *_ = ST.view_loss(model, rs, gt[:, y0:y1], compute_locally=cl, band=(y0, y1), scale_reg_weight=0.0)
            total = total + loss
    total.backward()
    return float(total.item()), [p.grad.detach().cpu() for p in model]


def _worker(rank, port, cam_ids, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WS, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from blitzgs_b200 import distributed as D, dist_step as DS, scene as S
        sc = _scene()
        H, W = 192, 256
        D.init_context(rank, WS, H, W, bsz=len(cam_ids))
        shard = D.zorder_shards(sc.xyz, WS)[rank]
        model = [t[shard].contiguous().to(dev).requires_grad_(True)
                 for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)]
        cams = [sc.cameras[c] for c in cam_ids]
        hist = D.DivisionStrategyHistoryFinal(cams, WS, rank)
        strategies, _ = D.start_strategy_final(cams, hist)
        rasters = [S.raster_settings(c.to(dev), device=dev) for c in cams]
        gts = []
        for k, c in enumerate(cam_ids):
            rr = strategies[k].row_range(rank)
            if rr is None:
                gts.append(None)
                continue
            g = S.target_image(c, H, W).to(dev)
            gts.append(g[:, rr[0] * 16: min(H, rr[1] * 16)])
        loss = DS.batch_loss(model, rasters, gts, strategies, reg_w=0.0)
        loss.backward()
        lt = loss.detach().reshape(1)
        dist.all_reduce(lt)
        grads = []
        for p in model:
            full = torch.zeros((sc.P,) + tuple(p.shape[1:]), device=dev)
            full[shard.to(dev)] = p.grad
            dist.all_reduce(full)
            grads.append(full.cpu())
        bands = [[tuple(st.division_pos[i:i + 2]) for i in range(st.world_size)] for st in strategies]
        if rank == 0:
            q.put(("ok", float(lt.item()), grads, bands))
        dist.barrier()
    except BaseException as ex:
        q.put(("err", repr(ex), None, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cam_ids", [[0, 1], [0]], ids=["whole-views", "split-view"])
def test_two_rank_step_matches_single_gpu(cam_ids):
    if torch.cuda.device_count() < WS:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, cam_ids, q)) for r in range(WS)]
    for p in procs:
        p.start()
    status, loss, grads, bands = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert status == "ok", loss
    sc = _scene()
    ref_loss, ref_grads = _single_gpu_reference(sc, cam_ids, bands, torch.device("cuda", 0))
    assert abs(loss - ref_loss) < 1e-5 * max(1.0, abs(ref_loss)), (loss, ref_loss)
    from tests.helpers import assert_grad_close
    for n, a, b in zip(["xyz", "scaling", "rotation", "opacity", "dc", "rest"], grads, ref_grads):
        assert_grad_close(a, b, 1e-4, n)
