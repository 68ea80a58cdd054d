"""N-GPU step vs the single-GPU step on the same seeded scene (needs >= 2 GPUs).

Two NCCL ranks, each owning a z-order shard of a scene stored in z-order
(as the bench stores it); the batch's cameras are split into tile-row bands
by start_strategy_final.  Each rank's received rows arrive in ascending
global id, so its per-tile Gaussian lists, tile ranges, per-pixel
contributor counts and image are bit-identical to the single-GPU render of
the same band.  Gradients are gathered by global Gaussian id and compared
with the single-GPU result of the same band layout (tolerance: 1e-4
relative, normwise, per parameter tensor).  With densification statistics
(``batch_loss(densify=...)``) and every camera rendered whole by one rank,
the gathered max_radii2D and denom equal those of the single-GPU step
exactly and the accumulated viewspace-gradient norms agree within 1e-4."""
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
    from blitzgs_b200 import distributed as D, scene as S
    sc = S.tiny(seed=31, P=30000, H=192, W=256)
    # a second camera from another side
    c2 = S.look_at_camera([2.5, -0.5, -1.5], [0, 0, 0], [0, -1, 0], 256, 192, 1.0, uid=1)
    sc.cameras.append(c2)
    order = D.zorder_shards(sc.xyz, 1)[0]  # stored in z-order: the shards are contiguous id ranges
    for n in ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"):
        setattr(sc, n, getattr(sc, n)[order].contiguous())
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


def _single_gpu_densify(sc, cam_ids, dev):
    """Densification statistics of the single-GPU step over whole views."""
    from blitzgs_b200 import densify as DZ, scene as S, step as ST
    model = [t.to(dev).requires_grad_(True) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                      sc.features_dc, sc.features_rest)]
    stats = DZ.DensificationStats(sc.P, dev)
    total = 0
    for c in cam_ids:
        cam = sc.cameras[c].to(dev)
        gt = S.target_image(c, cam.image_height, cam.image_width).to(dev)
        rs = S.raster_settings(cam, device=dev)
        loss, *_ = ST.view_loss(model, rs, gt, scale_reg_weight=0.0, densify=stats)
        total = total + loss
    total.backward()
    return [t.detach().cpu() for t in (stats.max_radii2D, stats.xyz_gradient_accum, stats.denom)]


def _worker(rank, port, cam_ids, q, densify=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WS, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from blitzgs_b200 import densify as DZ, distributed as D, dist_step as DS, ops, scene as S
        captured = []
        real_render = ops.render_forward

        def capture(*a, **k):
            out = real_render(*a, **k)
            color, st = out[0], out[5]
            captured.append((color.cpu(), st.point_list[:st.R].cpu(), st.ranges.cpu(), st.n_contrib.cpu()))
            return out

        ops.render_forward = capture
        sc = _scene()
        H, W = 192, 256
        D.init_context(rank, WS, H, W, bsz=len(cam_ids))
        shard = D.zorder_shards(sc.xyz, WS)[rank]
        assert torch.equal(shard, torch.arange(int(shard[0]), int(shard[0]) + len(shard)))
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
        stats = DZ.DensificationStats(len(shard), dev) if densify else None
        loss = DS.batch_loss(model, rasters, gts, strategies, reg_w=0.0, densify=stats)
        loss.backward()
        lt = loss.detach().reshape(1)
        dist.all_reduce(lt)
        grads = []
        for p in model:
            full = torch.zeros((sc.P,) + tuple(p.shape[1:]), device=dev)
            full[shard.to(dev)] = p.grad
            dist.all_reduce(full)
            grads.append(full.cpu())
        dz = None
        if stats is not None:
            # shards are disjoint id ranges: the sum of the zero-padded rows is the whole
            dz = []
            for t in (stats.max_radii2D, stats.xyz_gradient_accum, stats.denom):
                full = torch.zeros((sc.P,) + tuple(t.shape[1:]), device=dev)
                full[shard.to(dev)] = t
                dist.all_reduce(full)
                dz.append(full.cpu())
        bands = [[tuple(st.division_pos[i:i + 2]) for i in range(st.world_size)] for st in strategies]
        mine = [(k, strategies[k].row_range(rank)) for k in range(len(cam_ids)) if rank in strategies[k].gpu_ids]
        q.put(("renders", rank, list(zip(mine, captured)), None, None))
        if rank == 0:
            q.put(("ok", float(lt.item()), grads, bands, dz))
        dist.barrier()
    except BaseException as ex:
        q.put(("err", repr(ex), None, None, None))
    finally:
        dist.destroy_process_group()


def _run(cam_ids, densify=False):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, cam_ids, q, densify)) for r in range(WS)]
    for p in procs:
        p.start()
    renders, result = [], None
    for _ in range(WS + 1):
        item = q.get(timeout=300)
        if item[0] == "renders":
            renders += item[2]
        elif item[0] == "err":
            result = item
            break
        else:
            result = item
    for p in procs:
        p.join(timeout=120)
    assert result[0] == "ok", result[1]
    return renders, result


@pytest.mark.parametrize("cam_ids", [[0, 1], [0]], ids=["whole-views", "split-view"])
def test_two_rank_step_matches_single_gpu(cam_ids):
    if torch.cuda.device_count() < WS:
        pytest.skip("needs 2 GPUs")
    renders, (_, loss, grads, bands, _) = _run(cam_ids)
    sc = _scene()
    _check_renders_bit_identical(sc, cam_ids, renders)
    ref_loss, ref_grads = _single_gpu_reference(sc, cam_ids, bands, torch.device("cuda", 0))
    assert abs(loss - ref_loss) < 1e-5 * max(1.0, abs(ref_loss)), (loss, ref_loss)
    from tests.helpers import assert_grad_close
    for n, a, b in zip(["xyz", "scaling", "rotation", "opacity", "dc", "rest"], grads, ref_grads):
        assert_grad_close(a, b, 1e-4, n)


def test_two_rank_densification_stats_match_single_gpu():
    """batch_loss(densify=...) on two ranks: every camera of the batch is
    rendered whole by one rank, so each owner's statistics (max radius, the
    norm of the viewspace gradient summed over the receivers, the count) are
    those of the single-GPU step over the same whole views."""
    if torch.cuda.device_count() < WS:
        pytest.skip("needs 2 GPUs")
    cam_ids = [0, 1]
    _, (_, _, _, bands, dz) = _run(cam_ids, densify=True)
    sc = _scene()
    gy = (sc.cameras[0].image_height + 15) // 16
    for k, b in enumerate(bands):
        nonempty = [(r0, r1) for r0, r1 in b if r1 > r0]
        assert nonempty == [(0, gy)], f"camera {k} is not rendered whole by one rank: {b}"
    ref = _single_gpu_densify(sc, cam_ids, torch.device("cuda", 0))
    assert torch.equal(dz[0], ref[0]), "max_radii2D differs"
    assert torch.equal(dz[2], ref[2]), "denom differs"
    from tests.helpers import assert_grad_close
    assert_grad_close(dz[1], ref[1], 1e-4, "xyz_gradient_accum")


def _check_renders_bit_identical(sc, cam_ids, renders):
    """Each rank's band render equals the single-GPU render of that band:
    its received rows are the Gaussians routed to it in ascending global id,
    so mapping its per-tile lists through that id list gives the single-GPU
    lists exactly."""
    from blitzgs_b200 import ops, scene as S
    dev = torch.device("cuda", 0)
    xyz, s_raw, q_raw, o_raw, dc, rest = [t.to(dev) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                              sc.features_dc, sc.features_rest)]
    assert renders, "no rank rendered anything"
    for (k, (r0, r1)), (color, pl, ranges, n_contrib) in renders:
        cam = sc.cameras[cam_ids[k]].to(dev)
        rs = S.raster_settings(cam, device=dev)
        H, W = cam.image_height, cam.image_width
        gx, gy = ops.grid_dims(H, W)
        m2, d, r, co, rgb = ops.preprocess_forward_raw(xyz, s_raw, q_raw, o_raw.reshape(-1),
                                                       ops.sh_layout(dc=dc, rest=rest), rs, want_list=False,
                                                       two_pass=False)[:5]
        routed = ops.local2j_ids_bool(H, W, 0, 1, m2, r, torch.tensor([r0 * gx, r1 * gx], dtype=torch.int32,
                                                                         device=dev))[:, 0] & (r > 0)
        gids = torch.nonzero(routed).flatten().cpu()
        cl = torch.zeros((gy, gx), dtype=torch.bool, device=dev)
        cl[r0:r1] = True
        ref_color, _, _, _, _, st = ops.render_forward(m2, d, r, co, rgb, rs.bg, cl, H, W)
        assert len(pl) == st.R, (k, len(pl), st.R)
        assert torch.equal(gids[pl.long()], st.point_list[:st.R].cpu().long()), f"camera {k}: tile lists differ"
        assert torch.equal(ranges, st.ranges.cpu()), f"camera {k}: ranges differ"
        y0, y1 = r0 * 16, min(H, r1 * 16)
        nc_ref = st.n_contrib.cpu().view(H, W)[y0:y1]
        assert torch.equal(n_contrib.view(H, W)[y0:y1], nc_ref), f"camera {k}: n_contrib differs"
        assert torch.equal(color[:, y0:y1].view(torch.int32), ref_color.cpu()[:, y0:y1].view(torch.int32)), \
            f"camera {k}: band image differs"
