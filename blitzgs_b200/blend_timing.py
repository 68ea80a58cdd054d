"""Blend kernel timing with and without the per-strip contributor lists.

    python -m blitzgs_b200.blend_timing

Renders four cameras of the city workload (8M Gaussians, z-order layout)
through the training step, keeps each view's real blend inputs, then times
blitz_render_blend (lists recorded or not) and blitz_render_backward (full
list walk or strip lists) on them with CUDA events (warm L2, 10 rounds of
the four views, median of 5 repetitions), after checking that the forward
outputs are unchanged and the backward records agree.  Timing tool, not a
test: needs a GPU and the built library."""
import statistics

import torch

from . import _lib as L
from . import distributed as D
from . import ops, scene as S, step as ST


def main():
    dev = torch.device("cuda", 0)
    sc = S.city(seed=0)
    order = D.zorder_shards(sc.xyz, 1)[0]
    model = [t[order].contiguous().to(dev).requires_grad_(True) for t in
             (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)]
    views = []
    for ci in range(4):
        cam = sc.cameras[ci].to(dev)
        gt = S.target_image(ci, cam.image_height, cam.image_width).to(dev)
        loss, *_ = ST.view_loss(model, S.raster_settings(cam, device=dev), gt, sparse_grad=True)
        holder = []
        orig_rb = ops.render_backward

        def rb(state, means2D, conic, rgb, bg, cl, dL_dpix, grad_accum=None, record_rows=None, n_rows=None):
            holder.append((state, means2D, conic, rgb, bg, cl, dL_dpix.clone(), record_rows, n_rows))
            return orig_rb(state, means2D, conic, rgb, bg, cl, dL_dpix, grad_accum, record_rows, n_rows)

        ops.render_backward = rb
        loss.backward()
        ops.render_backward = orig_rb
        torch.cuda.synchronize()
        views.append(holder[0])
    lib = L.load()
    st = L.stream_ptr()
    print("R per view:", [v[0].R for v in views], "active entries:",
          [int(v[0].strip_counts.sum()) for v in views], flush=True)


    def fwd(v, lists, outs):
        state, means2D, conic, rgb, bg, cl = v[:6]
        T = state.ranges.numel() // 2
        return lib.blitz_render_blend(means2D.shape[0], state.H, state.W, L.ptr(means2D), L.ptr(conic), L.ptr(rgb),
                                      L.ptr(bg), None, L.ptr(state.point_list), L.ptr(state.ranges), L.ptr(outs[0]),
                                      L.ptr(outs[1]), L.ptr(outs[2]), L.ptr(outs[3]), L.ptr(outs[4]), L.ptr(outs[5]),
                                      L.ptr(outs[6]), *(L.ptr(x) for x in (lists if lists else (None, None, None))), st)


    def bwd(v, lists, acc):
        state, means2D, conic, rgb, bg, cl, dL_dpix, record_rows, n_rows = v
        lz = (state.strip_ids, state.strip_pos, state.strip_counts) if lists else (None, None, None)
        return lib.blitz_render_backward(means2D.shape[0], state.H, state.W, L.ptr(state.point_list), L.ptr(state.ranges),
                                         L.ptr(state.final_T), L.ptr(state.n_contrib), L.ptr(means2D), L.ptr(conic),
                                         L.ptr(rgb), L.ptr(bg), None, L.ptr(dL_dpix), L.ptr(record_rows),
                                         *(L.ptr(x) for x in lz), L.ptr(acc), st)


    outs = []
    for v in views:
        state, means2D = v[0], v[1]
        H, W, T = state.H, state.W, state.ranges.numel() // 2
        o = [torch.empty(H * W, device=dev), torch.empty(H * W, dtype=torch.int32, device=dev),
             torch.empty(3, H, W, device=dev)] + [torch.empty(T, dtype=torch.int32, device=dev) for _ in range(3)] + \
            [torch.zeros(means2D.shape[0], dtype=torch.int32, device=dev)]
        lz = [torch.empty(8 * state.R, dtype=torch.int32, device=dev), torch.empty(8 * state.R, dtype=torch.int32, device=dev),
              torch.empty(8 * T, dtype=torch.int32, device=dev)]
        outs.append((o, lz))
    for vi, v in enumerate(views):
        o, lz = outs[vi]
        assert fwd(v, None, o) == 0
        c0 = o[2].clone(); n0 = o[1].clone()
        assert fwd(v, lz, o) == 0
        torch.cuda.synchronize()
        same = torch.equal(c0, o[2]) and torch.equal(n0, o[1])
        samelists = torch.equal(lz[2], v[0].strip_counts)
        rows = max(int(v[8]), 1)
        a = torch.zeros(rows, 16, device=dev); b = torch.zeros(rows, 16, device=dev)
        assert bwd(v, False, a) == 0 and bwd(v, True, b) == 0
        torch.cuda.synchronize()
        print(f"view {vi}: fwd same with lists {same}, counts same as step's {samelists}, "
              f"bwd lists vs walk rel err {((a - b).norm() / a.norm()).item():.2e}", flush=True)

    res = {k: [] for k in ("fwd_walk", "fwd_lists", "bwd_walk", "bwd_lists")}
    acc = [torch.zeros(max(int(v[8]), 1), 16, device=dev) for v in views]
    for rep in range(6):
        for k in res:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(10):
                for vi, v in enumerate(views):
                    if k == "fwd_walk":
                        fwd(v, None, outs[vi][0])
                    elif k == "fwd_lists":
                        fwd(v, outs[vi][1], outs[vi][0])
                    elif k == "bwd_walk":
                        bwd(v, False, acc[vi])
                    else:
                        bwd(v, True, acc[vi])
            e1.record()
            torch.cuda.synchronize()
            res[k].append(e0.elapsed_time(e1) / (10 * len(views)))
    for k, t in res.items():
        print(f"{k:10s} {statistics.median(t[1:]):.4f} ms (min {min(t[1:]):.4f})")


if __name__ == "__main__":
    main()
