"""Fused single-process training step: preprocess -> binning -> blend -> L1+SSIM
-> backward, per camera, on the sm_100a kernels.

This is the body of the reference's distributed_preprocess3dgs_and_all2all_final
+ render_final + batched_loss_computation + loss.backward() for the Gaussians
and tile rows a rank owns (gaussian_renderer/__init__.py:220-413, 664-854,
gaussian_renderer/loss_distribution.py:220-329), with these changes, which keep
results identical:
  * SH coefficients are read from _features_dc / _features_rest in place (the
    reference concatenates them with torch.cat and splits them again in C++);
  * one autograd node per camera covers preprocess, render and loss, so no
    per-Gaussian intermediate is materialised for autograd and the render
    gradient record [P,16] feeds the preprocess backward directly;
  * the only host synchronisation is the two-number readback that sizes the
    binning buffers;
  * the loss is combined from the L1/SSIM sums and the regulariser on the
    device, with the float32 rounding of the same PyTorch expression, so no
    scalar PyTorch op (or its autograd node) runs per camera;
  * the blend forward records each 8x4-pixel strip's contributing Gaussians
    and the blend backward replays only those (same pairs, same order).
Parameter activations (exp, sigmoid, normalize) run inside the preprocess
kernels with PyTorch's float arithmetic, and their backward is chained there
too, so no activation or regulariser kernel runs in PyTorch.
"""
import sys

import torch
from torch.autograd.graph import get_gradient_edge

from . import densify as D
from . import ops

LAMBDA_DSSIM = 0.2


class _GradBuffers:
    """Dense parameter gradients written in place.

    A camera's dense gradient is zero except at the rows of the Gaussians it
    sees (a few percent of the model), yet a fresh dense tensor has to be
    zero-filled in full (236 B per Gaussian, 1.9 GB per view at 8M).  When
    ``loss.backward()`` would accumulate into the parameters' ``.grad``, the
    fused step writes those rows straight into ``.grad`` instead: into the
    existing gradient (accumulating over the views of a batch), or, when
    ``.grad`` is None, into a buffer kept here whose rows written earlier are
    zeroed again -- only those rows -- before it is handed out.  A buffer is
    reused only when nothing else references its memory and its version
    counter shows no in-place change since this class last wrote it;
    otherwise it is zero-filled in full.  Not used under
    ``torch.autograd.grad`` or with gradient hooks on the parameters (the
    gradients are then returned the usual way)."""

    def __init__(self):
        self._entries = []  # dicts: t (buffer), dirty (row index tensors), version

    @staticmethod
    def _unshared(t):
        # references: the entry, the caller's local and this call's argument
        return sys.getrefcount(t) <= 4 and torch._C._storage_Use_Count(t.untyped_storage()._cdata) <= 2

    @staticmethod
    def _clean(entries):
        """Zero what earlier views wrote into the buffers: the listed rows,
        in one launch per row list for every buffer that shares it, or the
        whole buffer when its contents are unknown."""
        lists = {}
        for e in entries:
            t = e["t"]
            if e["dirty"] is None or e["version"] != t._version:
                t.zero_()
            else:
                for rows, n in e["dirty"]:
                    lists.setdefault(id(rows), (rows, n, []))[2].append(t)
            e["dirty"] = []
        for rows, n, ts in lists.values():
            for k in range(0, len(ts), 8):
                ops.zero_rows(ts[k:k + 8], rows, n)
        for e in entries:
            e["version"] = e["t"]._version

    def _take(self, like, taken):
        for e in self._entries:
            t = e["t"]
            if (t.shape == like.shape and t.dtype == like.dtype and t.device == like.device
                    and not any(e is x for x in taken) and self._unshared(t)):
                return e
        e = {"t": torch.empty_like(like, memory_format=torch.contiguous_format), "dirty": None, "version": -1}
        self._entries.append(e)
        return e

    def _owned(self, g):
        for e in self._entries:
            if e["t"] is g:
                return e
        return None

    def targets(self, params, nodes):
        """(entries, accumulate) to write this view's gradient rows into, or
        None to return the gradients the usual way."""
        try:
            if not all(torch._C._will_engine_execute_node(n) for n in nodes):
                return None
        except RuntimeError:  # torch.autograd.grad: no accumulation into .grad
            return None
        for p in params:
            if p._backward_hooks or getattr(p, "_post_accumulate_grad_hooks", None):
                return None
        gs = [p.grad for p in params]
        if all(g is None for g in gs):
            taken = []
            for p in params:  # parameters of one shape get one buffer each
                taken.append(self._take(p, taken))
            self._clean(taken)
            return taken, False
        if any(g is None for g in gs):
            return None
        out = []
        for p, g in zip(params, gs):
            e = self._owned(g)
            if e is not None and e["version"] == g._version:
                out.append(e)
            elif (g.layout == torch.strided and g.is_contiguous() and g.dtype == torch.float32
                  and g.device == p.device and g.shape == p.shape and not g.requires_grad):
                out.append({"t": g, "foreign": True})  # a gradient we do not track: add to it
            else:
                return None
        return out, True

    def written(self, params, entries, rows, fresh):
        """``rows`` = (device index tensor, count): the rows this view wrote."""
        for p, e in zip(params, entries):
            if fresh:
                p.grad = e["t"]
            if not e.get("foreign"):
                e["dirty"].append(rows)
                e["version"] = e["t"]._version


_GRADS = _GradBuffers()


class _ViewLoss(torch.autograd.Function):
    """Raw parameters (xyz, _scaling, _rotation, _opacity, _features_dc,
    _features_rest) -> (loss, sum L1, sum SSIM) of one camera band;
    activations, loss combination and their backward run in the kernels, so
    the whole camera is one autograd node."""

    @staticmethod
    def forward(ctx, xyz, s_raw, q_raw, o_raw, dc, rest, raster, gt, compute_locally, band, exact_norm, sparse_grad,
                lambda_dssim, reg_weight, densify):
        H, W = int(raster.image_height), int(raster.image_width)
        sh = ops.sh_layout(dc=dc, rest=rest)
        rot_norm = q_raw.norm(dim=1) if exact_norm else None
        use_list = compute_locally is None or sparse_grad
        means2D, depths, radii, conic, rgb, reg, vlist, vcount, counts, totals, slot_of = ops.preprocess_forward_raw(
            xyz, s_raw, q_raw, o_raw.reshape(-1), sh, raster, rot_norm, want_reg=True, want_list=use_list,
            want_counts=True, compute_locally=compute_locally, want_slots=use_list)
        color, n_render, n_consider, n_contrib, out_observe, state = ops.render_forward(
            means2D, depths, radii, conic, rgb, raster.bg, compute_locally, H, W, counts=counts, totals=totals,
            vis_count=vcount)
        y0, y1 = band
        img_band = color[:, y0:y1, :]
        sums, partials = ops.loss_forward(img_band, gt)
        consts = (lambda_dssim, H * W * 3, reg_weight)
        out = ops.loss_combine(sums, reg if reg_weight else None, *consts)
        ctx.raster = raster
        ctx.band = band
        ctx.HW = (H, W)
        ctx.state = state
        ctx.cl = compute_locally
        ctx.sparse_grad = sparse_grad
        ctx.consts = consts
        ctx.densify = densify
        ctx.params = None
        if not sparse_grad and vlist is not None:
            params = (xyz, s_raw, q_raw, o_raw, dc, rest)
            if all(t.is_leaf and t.requires_grad for t in params):
                ctx.params = params
                ctx.nodes = [get_gradient_edge(t).node for t in params]
        if densify is not None:
            D.update_max_radii(densify, radii)
        ctx.save_for_backward(xyz, s_raw, q_raw, o_raw, dc, rest, means2D, conic, rgb, radii, gt, partials,
                              img_band, rot_norm, vlist, vcount, slot_of, out)
        ctx.mark_non_differentiable(radii, out_observe, color)
        return out[0], out[1], out[2], radii, out_observe, color

    @staticmethod
    def backward(ctx, g_loss, g_l1, g_ss, *_unused):
        (xyz, s_raw, q_raw, o_raw, dc, rest, means2D, conic, rgb, radii, gt, partials, img_band, rot_norm, vlist,
         vcount, slot_of, out) = ctx.saved_tensors
        H, W = ctx.HW
        y0, y1 = ctx.band
        dev = xyz.device
        scales = ops.loss_combine_backward(g_loss, g_l1, g_ss, out, *ctx.consts)
        g_band = ops.loss_backward(img_band, gt, partials, scales[0:2])
        if y0 == 0 and y1 == H:
            dL_dpix = g_band
        else:
            dL_dpix = torch.zeros((3, H, W), dtype=torch.float32, device=dev)
            dL_dpix[:, y0:y1, :] = g_band
        L = ctx.state.n_list
        grads_dense = None
        inplace = _GRADS.targets(ctx.params, ctx.nodes) if ctx.params is not None else None
        if inplace is None and not ctx.sparse_grad and vlist is not None:
            # The dense gradients are zero except at listed rows.  Their fill is
            # pure HBM writes (236 B per Gaussian); on a side stream it runs
            # beside the issue-bound loss and render backward instead of after them.
            grads_dense = [torch.empty_like(t) for t in (xyz, s_raw, q_raw, o_raw, dc, rest)]
            _zero_fill_async(grads_dense)
        try:
            # gradient record: one row per listed Gaussian (slot_of) instead of P rows
            rec = ops.render_backward(ctx.state, means2D, conic, rgb, ctx.raster.bg, ctx.cl, dL_dpix,
                                      record_rows=slot_of, n_rows=L)
        finally:
            if grads_dense is not None:
                _zero_fill_wait()
        if ctx.densify is not None:
            # the viewspace gradient of the visible Gaussians: record rows
            # are list slots (slot_of) or, without a list, Gaussian ids
            if slot_of is not None:
                D.accumulate_grad(ctx.densify, vlist[:L].to(torch.int64), rec[:L, 0:2])
            else:
                vis = torch.nonzero(radii > 0).flatten()
                D.accumulate_grad(ctx.densify, vis, rec[vis, 0:2])
        sh = ops.sh_layout(dc=dc, rest=rest)
        M = rest.shape[1]
        rows = ops.ROWS_UPSTREAM_BY_SLOT if slot_of is not None else 0
        if ctx.sparse_grad:
            # row j = the j-th listed Gaussian: every row written, no P-sized buffer
            rows |= ops.ROWS_OUTPUT_BY_SLOT
            n = max(L, 1)
            shapes = [xyz.shape[1:], s_raw.shape[1:], q_raw.shape[1:], o_raw.shape[1:], dc.shape[1:], rest.shape[1:]]
            g_xyz, g_s, g_q, g_o, g_dc, g_rest = [torch.empty((n,) + tuple(sz), dtype=torch.float32, device=dev)
                                                  for sz in shapes]
        elif inplace is not None:
            g_xyz, g_s, g_q, g_o, g_dc, g_rest = [e["t"] for e in inplace[0]]
        elif grads_dense is not None:
            g_xyz, g_s, g_q, g_o, g_dc, g_rest = grads_dense
        else:
            g_xyz, g_s, g_q, g_dc, g_rest = (torch.empty_like(t) for t in (xyz, s_raw, q_raw, dc, rest))
            g_o = torch.empty_like(o_raw)
        ops.preprocess_backward_raw(radii, means2D, xyz, s_raw, q_raw, o_raw.reshape(-1), sh, ctx.raster,
                                    rec[:, 0:2], rec[:, 8:12], rec[:, 12:15],
                                    (g_xyz, g_s, g_q, g_o, (g_dc, 3), (g_rest, max(M, 1) * 3)), rot_norm=rot_norm,
                                    reg_scale=scales[2:3], vis_list=vlist, vis_count=vcount, rows=rows,
                                    accumulate=inplace is not None and inplace[1])
        if inplace is not None:
            # written straight into .grad: nothing left for autograd to accumulate
            _GRADS.written(ctx.params, inplace[0], (vlist, L), fresh=not inplace[1])
            return (None,) * 15
        grads = [g_xyz, g_s, g_q, g_o, g_dc, g_rest]
        if ctx.sparse_grad:
            idx = vlist[:L].to(torch.int64).unsqueeze(0)
            # the rows are the visible list: unique and in range by construction
            with torch.sparse.check_sparse_tensor_invariants(enable=False):
                grads = [torch.sparse_coo_tensor(idx, g[:L], p.shape, check_invariants=False)
                         for g, p in zip(grads, (xyz, s_raw, q_raw, o_raw, dc, rest))]
        return (*grads, None, None, None, None, None, None, None, None, None)


def _zero_fill_async(tensors):
    """Zero ``tensors`` on the library's side stream, after the current
    stream's pending work (which may still use their recycled memory).  The
    caller runs ``_zero_fill_wait()`` before the current stream touches them,
    so every later use and free is ordered after the fill on the tensors' own
    stream (no record_stream: that would hold the memory back from the
    allocator's reuse)."""
    ops.zero_fill_async(tensors)


def _zero_fill_wait():
    ops.zero_fill_wait()


def view_loss(model, raster, gt_band, compute_locally=None, band=None, lambda_dssim=LAMBDA_DSSIM,
              scale_reg_weight=10.0, exact_norm=False, sparse_grad=False, densify=None):
    """Loss of one camera exactly as batched_loss_computation forms it
    (loss_distribution.py:303-322): (1-l) L1/N3 + l (1 - SSIM/N3) +
    10 mean(min-axis scale of the Gaussians the exchange sends), N3 = 3 H W.

    ``model`` = raw (xyz, _scaling, _rotation, _opacity, _features_dc,
    _features_rest); the activations run inside the preprocess kernels.
    The kernel computes ||_rotation|| with the summation order of PyTorch's
    norm (bit-identical); ``exact_norm=True`` takes it from PyTorch instead.
    ``sparse_grad=True`` makes the parameter gradients sparse COO tensors
    holding only the rows of the Gaussians with radius > 0 (every other row
    of the dense gradient is exactly zero), for optimizers that take sparse
    gradients such as torch.optim.SparseAdam -- the update rule of the
    reference's SparseGaussianAdam, which only touches visible rows.
    ``densify`` (a densify.DensificationStats) receives this camera's
    densification statistics: max_radii2D in the forward, the viewspace
    gradient norm and count of every visible Gaussian in the backward.
    Returns (loss, l1_sum, ssim_sum, radii, out_observe, color)."""
    xyz, s_raw, q_raw, o_raw, dc, rest = model
    H = int(raster.image_height)
    band = band or (0, H)
    return _ViewLoss.apply(xyz, s_raw, q_raw, o_raw, dc, rest, raster, gt_band, compute_locally, band, exact_norm,
                           sparse_grad, float(lambda_dssim), float(scale_reg_weight), densify)
