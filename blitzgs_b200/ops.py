"""Tensor-level wrappers of the C ABI: allocate outputs, call, return tensors.

These are the building blocks of both the reference-compatible operator API
(``blitzgs_b200.rasterizer``) and the fused training step
(``blitzgs_b200.step``).  Every function runs on the current CUDA stream and
raises if the native library is absent or the tensors are not on a GPU.
"""
import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ptr

TILE = 16


class StageTimer:
    """Optional CUDA-event timing of each native call, on the launching stream.

    Disabled by default (no events, no overhead).  When enabled, every wrapper
    below records (stage, start, end) events; ``summary()`` synchronises and
    returns {stage: (calls, total_ms)}.  Used by bench.py for the live
    per-kernel roofline numbers."""

    def __init__(self):
        self.enabled = False
        self.records = []

    def begin(self, name):
        if not self.enabled:
            return None
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        return (name, a, b)

    def end(self, tok, lazy=None, **meta):
        """Record the end event; ``lazy`` (a callable returning a dict) is
        evaluated only after it, so its kernels stay outside the timed span."""
        if tok is None:
            return
        tok[2].record()
        if lazy is not None:
            meta.update(lazy())
        self.records.append((tok[0], tok[1], tok[2], meta))

    def summary(self):
        out = {}
        for name, a, b, meta in self.records:
            b.synchronize()
            c, t, m = out.get(name, (0, 0.0, []))
            out[name] = (c + 1, t + a.elapsed_time(b), m + [meta])
        return out

    def reset(self):
        self.records = []


TIMER = StageTimer()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("blitzgs_b200 operators need CUDA tensors (there is no CPU path)")


def _f32c(t):
    if t.dtype != torch.float32:
        raise RuntimeError(f"expected float32 tensor, got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def grid_dims(H, W):
    return (W + TILE - 1) // TILE, (H + TILE - 1) // TILE


class _Scratch:
    """Grow-only per-device scratch buffer (never shrinks).  ``zeroed``
    buffers start at zero when (re)allocated."""

    def __init__(self, zeroed=False):
        self.bufs = {}
        self.zeroed = zeroed

    def get(self, device, nbytes):
        key = (device.type, device.index)
        buf = self.bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            cap = max(nbytes, int((buf.numel() if buf is not None else 0) * 1.25))
            cap = (cap + (1 << 20) - 1) // (1 << 20) * (1 << 20)
            self.bufs[key] = None
            buf = (torch.zeros if self.zeroed else torch.empty)(cap, dtype=torch.uint8, device=device)
            self.bufs[key] = buf
        return buf

    def peek(self, device):
        return self.bufs.get((device.type, device.index))


SCRATCH = _Scratch()
# candidate list and ordered-scan state of the two-kernel raw preprocess; its
# first 4 bytes are the scans' status word (checked at the totals readback)
PRE_SCRATCH = _Scratch(zeroed=True)


def sh_layout(shs=None, dc=None, rest=None):
    """Return (dc, dc_stride, rest, rest_stride, M) for the kernel's SH addressing.

    Either ``shs`` [P,K,3] (K coefficients, DC first, contiguous) or the split
    ``dc`` [P,1,3] / ``rest`` [P,K-1,3] tensors (each contiguous) are read in
    place without copies.
    """
    if shs is not None:
        shs = _f32c(shs)
        if shs.dim() != 3 or shs.shape[2] != 3 or shs.shape[1] < 1:
            raise RuntimeError("sh must have dimensions (num_points, num_sh_coeffs, 3) with num_sh_coeffs >= 1")
        K = shs.shape[1]
        stride = K * 3
        rest_t = shs.view(-1)[3:] if K > 1 else shs
        return shs, stride, rest_t, stride, K - 1, (shs,)
    dc = _f32c(dc)
    rest = _f32c(rest)
    M = rest.shape[1] if rest.dim() == 3 else 0
    return dc, 3, rest, max(M, 1) * 3, M, (dc, rest)


def preprocess_forward(means3D, scales, rotations, opacities, sh, raster, *, want_cov3D=False,
                       want_clamped=False, error_word=None, culling=None, want_rects=False):
    """EWA preprocess.  ``sh`` is the tuple from :func:`sh_layout`.
    ``culling`` (bool [P]) skips the Gaussians it marks; ``want_rects`` also
    returns the float half-extents [P,2] of each screen rectangle (the full
    rasterizer's binning input) as an eighth value."""
    _require_cuda(means3D, scales, rotations, opacities)
    means3D, scales, rotations = _f32c(means3D), _f32c(scales), _f32c(rotations)
    opacities = _f32c(opacities)
    dc, dcs, rest, rs, M, _keep = sh
    P = means3D.shape[0]
    dev = means3D.device
    means2D = torch.empty((P, 2), dtype=torch.float32, device=dev)
    depths = torch.empty((P,), dtype=torch.float32, device=dev)
    radii = torch.empty((P,), dtype=torch.int32, device=dev)
    conic = torch.empty((P, 4), dtype=torch.float32, device=dev)
    rgb = torch.empty((P, 3), dtype=torch.float32, device=dev)
    cov3D = torch.empty((P, 6), dtype=torch.float32, device=dev) if want_cov3D else None
    clamped = torch.empty((P, 3), dtype=torch.bool, device=dev) if want_clamped else None
    rects = torch.empty((P, 2), dtype=torch.float32, device=dev) if want_rects else None
    if culling is not None:
        culling = culling.reshape(-1).to(device=dev, dtype=torch.bool).contiguous()
        if culling.numel() != P:
            raise RuntimeError(f"culling must have {P} entries, got {culling.numel()}")
    if P > 0:
        tok = TIMER.begin("preprocess_fwd")
        _lib.call("blitz_preprocess_forward", P, int(raster.sh_degree), M, ptr(means3D), ptr(scales),
                  ptr(rotations), ptr(dc), dcs, ptr(rest), rs, ptr(opacities),
                  float(raster.scale_modifier), ptr(_f32c(raster.viewmatrix)),
                  ptr(_f32c(raster.projmatrix)), ptr(_f32c(raster.campos)), float(raster.tanfovx),
                  float(raster.tanfovy), int(raster.image_height), int(raster.image_width),
                  int(bool(raster.prefiltered)), ptr(means2D), ptr(depths), ptr(radii), ptr(cov3D),
                  ptr(conic), ptr(rgb), ptr(clamped), ptr(culling), ptr(rects), ptr(error_word),
                  _lib.stream_ptr())
        TIMER.end(tok, P=P)
    if want_rects:
        return means2D, depths, radii, conic, rgb, cov3D, clamped, rects
    return means2D, depths, radii, conic, rgb, cov3D, clamped


def preprocess_backward(radii, means3D, scales, rotations, sh, raster, g_means2D, g_conic, g_colors,
                        out=None, accumulate=False):
    """Backward of :func:`preprocess_forward`.

    ``g_means2D`` / ``g_conic`` / ``g_colors`` may be strided row views (e.g.
    slices of the [P,16] render-gradient record); rows are addressed with
    their row stride.  ``out`` = (dmeans3D, dscales, drot, dopacity, ddc, drest)
    to write into (required when ``accumulate``); ``ddc`` / ``drest`` follow the
    SH addressing of ``sh``'s layout with their own strides.
    """
    dc, dcs, rest, rs, M, _keep = sh
    P = means3D.shape[0]
    dev = means3D.device
    for g, w in ((g_means2D, 2), (g_conic, 4), (g_colors, 3)):
        if g.dim() != 2 or g.stride(1) != 1 or g.shape[1] < w:
            raise RuntimeError("gradient rows must be unit-stride")
    if out is None:
        dmeans3D = torch.empty((P, 3), dtype=torch.float32, device=dev)
        dscales = torch.empty((P, 3), dtype=torch.float32, device=dev)
        drot = torch.empty((P, 4), dtype=torch.float32, device=dev)
        dop = torch.empty((P, 1), dtype=torch.float32, device=dev)
        dsh = torch.empty((P, M + 1, 3), dtype=torch.float32, device=dev)
        ddc, ddcs = dsh, (M + 1) * 3
        drest, drs = dsh.view(-1)[3:] if M > 0 else dsh, (M + 1) * 3
        out_t = (dmeans3D, dscales, drot, dop, dsh)
    else:
        dmeans3D, dscales, drot, dop, (ddc, ddcs), (drest, drs) = out
        out_t = None
    if P > 0:
        tok = TIMER.begin("preprocess_bwd")
        _lib.call("blitz_preprocess_backward", P, int(raster.sh_degree), M, ptr(radii), ptr(means3D),
                  ptr(scales), ptr(rotations), ptr(dc), dcs, ptr(rest), rs,
                  float(raster.scale_modifier), ptr(raster.viewmatrix), ptr(raster.projmatrix),
                  ptr(raster.campos), float(raster.tanfovx), float(raster.tanfovy),
                  int(raster.image_height), int(raster.image_width), ptr(g_means2D), g_means2D.stride(0),
                  ptr(g_conic), g_conic.stride(0), ptr(g_colors), g_colors.stride(0), ptr(dmeans3D),
                  ptr(dscales), ptr(drot), ptr(dop), ptr(ddc), ddcs, ptr(drest), drs,
                  int(bool(accumulate)), _lib.stream_ptr())
        TIMER.end(tok, P=P, visible=None)
    elif out is None:
        for t in out_t:
            t.zero_()
    return out_t


def preprocess_forward_raw(xyz, scaling_raw, rotation_raw, opacity_raw, sh, raster, rot_norm=None, *,
                           want_reg=True, want_list=True, want_counts=False, compute_locally=None,
                           two_pass=True, want_slots=False, vis_count=None, exchange=None, out=None):
    """Preprocess from the raw model parameters (activations fused into the
    kernel).  Returns (means2D, depths, radii, conic_opacity, rgb, reg_sums
    double[2] or None, vis_list or None, vis_count or None, counts or None,
    totals or None, slot_of or None).

    With ``want_list`` only the rows of listed Gaussians (radius > 0) of
    means2D / depths / conic_opacity / rgb are written; radii is complete.
    ``want_counts`` fuses the binning's tile count (under ``compute_locally``)
    into the same kernel; pass counts/totals on to ``render_forward``.
    ``two_pass`` runs the cull and the full computation as two kernels (with
    a scratch candidate list); False runs the single persistent kernel.
    ``want_slots`` returns slot_of [P] (list position of each listed
    Gaussian), which indexes the compact gradient record of the backward.
    ``vis_count``: caller's zeroed int32 [1] counter for the list length.
    ``exchange`` = (tile_lo, tile_hi, records, dest_mask, dest_counts): the
    multi-GPU exchange outputs (see blitz_exchange_out in the C header).
    ``out`` = (means2D, depths, radii, conic_opacity, rgb, vis_list): caller
    buffers to write instead of fresh allocations."""
    _require_cuda(xyz, scaling_raw, rotation_raw, opacity_raw)
    xyz, scaling_raw, rotation_raw, opacity_raw = map(_f32c, (xyz, scaling_raw, rotation_raw, opacity_raw))
    dc, dcs, rest, rs, M, _keep = sh
    P = xyz.shape[0]
    dev = xyz.device
    H, W = int(raster.image_height), int(raster.image_width)
    if out is not None:
        means2D, depths, radii, conic, rgb, vlist = out
        vlist = vlist if want_list else None
    else:
        means2D = torch.empty((P, 2), dtype=torch.float32, device=dev)
        depths = torch.empty((P,), dtype=torch.float32, device=dev)
        radii = torch.empty((P,), dtype=torch.int32, device=dev)
        conic = torch.empty((P, 4), dtype=torch.float32, device=dev)
        rgb = torch.empty((P, 3), dtype=torch.float32, device=dev)
        vlist = torch.empty((max(P, 1),), dtype=torch.int32, device=dev) if want_list else None
    # the regulariser sums and the list counter start at zero: one fill for both
    zeros = torch.zeros((3,), dtype=torch.int64, device=dev) if (want_reg or (want_list and vis_count is None)) \
        else None
    reg = zeros[:2].view(torch.float64) if want_reg else None
    vcount = (vis_count if vis_count is not None else zeros[2:].view(torch.int32)[:1]) if want_list else None
    xo = None
    if exchange is not None:
        lo, hi, xrec, xmask, xcnt = exchange
        xo = ExchangeOut(int(lo.numel()), ptr(lo), ptr(hi), ptr(xrec), ptr(xmask), ptr(xcnt))
    counts = torch.empty((max(P, 1),), dtype=torch.int32, device=dev) if want_counts else None
    totals = torch.empty((2,), dtype=torch.int64, device=dev) if want_counts else None
    cl = _tile_mask(compute_locally, H, W) if want_counts else None
    slot_of = torch.empty((max(P, 1),), dtype=torch.int32, device=dev) if (want_slots and want_list) else None
    if P > 0:
        scratch = PRE_SCRATCH.get(dev, _lib.load().blitz_preprocess_scratch_bytes(P)) if two_pass else None
        tok = TIMER.begin("preprocess_fwd")
        _lib.call("blitz_preprocess_forward_raw", P, int(raster.sh_degree), M, ptr(xyz), ptr(scaling_raw),
                  ptr(rotation_raw), ptr(rot_norm), ptr(opacity_raw), ptr(dc), dcs, ptr(rest), rs,
                  float(raster.scale_modifier), ptr(_f32c(raster.viewmatrix)), ptr(_f32c(raster.projmatrix)),
                  ptr(_f32c(raster.campos)), float(raster.tanfovx), float(raster.tanfovy),
                  H, W, ptr(means2D), ptr(depths), ptr(radii),
                  ptr(conic), ptr(rgb), ptr(reg), ptr(vlist), ptr(vcount), ptr(cl), ptr(counts), ptr(totals),
                  ptr(slot_of), ctypes.addressof(xo) if xo is not None else None, ptr(scratch),
                  scratch.numel() if two_pass else 0, _lib.stream_ptr())
        TIMER.end(tok, P=P, fused_count=want_counts, lazy=lambda: {"n_list": vcount} if want_list else {})
    elif want_counts:
        totals.zero_()
    return means2D, depths, radii, conic, rgb, reg, vlist, vcount, counts, totals, slot_of


class ExchangeOut(ctypes.Structure):
    """blitz_exchange_out of include/blitzgs_b200.h."""
    _fields_ = [("n_ranks", ctypes.c_int), ("tile_lo", ctypes.c_void_p), ("tile_hi", ctypes.c_void_p),
                ("records", ctypes.c_void_p), ("dest_mask", ctypes.c_void_p), ("dest_counts", ctypes.c_void_p)]


PACK_SCRATCH = _Scratch(zeroed=True)  # ordered-scan state of the exchange pack; first 4 bytes: status word


def queue_scan_status(device):
    """Queue, on the current stream, copies of the status words of the
    ordered scans of the preprocess and the exchange pack on ``device`` into
    pinned host memory; call check_scan_status(handle) after the stream has
    been synchronised (e.g. by a readback that follows).  No extra sync."""
    bufs = [b for b in (PRE_SCRATCH.peek(device), PACK_SCRATCH.peek(device)) if b is not None]
    host, host_np = _pinned(device, 2, torch.int32, "scan-status")
    host_np[:] = 0
    for i, b in enumerate(bufs):
        host[i:i + 1].copy_(b[:4].view(torch.int32), non_blocking=True)
    return host_np, bufs


def check_scan_status(handle):
    """Raise if a status word read by queue_scan_status shows that an
    ordered scan gave up waiting (and clear the words)."""
    host_np, bufs = handle
    words = [int(x) for x in host_np[:len(bufs)]]
    if any(words):
        for b in bufs:
            b[:4].zero_()
        raise RuntimeError(f"blitzgs_b200: an ordered scan gave up waiting (status words {words})")


def exchange_pack(n_rows, records, dest_mask, dest_offset, send, send_row, row_base):
    """Pack n_rows exchange records into the send buffer (blitz_exchange_pack);
    dest_offset: list of per-rank starting rows.  Each rank's segment keeps
    the rows' order."""
    n_ranks = len(dest_offset)
    offs = (ctypes.c_int64 * n_ranks)(*[int(x) for x in dest_offset])
    lib = _lib.load()
    scratch = PACK_SCRATCH.get(records.device, lib.blitz_exchange_pack_scratch_bytes(int(n_rows), n_ranks))
    _lib.call("blitz_exchange_pack", int(n_rows), n_ranks, ptr(records), ptr(dest_mask), ctypes.addressof(offs),
              ptr(send), ptr(send_row), int(row_base), ptr(scratch), scratch.numel(), _lib.stream_ptr())


def exchange_pack_batch(n_rows, cam_stride, records, dest_mask, dest_offset, row_base, send, send_row):
    """blitz_exchange_pack_batch: camera k's n_rows[k] rows (records /
    dest_mask rows from k*cam_stride) to send, rank r's segment of camera k
    starting at dest_offset[k][r]; send_row gets row_base[k] + j."""
    n_cams = len(n_rows)
    if n_cams == 0:
        return
    n_ranks = len(dest_offset[0])
    nr = (ctypes.c_int64 * n_cams)(*[int(x) for x in n_rows])
    rb = (ctypes.c_int64 * n_cams)(*[int(x) for x in row_base])
    do = (ctypes.c_int64 * (n_cams * n_ranks))(*[int(x) for row in dest_offset for x in row])
    lib = _lib.load()
    scratch = PACK_SCRATCH.get(records.device, lib.blitz_exchange_pack_scratch_bytes(max(int(x) for x in n_rows),
                                                                                     n_ranks))
    _lib.call("blitz_exchange_pack_batch", n_cams, n_ranks, nr, int(cam_stride), ptr(records), ptr(dest_mask), do, rb,
              ptr(send), ptr(send_row), ptr(scratch), scratch.numel(), _lib.stream_ptr())


def _tanfov(rasters):
    n = len(rasters)
    return (ctypes.c_float * (2 * n))(*[float(v) for r in rasters for v in (r.tanfovx, r.tanfovy)])


def preprocess_forward_raw_batch(xyz, scaling_raw, rotation_raw, opacity_raw, sh, rasters, cams, cam_stride, out,
                                 counts, exchange=None):
    """blitz_preprocess_forward_raw_batch over the cameras of ``rasters``.
    ``cams`` = (viewmatrices [n,16], projmatrices [n,16], campos [n,3])
    device tensors; ``out`` = (means2D, depths, radii, conic_opacity, rgb,
    vis_list) with camera k's rows from k*cam_stride; ``counts`` int32
    [n, 1+ranks] zeroed; ``exchange`` = (tile_bounds int32 [n,2,ranks],
    records, dest_mask) or None."""
    _require_cuda(xyz, scaling_raw, rotation_raw, opacity_raw)
    dc, dcs, rest, rs, M, _keep = sh
    P = xyz.shape[0]
    n = len(rasters)
    if n == 0 or P == 0:
        return
    r0 = rasters[0]
    H, W = int(r0.image_height), int(r0.image_width)
    views, projs, campos = cams
    means2D, depths, radii, conic, rgb, vlist = out
    n_ranks = 0 if exchange is None else int(exchange[0].shape[-1])
    tb, rec, mask = exchange if exchange is not None else (None, None, None)
    scratch = PRE_SCRATCH.get(xyz.device, _lib.load().blitz_preprocess_batch_scratch_bytes(n, P))
    tok = TIMER.begin("preprocess_fwd")
    _lib.call("blitz_preprocess_forward_raw_batch", n, P, int(r0.sh_degree), M, ptr(xyz), ptr(scaling_raw),
              ptr(rotation_raw), ptr(opacity_raw), ptr(dc), dcs, ptr(rest), rs, float(r0.scale_modifier), ptr(views),
              ptr(projs), ptr(campos), _tanfov(rasters), H, W, int(cam_stride), ptr(means2D), ptr(depths),
              ptr(radii), ptr(conic), ptr(rgb), ptr(vlist), ptr(counts), n_ranks, ptr(tb), ptr(rec), ptr(mask),
              ptr(scratch), scratch.numel(), _lib.stream_ptr())
    TIMER.end(tok, P=P * n)


def preprocess_backward_raw_batch(radii, means2D, vis_list, counts, cam_stride, xyz, scaling_raw, rotation_raw,
                                  opacity_raw, sh, rasters, cams, upstream, upstream_row0, out):
    """blitz_preprocess_backward_raw_batch: every camera's listed backward
    added into ``out`` = (g_xyz, g_scaling, g_rotation, g_opacity, (g_dc,
    stride), (g_rest, stride))."""
    dc, dcs, rest, rs, M, _keep = sh
    P = xyz.shape[0]
    n = len(rasters)
    if n == 0 or P == 0:
        return
    r0 = rasters[0]
    H, W = int(r0.image_height), int(r0.image_width)
    views, projs, campos = cams
    gx, gs, gq, go, (gdc, gdcs), (grest, grs) = out
    rows0 = (ctypes.c_int64 * n)(*[int(v) for v in upstream_row0])
    tok = TIMER.begin("preprocess_bwd")
    _lib.call("blitz_preprocess_backward_raw_batch", n, P, int(r0.sh_degree), M, ptr(radii), ptr(means2D),
              ptr(vis_list), ptr(counts), int(counts.stride(0)), int(cam_stride), ptr(xyz), ptr(scaling_raw),
              ptr(rotation_raw), ptr(opacity_raw), ptr(dc), dcs, ptr(rest), rs, float(r0.scale_modifier), ptr(views),
              ptr(projs), ptr(campos), _tanfov(rasters), H, W, ptr(upstream), rows0, ptr(gx), ptr(gs), ptr(gq),
              ptr(go), ptr(gdc), gdcs, ptr(grest), grs, _lib.stream_ptr())
    TIMER.end(tok, P=P * n)


def _segments(segs):
    n = len(segs)
    start = (ctypes.c_int64 * max(n, 1))(*[int(a) for a, _ in segs])
    count = (ctypes.c_int64 * max(n, 1))(*[int(c) for _, c in segs])
    return n, start, count


def exchange_unpack(records, segs, reg=None):
    """Rows of one camera = the runs ``segs`` [(start, count), ...] of the
    received [*,12] records, unpacked into (conic [n,4], means2D [n,2],
    rgb [n,3], depths [n], radii int32 [n]); ``reg`` (double [2], zeroed)
    accumulates the min-scale sum and count over rows with radius > 0."""
    n = sum(int(c) for _, c in segs)
    dev = records.device
    conic = torch.empty((n, 4), dtype=torch.float32, device=dev)
    m2 = torch.empty((n, 2), dtype=torch.float32, device=dev)
    rgb = torch.empty((n, 3), dtype=torch.float32, device=dev)
    depth = torch.empty((n,), dtype=torch.float32, device=dev)
    radii = torch.empty((n,), dtype=torch.int32, device=dev)
    k, start, count = _segments(segs)
    _lib.call("blitz_exchange_unpack", k, start, count, ptr(records), ptr(conic), ptr(m2), ptr(rgb), ptr(depth),
              ptr(radii), ptr(reg), _lib.stream_ptr())
    return conic, m2, rgb, depth, radii


def grad_records_pack(rec16, radii, reg_scale, segs, send):
    """Render-backward records of one camera's rows -> 12-float gradient
    records at the send rows of the runs ``segs``."""
    k, start, count = _segments(segs)
    _lib.call("blitz_grad_records_pack", k, start, count, ptr(rec16), ptr(radii), ptr(reg_scale), ptr(send),
              _lib.stream_ptr())


ROWS_UPSTREAM_BY_SLOT = 1  # BLITZ_ROWS_UPSTREAM_BY_SLOT
ROWS_OUTPUT_BY_SLOT = 2    # BLITZ_ROWS_OUTPUT_BY_SLOT


def preprocess_backward_raw(radii, means2D, xyz, scaling_raw, rotation_raw, opacity_raw, sh, raster,
                            g_means2D, g_conic, g_colors, out, rot_norm=None, reg_scale=None, vis_list=None,
                            vis_count=None, accumulate=False, rows=0, g_minscale=None):
    """Gradients w.r.t. the raw parameters into ``out`` = (g_xyz, g_scaling,
    g_rotation, g_opacity, (g_dc, stride), (g_rest, stride)).  With a visible
    list the outputs must be zero-filled (or accumulating), unless ``rows``
    has ROWS_OUTPUT_BY_SLOT: then row j of every output is the j-th listed
    Gaussian's gradient.  ROWS_UPSTREAM_BY_SLOT reads the upstream gradients
    at row j (the compact record)."""
    dc, dcs, rest, rs, M, _keep = sh
    P = xyz.shape[0]
    gx, gs, gq, go, (gdc, gdcs), (grest, grs) = out
    if P > 0:
        tok = TIMER.begin("preprocess_bwd")
        _lib.call("blitz_preprocess_backward_raw", P, int(raster.sh_degree), M, ptr(radii), ptr(means2D),
                  ptr(xyz), ptr(scaling_raw), ptr(rotation_raw), ptr(rot_norm), ptr(opacity_raw), ptr(dc), dcs,
                  ptr(rest), rs, float(raster.scale_modifier), ptr(raster.viewmatrix), ptr(raster.projmatrix),
                  ptr(raster.campos), float(raster.tanfovx), float(raster.tanfovy), int(raster.image_height),
                  int(raster.image_width), ptr(g_means2D), g_means2D.stride(0), ptr(g_conic), g_conic.stride(0),
                  ptr(g_colors), g_colors.stride(0), ptr(reg_scale), ptr(g_minscale),
                  g_minscale.stride(0) if g_minscale is not None else 0, ptr(vis_list), ptr(vis_count), ptr(gx),
                  ptr(gs), ptr(gq), ptr(go), ptr(gdc), gdcs, ptr(grest), grs, int(bool(accumulate)), int(rows),
                  _lib.stream_ptr())
        TIMER.end(tok, P=P, lazy=lambda: {"n_list": vis_count} if vis_list is not None else {})
    return out


@dataclass
class RenderState:
    """What the render backward needs from its forward (caller-owned buffers)."""
    H: int
    W: int
    R: int
    n_vis: int
    point_list: torch.Tensor  # int32 [R]
    ranges: torch.Tensor      # int32 [T,2]
    final_T: torch.Tensor     # f32 [H*W]
    n_contrib: torch.Tensor   # int32 [H*W]
    n_list: int = None        # length of the preprocess's visible list, when read back
    strip_ids: torch.Tensor = None     # int32 [8R]: per warp strip, the Gaussians that contributed
    strip_pos: torch.Tensor = None     # int32 [8R]: their tile-list positions
    strip_counts: torch.Tensor = None  # int32 [8T]


_PINNED = {}


def _pinned(dev, n, dtype, tag=""):
    """Reused pinned host buffer and a numpy view of it (reading a number
    through numpy costs far less than indexing the tensor)."""
    key = (dev.index, n, dtype, tag)
    t = _PINNED.get(key)
    if t is None:
        buf = torch.empty(n, dtype=dtype, pin_memory=True)
        t = _PINNED[key] = (buf, buf.numpy())
    return t


def _tile_mask(compute_locally, H, W):
    if compute_locally is None:
        return None
    gx, gy = grid_dims(H, W)
    cl = compute_locally.contiguous().view(-1)
    if cl.dtype != torch.bool or cl.numel() != gx * gy:
        raise RuntimeError(f"compute_locally must be bool with {gx * gy} tiles")
    return cl


def render_count(means2D, radii, compute_locally, H, W, counts, totals):
    """Per-Gaussian tile counts under ``compute_locally`` into ``counts``
    int32 [P] and the device totals {R, n_vis} into ``totals`` int64 [2]."""
    P = means2D.shape[0]
    cl = _tile_mask(compute_locally, H, W)
    _lib.call("blitz_render_count", P, H, W, ptr(_f32c(means2D)), ptr(radii), ptr(cl), ptr(counts), ptr(totals),
              _lib.stream_ptr())


# per (device, tile count): capacities (instances, visible Gaussians) of the
# render buffers, 25% above the largest totals seen
_RENDER_CAPS = {}


def render_caps_known(dev, H, W):
    """Whether render_forward would issue this size's binning before its
    totals readback (buffer capacities are known from an earlier view)."""
    gx, gy = grid_dims(H, W)
    return (dev.index, gx * gy) in _RENDER_CAPS


def render_forward(means2D, depths, radii, conic_opacity, rgb, bg, compute_locally, H, W, counts=None, totals=None,
                   vis_count=None, strip_lists=True, totals_host=None, caps_update=False):
    """Binning + blending of one camera.  Returns (color, n_render, n_consider,
    n_contrib_tile, out_observe, state).  ``counts``/``totals`` from
    ``preprocess_forward_raw(want_counts=True)`` skip the count pass;
    ``vis_count`` is read back with the totals (state.n_list).
    ``strip_lists`` records, per 8x4-pixel warp strip, the Gaussians that
    contributed to it (2 x 32 bytes per tile instance of device memory), so
    the backward replays only those.  ``totals_host`` = (R, n_vis) already
    read back by the caller (with ``counts``): no readback here;
    ``caps_update`` then still records them for later views' capacities.
    Without ``totals_host``, once a view of this size has been rendered, the
    binning and blend are issued with capacities before the totals are
    read back (see blitz_render_bin)."""
    _require_cuda(means2D, depths, radii, conic_opacity, rgb, bg)
    means2D, depths, conic_opacity, rgb, bg = map(_f32c, (means2D, depths, conic_opacity, rgb, bg))
    radii = radii.contiguous()
    if radii.dtype != torch.int32:
        raise RuntimeError("radii must be int32")
    P = means2D.shape[0]
    dev = means2D.device
    gx, gy = grid_dims(H, W)
    T = gx * gy
    cl = _tile_mask(compute_locally, H, W)
    st = _lib.stream_ptr()
    if counts is None:
        counts = torch.empty((max(P, 1),), dtype=torch.int32, device=dev)
        totals = torch.empty((2,), dtype=torch.int64, device=dev)
        tok = TIMER.begin("bin_count")
        _lib.call("blitz_render_count", P, H, W, ptr(means2D), ptr(radii), ptr(cl), ptr(counts), ptr(totals), st)
        TIMER.end(tok, P=P)
    # Everything whose size does not depend on the totals is allocated (and
    # out_observe zeroed) before the binning is issued.
    ranges = torch.empty((T, 2), dtype=torch.int32, device=dev)
    final_T = torch.empty((H * W,), dtype=torch.float32, device=dev)
    n_contrib = torch.empty((H * W,), dtype=torch.int32, device=dev)
    color = torch.empty((3, H, W), dtype=torch.float32, device=dev)
    n_render = torch.empty((T,), dtype=torch.int32, device=dev)
    n_consider = torch.empty((T,), dtype=torch.int32, device=dev)
    n_contrib_tile = torch.empty((T,), dtype=torch.int32, device=dev)
    out_observe = torch.zeros((P,), dtype=torch.int32, device=dev)
    strip_counts = torch.empty((T * 8,), dtype=torch.int32, device=dev) if strip_lists else None
    def read_totals():
        host, host_np = _pinned(dev, 2, torch.int64)
        host_n, host_n_np = _pinned(dev, 1, torch.int32) if vis_count is not None else (None, None)
        pre = PRE_SCRATCH.peek(dev)
        host_s = _pinned(dev, 1, torch.int32, "status")[0] if pre is not None else None
        _lib.call("blitz_read_totals", ptr(totals), ptr(vis_count), ptr(pre), host.data_ptr(),
                  host_n.data_ptr() if host_n is not None else None,
                  host_s.data_ptr() if host_s is not None else None, st)
        return int(host_np[0]), int(host_np[1]), (int(host_n_np[0]) if vis_count is not None else None)

    def issue(R, n_vis):
        """Binning + blend with buffers for up to R instances and n_vis
        visible Gaussians (the kernels read the exact totals on the device)."""
        point_list = torch.empty((max(R, 1),), dtype=torch.int32, device=dev)
        strip_ids = torch.empty((8 * max(R, 1),), dtype=torch.int32, device=dev) if strip_lists else None
        strip_pos = torch.empty((8 * max(R, 1),), dtype=torch.int32, device=dev) if strip_lists else None
        scratch = SCRATCH.get(dev, _lib.load().blitz_render_scratch_bytes(P, n_vis, R, H, W))
        tok = TIMER.begin("binning")
        _lib.call("blitz_render_bin", P, n_vis, R, H, W, ptr(means2D), ptr(depths), ptr(radii), ptr(cl), ptr(counts),
                  ptr(scratch), scratch.numel(), ptr(point_list), ptr(ranges), st)
        # R / n_vis are the buffer capacities; "totals" (device {R, n_vis}) the view's own
        TIMER.end(tok, P=P, R=R, n_vis=n_vis,
                  lazy=(lambda: {"totals": totals.reshape(-1)[:2].clone()}) if totals is not None else None)
        tok = TIMER.begin("blend_fwd")
        _lib.call("blitz_render_blend", P, H, W, ptr(means2D), ptr(conic_opacity), ptr(rgb), ptr(bg), ptr(cl),
                  ptr(point_list), ptr(ranges), ptr(final_T), ptr(n_contrib), ptr(color), ptr(n_render),
                  ptr(n_consider), ptr(n_contrib_tile), ptr(out_observe), ptr(strip_ids), ptr(strip_pos),
                  ptr(strip_counts), st)
        TIMER.end(tok, P=P, R=R, n_vis=n_vis, H=H, W=W,
                  lazy=lambda: {"pairs": (n_consider.sum(dtype=torch.int64), n_contrib_tile.sum(dtype=torch.int64))})
        return point_list, strip_ids, strip_pos

    key = (dev.index, T)
    caps = _RENDER_CAPS.get(key) if totals_host is None else None
    if totals_host is not None:
        R, n_vis = int(totals_host[0]), int(totals_host[1])
        n_list = None
        point_list, strip_ids, strip_pos = issue(R, n_vis)
    elif caps is not None:
        # Issue the binning and blend with buffers sized from earlier views,
        # then read the totals: the host waits while the GPU already runs
        # them instead of the GPU waiting for the host.  A view that needs
        # more is binned and blended again with exact sizes (nothing
        # downstream has read the outputs yet).
        R_cap, V_cap = caps[0], min(caps[1], P)
        # the totals (and the scan status words) are copied before the
        # binning in stream order; the host waits for that copy only
        host, host_np = _pinned(dev, 2, torch.int64, "spec")
        host.copy_(totals.view(-1)[:2], non_blocking=True)
        host_n, host_n_np = _pinned(dev, 1, torch.int32, "spec") if vis_count is not None else (None, None)
        if vis_count is not None:
            host_n.copy_(vis_count.view(-1)[:1], non_blocking=True)
        status = queue_scan_status(dev)
        copied = torch.cuda.Event()
        copied.record()
        point_list, strip_ids, strip_pos = issue(R_cap, V_cap)
        copied.synchronize()
        check_scan_status(status)
        R, n_vis = int(host_np[0]), int(host_np[1])
        n_list = int(host_n_np[0]) if vis_count is not None else None
        if R > R_cap or n_vis > V_cap:
            out_observe.zero_()
            point_list, strip_ids, strip_pos = issue(R, n_vis)
    else:
        R, n_vis, n_list = read_totals()
        point_list, strip_ids, strip_pos = issue(R, n_vis)
    if totals_host is None or caps_update:
        old = _RENDER_CAPS.get(key, (0, 0))
        _RENDER_CAPS[key] = (max(old[0], (R * 5 + 3) // 4), max(old[1], (n_vis * 5 + 3) // 4))
    state = RenderState(H, W, R, n_vis, point_list, ranges, final_T, n_contrib, n_list, strip_ids, strip_pos,
                        strip_counts)
    return color, n_render, n_consider, n_contrib_tile, out_observe, state


def rasterize_forward(means2D, depths, radii, rects, conic_opacity, rgb, bg, H, W, *, max_count=False,
                      simp=False, strip_lists=True, blend=True):
    """Binning and blending of the full (non-distributed) rasterizer
    (_C.rasterize_gaussians / _simp): each Gaussian's float rectangle
    ``rects`` restricted to the tiles that pass the exact tile test.
    Returns (color, state, stats) with stats a dict of the requested
    per-Gaussian statistics: "max_count" float [P] (``max_count`` or
    ``simp``), "accum_weights" float [P] and "accum_count" int32 [P]
    (``simp``).  ``blend=False`` stops after the binning (color None; the
    state holds the lists only)."""
    _require_cuda(means2D, depths, radii, rects, conic_opacity, rgb, bg)
    means2D, depths, rects, conic_opacity, rgb, bg = map(_f32c, (means2D, depths, rects, conic_opacity, rgb, bg))
    radii = radii.contiguous()
    if radii.dtype != torch.int32:
        raise RuntimeError("radii must be int32")
    P = means2D.shape[0]
    dev = means2D.device
    gx, gy = grid_dims(H, W)
    T = gx * gy
    st = _lib.stream_ptr()
    counts = torch.empty((max(P, 1),), dtype=torch.int32, device=dev)
    totals = torch.empty((2,), dtype=torch.int64, device=dev)
    tok = TIMER.begin("bin_count")
    _lib.call("blitz_rasterize_count", P, H, W, ptr(means2D), ptr(radii), ptr(rects), ptr(conic_opacity), ptr(counts),
              ptr(totals), st)
    TIMER.end(tok, P=P)
    ranges = torch.empty((T, 2), dtype=torch.int32, device=dev)
    final_T = torch.empty((H * W,), dtype=torch.float32, device=dev)
    n_contrib = torch.empty((H * W,), dtype=torch.int32, device=dev)
    color = torch.empty((3, H, W), dtype=torch.float32, device=dev)
    stats = {}
    if max_count or simp:
        stats["max_count"] = torch.zeros((P,), dtype=torch.float32, device=dev)
    if simp:
        stats["accum_weights"] = torch.zeros((P,), dtype=torch.float32, device=dev)
        stats["accum_count"] = torch.zeros((P,), dtype=torch.int32, device=dev)
    host, host_np = _pinned(dev, 2, torch.int64)
    _lib.call("blitz_read_totals", ptr(totals), None, None, host.data_ptr(), None, None, st)
    R, n_vis = int(host_np[0]), int(host_np[1])
    point_list = torch.empty((max(R, 1),), dtype=torch.int32, device=dev)
    scratch = SCRATCH.get(dev, _lib.load().blitz_render_scratch_bytes(P, n_vis, R, H, W))
    tok = TIMER.begin("binning")
    _lib.call("blitz_rasterize_bin", P, n_vis, R, H, W, ptr(means2D), ptr(depths), ptr(radii), ptr(rects),
              ptr(conic_opacity), ptr(counts), ptr(scratch), scratch.numel(), ptr(point_list), ptr(ranges), st)
    TIMER.end(tok, P=P, R=R, n_vis=n_vis)
    if not blend:
        return None, RenderState(H, W, R, n_vis, point_list, ranges, final_T, n_contrib), stats
    strip = strip_lists and not stats
    strip_ids = torch.empty((8 * max(R, 1),), dtype=torch.int32, device=dev) if strip else None
    strip_pos = torch.empty((8 * max(R, 1),), dtype=torch.int32, device=dev) if strip else None
    strip_counts = torch.empty((T * 8,), dtype=torch.int32, device=dev) if strip else None
    tok = TIMER.begin("blend_fwd")
    if stats:
        _lib.call("blitz_rasterize_blend", P, H, W, ptr(means2D), ptr(conic_opacity), ptr(rgb), ptr(bg),
                  ptr(point_list), ptr(ranges), ptr(final_T), ptr(n_contrib), ptr(color), ptr(stats.get("max_count")),
                  ptr(stats.get("accum_weights")), ptr(stats.get("accum_count")), st)
    else:
        tile_i = torch.empty((3, T), dtype=torch.int32, device=dev)
        observe = torch.zeros((max(P, 1),), dtype=torch.int32, device=dev)
        _lib.call("blitz_render_blend", P, H, W, ptr(means2D), ptr(conic_opacity), ptr(rgb), ptr(bg), None,
                  ptr(point_list), ptr(ranges), ptr(final_T), ptr(n_contrib), ptr(color), ptr(tile_i[0]),
                  ptr(tile_i[1]), ptr(tile_i[2]), ptr(observe), ptr(strip_ids), ptr(strip_pos), ptr(strip_counts), st)
    TIMER.end(tok, P=P, R=R, n_vis=n_vis, H=H, W=W)
    state = RenderState(H, W, R, n_vis, point_list, ranges, final_T, n_contrib, None, strip_ids, strip_pos,
                        strip_counts)
    return color, state, stats


def rasterize_depth(means2D, conic_opacity, rgb, bg, state, means3D, scales, rotations, raster):
    """rasterize_gaussians_depth's blend over the lists of
    :func:`rasterize_forward`: (color [3,H,W], out_pts [3,H,W], depth
    [1,H,W], accum_alpha [1,H,W], gidx int32 [1,H,W], discriminants [1,H,W])."""
    means2D, conic_opacity, rgb, bg, means3D, scales, rotations = map(
        _f32c, (means2D, conic_opacity, rgb, bg, means3D, scales, rotations))
    H, W = state.H, state.W
    dev = means2D.device
    f = lambda c=1: torch.empty((c, H, W), dtype=torch.float32, device=dev)  # noqa: E731
    color, pts, depth, alpha, disc = f(3), f(3), f(), f(), f()
    gidx = torch.empty((1, H, W), dtype=torch.int32, device=dev)
    _lib.call("blitz_rasterize_depth", means2D.shape[0], H, W, ptr(means2D), ptr(conic_opacity), ptr(rgb), ptr(bg),
              ptr(state.point_list), ptr(state.ranges), ptr(means3D), ptr(scales), ptr(rotations),
              ptr(_f32c(raster.projmatrix)), ptr(_f32c(raster.campos)), ptr(color), ptr(pts), ptr(depth), ptr(alpha),
              ptr(gidx), ptr(disc), _lib.stream_ptr())
    return color, pts, depth, alpha, gidx, disc


def mark_visible(means3D, viewmatrix, projmatrix):
    """bool [P]: view depth > 0.2 (the frustum test of markVisible)."""
    _require_cuda(means3D)
    means3D = _f32c(means3D)
    P = means3D.shape[0]
    present = torch.zeros((P,), dtype=torch.bool, device=means3D.device)
    _lib.call("blitz_mark_visible", P, ptr(means3D), ptr(_f32c(viewmatrix)), ptr(_f32c(projmatrix)), ptr(present),
              _lib.stream_ptr())
    return present


def render_backward(state, means2D, conic_opacity, rgb, bg, compute_locally, dL_dpix, grad_accum=None,
                    record_rows=None, n_rows=None):
    """Returns the per-Gaussian gradient record (see include/blitzgs_b200.h):
    [P,16], or [n_rows,16] with Gaussian i at row record_rows[i]."""
    means2D, conic_opacity, rgb, bg = map(_f32c, (means2D, conic_opacity, rgb, bg))
    dL_dpix = _f32c(dL_dpix)
    P = means2D.shape[0]
    if grad_accum is None:
        rows = P if record_rows is None else max(int(n_rows), 1)
        grad_accum = torch.zeros((rows, 16), dtype=torch.float32, device=means2D.device)
    cl = compute_locally.contiguous().view(-1) if compute_locally is not None else None
    tok = TIMER.begin("blend_bwd")
    _lib.call("blitz_render_backward", P, state.H, state.W, ptr(state.point_list), ptr(state.ranges),
              ptr(state.final_T), ptr(state.n_contrib), ptr(means2D), ptr(conic_opacity), ptr(rgb), ptr(bg),
              ptr(cl), ptr(dL_dpix), ptr(record_rows), ptr(state.strip_ids), ptr(state.strip_pos),
              ptr(state.strip_counts), ptr(grad_accum), _lib.stream_ptr())
    TIMER.end(tok, P=P, R=state.R, lazy=lambda: {"pairs": (state.n_contrib.sum(dtype=torch.int64),)})
    return grad_accum


_WINDOW = None


def ssim_window():
    """The reference's normalised 11-tap Gaussian (sigma 1.5) as float32 values
    (utils/loss_utils.py:21-28: exp() in double, rounded to float32, divided
    by its float32 sum).  Returns (ctypes float[11], torch tensor)."""
    global _WINDOW
    if _WINDOW is None:
        g = torch.tensor([math.exp(-((x - 5) ** 2) / float(2 * 1.5 ** 2)) for x in range(11)],
                         dtype=torch.float32)
        g = g / g.sum()
        _WINDOW = ((ctypes.c_float * 11)(*g.tolist()), g)
    return _WINDOW


def loss_forward(img, gt):
    """Fused L1+SSIM sums over a band.  Returns (sums double[2], partials)."""
    _require_cuda(img, gt)
    img = _f32c(img)
    C, Hb, W = img.shape
    gt = gt.contiguous()
    win, _ = ssim_window()
    partials = torch.empty((C, Hb, W, 3), dtype=torch.float32, device=img.device)
    sums = torch.zeros((2,), dtype=torch.float64, device=img.device)
    gt_u8 = gt if gt.dtype == torch.uint8 else None
    gt_f = _f32c(gt) if gt.dtype != torch.uint8 else None
    tok = TIMER.begin("loss_fwd")
    _lib.call("blitz_loss_forward", C, Hb, W, ptr(img), ptr(gt_u8), ptr(gt_f), win, ptr(partials),
              ptr(sums), _lib.stream_ptr())
    TIMER.end(tok, pixels=C * Hb * W, gt_bytes=1 if gt_u8 is not None else 4)
    return sums, partials


def loss_backward(img, gt, partials, scale):
    img = _f32c(img)
    C, Hb, W = img.shape
    gt = gt.contiguous()
    win, _ = ssim_window()
    out = torch.empty_like(img)
    gt_u8 = gt if gt.dtype == torch.uint8 else None
    gt_f = _f32c(gt) if gt.dtype != torch.uint8 else None
    tok = TIMER.begin("loss_bwd")
    _lib.call("blitz_loss_backward", C, Hb, W, ptr(img), ptr(gt_u8), ptr(gt_f), win, ptr(partials),
              ptr(_f32c(scale)), ptr(out), _lib.stream_ptr())
    TIMER.end(tok, pixels=C * Hb * W, gt_bytes=1 if gt_u8 is not None else 4)
    return out


def loss_combine(sums, reg, lambda_dssim, n3, reg_weight):
    """The per-camera loss on the device: float32 [5] {loss, L1, SSIM, reg,
    cnt} with loss = (1-l) L1/N3 + l (1 - SSIM/N3) + w reg / max(cnt, 1)
    (reg = None: no regulariser)."""
    out = torch.empty((5,), dtype=torch.float32, device=sums.device)
    _lib.call("blitz_loss_combine", ptr(sums), ptr(reg), 1.0 - lambda_dssim, lambda_dssim, float(n3),
              float(reg_weight), ptr(out), _lib.stream_ptr())
    return out


def loss_combine_backward(g_loss, g_l1, g_ss, fwd_out, lambda_dssim, n3, reg_weight):
    """float32 [3] {dLoss/d(sum L1), dLoss/d(sum SSIM), dLoss/d reg} from the
    upstream gradients of loss, L1 and SSIM (None = 0)."""
    scales = torch.empty((3,), dtype=torch.float32, device=fwd_out.device)
    g = [None if t is None else _f32c(t) for t in (g_loss, g_l1, g_ss)]
    _lib.call("blitz_loss_combine_backward", ptr(g[0]), ptr(g[1]), ptr(g[2]), ptr(fwd_out), 1.0 - lambda_dssim,
              lambda_dssim, float(n3), float(reg_weight), ptr(scales), _lib.stream_ptr())
    return scales


def zero_fill_async(tensors):
    """Zero ``tensors`` on the library's side stream after the work already
    queued on the current stream; ``zero_fill_wait()`` orders the current
    stream after the fill.  The tensors must not be touched (or freed) by
    the current stream before that wait."""
    n = len(tensors)
    ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tensors])
    sizes = (ctypes.c_size_t * n)(*[t.numel() * t.element_size() for t in tensors])
    _lib.call("blitz_zero_fill_async", n, ptrs, sizes, _lib.stream_ptr())


def zero_rows(tensors, rows, n_rows):
    """Zero rows ``rows[:n_rows]`` (device uint32/int32 indices) of each
    contiguous tensor in ``tensors`` (at most 8, rows along dim 0), in one
    launch on the current stream."""
    n = len(tensors)
    if n == 0 or n_rows <= 0:
        return
    for t in tensors:
        if not t.is_contiguous() or t.dtype != torch.float32:
            raise RuntimeError("zero_rows: contiguous float32 tensors only")
    ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tensors])
    sizes = (ctypes.c_size_t * n)(*[t[0].numel() * 4 for t in tensors])
    _lib.call("blitz_zero_rows", n, ptrs, sizes, ptr(rows), int(n_rows), _lib.stream_ptr())


def zero_fill_wait():
    _lib.call("blitz_zero_fill_wait", _lib.stream_ptr())


def fp32_peak_tflops(seconds=0.3):
    """Measured FP32 FMA throughput of this GPU (TFLOP/s), timed with CUDA events."""
    dev = torch.device("cuda", torch.cuda.current_device())
    sink = torch.zeros(1, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 8
    st = _lib.stream_ptr()
    _lib.call("blitz_fp32_probe", blocks, 1000, ptr(sink), st)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    iters = 20000
    a.record()
    _lib.call("blitz_fp32_probe", blocks, iters, ptr(sink), st)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b)
    if ms < seconds * 1e3:
        iters = int(iters * seconds * 1e3 / max(ms, 1e-3))
        a.record()
        _lib.call("blitz_fp32_probe", blocks, iters, ptr(sink), st)
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b)
    return blocks * 256 * iters * 16 / (ms * 1e-3) / 1e12


def local2j_ids_bool(H, W, mp_rank, mp_world_size, means2D, radii, dist_global_strategy,
                     avoid_pixel_all2all=False):
    _require_cuda(means2D, radii, dist_global_strategy)
    P = means2D.shape[0]
    out = torch.empty((P, mp_world_size), dtype=torch.bool, device=means2D.device)
    _lib.call("blitz_get_local2j_ids_bool", int(H), int(W), int(mp_rank), int(mp_world_size), P,
              ptr(_f32c(means2D)), ptr(radii.contiguous()), ptr(dist_global_strategy.to(torch.int32).contiguous()),
              int(bool(avoid_pixel_all2all)), ptr(out), _lib.stream_ptr())
    return out


def local2j_ids_bool_adjust_mode6(H, W, mp_rank, mp_world_size, means2D, radii, rectangles,
                                  avoid_pixel_all2all=False):
    """Routing mask bool [P, mp_world_size] against per-rank tile rectangles
    int32 [mp_world_size, 4] = (row begin, row end, column begin, column end)."""
    _require_cuda(means2D, radii, rectangles)
    P = means2D.shape[0]
    out = torch.empty((P, mp_world_size), dtype=torch.bool, device=means2D.device)
    _lib.call("blitz_get_local2j_ids_bool_adjust_mode6", int(H), int(W), int(mp_rank), int(mp_world_size), P,
              ptr(_f32c(means2D)), ptr(radii.contiguous()), ptr(rectangles.to(torch.int32).contiguous()),
              int(bool(avoid_pixel_all2all)), ptr(out), _lib.stream_ptr())
    return out


def adam_update(param, grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps, N, M):
    """In-place sparse Adam step of param [N*M] for the Gaussians with
    visible[g] (blitz_adam_update; the reference's _C.adamUpdate)."""
    for t in (param, grad, exp_avg, exp_avg_sq):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError("adam_update needs contiguous float32 tensors")
    vis = visible.contiguous()
    if vis.dtype != torch.bool:
        vis = vis.to(torch.bool)
    tok = TIMER.begin("adam")
    _lib.call("blitz_adam_update", ptr(param), ptr(grad), ptr(exp_avg), ptr(exp_avg_sq), ptr(vis), float(lr),
              float(b1), float(b2), float(eps), int(N), int(M), _lib.stream_ptr())
    TIMER.end(tok, N=int(N), M=int(M))


def adam_update_rows(param, grad_rows, exp_avg, exp_avg_sq, rows, lr, b1, b2, eps, N, M, grad_scale=1.0):
    """In-place sparse Adam step of the Gaussians rows (int64 [n], distinct)
    whose gradients are the rows of grad_rows [n, M] (blitz_adam_update_rows),
    each gradient element first multiplied by grad_scale (float32)."""
    for t in (param, exp_avg, exp_avg_sq):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError("adam_update_rows needs contiguous float32 tensors")
    grad_rows = _f32c(grad_rows)
    rows = rows.to(torch.int64).contiguous()
    n = rows.numel()
    tok = TIMER.begin("adam")
    _lib.call("blitz_adam_update_rows", ptr(param), ptr(grad_rows), ptr(exp_avg), ptr(exp_avg_sq), ptr(rows), n,
              float(grad_scale), float(lr), float(b1), float(b2), float(eps), int(N), int(M), _lib.stream_ptr())
    TIMER.end(tok, N=int(N), M=int(M), n_rows=n)
