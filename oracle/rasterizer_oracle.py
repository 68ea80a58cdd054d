"""CPU oracle for the BlitzGS splatting training path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's cpu_baseline / reference-fallback leg.  The
product (blitzgs_b200) never imports this module.

A float32 PyTorch / numpy restatement of the reference algorithm, stage by
stage, each function citing the reference lines it follows:

  preprocess_forward   submodule/diff-gaussian-rasterization_f/cuda_rasterizer/
                       forward.cu:28-284, auxiliary.h:43-185
  preprocess_backward  backward.cu:18-400, as autograd of a differentiable
                       restatement with the reference's gradient conventions
  binning              submodule/diff-gaussian-rasterization_r/cuda_rasterizer/
                       rasterizer_impl.cu:74-138, 258-282, 602-665
  render_forward       r/cuda_rasterizer/forward.cu:263-413 (+ stats
                       rasterizer_impl.cu:213-256, 696-717)
  render_backward      r/cuda_rasterizer/backward.cu:324-530, written out in
                       closed form per tile
  full_binning         the full rasterizer's binning with the exact tile test,
                       f/cuda_rasterizer/rasterizer_impl.cu:52-97, 119-191
  render_stats         flag_max_count / render_simp statistics,
                       f/cuda_rasterizer/forward.cu:402-440, 566-590
  mark_visible         f/cuda_rasterizer/rasterizer_impl.cu:100-114
  loss                 utils/loss_utils.py:31-37, 83-124 and
                       gaussian_renderer/loss_distribution.py:220-263, 307-309

CPU float32 arithmetic does not contract a*b+c into FMA and CPU expf/logf
may differ from CUDA's in the last ulp, so integer outputs that hang on a
float compare (radii, n_contrib) can differ from the GPU's on rare boundary
cases; tests state the tolerance they allow.  Bit-exact parity against the
reference itself is checked with the golden vectors in tests/golden/, which
were produced by running the reference CUDA rasterizer.
"""
import math

import numpy as np
import torch
import torch.nn.functional as F

TILE = 16
SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = (1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792, 0.5462742152960396)
SH_C3 = (-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
         -0.4570457994644658, 1.445305721320277, -0.5900435899266435)

f32 = torch.float32


def _c(x):
    return torch.tensor(x, dtype=f32)


# ---------------------------------------------------------------------------
# Preprocess
# ---------------------------------------------------------------------------

def _xform3(p, M):
    """p [N,3]; M [16] column-major 4x4 (reference transformPoint4x3)."""
    return torch.stack([M[0] * p[:, 0] + M[4] * p[:, 1] + M[8] * p[:, 2] + M[12],
                        M[1] * p[:, 0] + M[5] * p[:, 1] + M[9] * p[:, 2] + M[13],
                        M[2] * p[:, 0] + M[6] * p[:, 1] + M[10] * p[:, 2] + M[14]], 1)


def _xform4(p, M):
    return torch.stack([M[0] * p[:, 0] + M[4] * p[:, 1] + M[8] * p[:, 2] + M[12],
                        M[1] * p[:, 0] + M[5] * p[:, 1] + M[9] * p[:, 2] + M[13],
                        M[2] * p[:, 0] + M[6] * p[:, 1] + M[10] * p[:, 2] + M[14],
                        M[3] * p[:, 0] + M[7] * p[:, 1] + M[11] * p[:, 2] + M[15]], 1)


def _rotmat(q):
    """Math-convention R (rows) of the reference's glm matrix (forward.cu:138-146)."""
    r, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    # glm::mat3(a..i) lists columns; math R[row][col] = glm[col][row]
    c0 = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - r * z), 2 * (x * z + r * y)], 1)
    c1 = torch.stack([2 * (x * y + r * z), 1 - 2 * (x * x + z * z), 2 * (y * z - r * x)], 1)
    c2 = torch.stack([2 * (x * z - r * y), 2 * (y * z + r * x), 1 - 2 * (x * x + y * y)], 1)
    return torch.stack([c0, c1, c2], 2)  # [N, row, col]; column c = glm column c


def _mm3(A, B):
    """Batched 3x3 product [N,3,3] @ [N,3,3] (either may be a single [3,3])
    summed left to right in float32 elementwise operations.  A BLAS call would
    round differently on different host CPUs (vector width, FMA), which made
    the oracle's radii -- and so whole splats -- depend on the machine."""
    rows = []
    for r in range(3):
        cols = []
        for c in range(3):
            cols.append(A[..., r, 0] * B[..., 0, c] + A[..., r, 1] * B[..., 1, c] + A[..., r, 2] * B[..., 2, c])
        rows.append(torch.stack(cols, -1))
    return torch.stack(rows, -2)


def cov3d(scales, q, mod=1.0):
    """Sigma = (S R)^T (S R) in glm semantics -> math Sigma = M_m^T M_m with
    M_m = S_m R_m ... returned as the 6-vector (s00,s01,s02,s11,s12,s22)."""
    R = _rotmat(q)
    S = torch.diag_embed(mod * scales)
    Mm = _mm3(S, R)  # glm M = S*R  <->  math S_m @ R_m
    Sig = _mm3(Mm.transpose(1, 2), Mm)
    return torch.stack([Sig[:, 0, 0], Sig[:, 0, 1], Sig[:, 0, 2], Sig[:, 1, 1], Sig[:, 1, 2], Sig[:, 2, 2]], 1)


def _cov2d(mean, V, fx, fy, tanx, tany, c6, clamp_detach=False):
    t = _xform3(mean, V)
    limx, limy = 1.3 * tanx, 1.3 * tany
    txtz, tytz = t[:, 0] / t[:, 2], t[:, 1] / t[:, 2]
    tz = t[:, 2]
    cx = torch.clamp(txtz, -limx, limx) * tz
    cy = torch.clamp(tytz, -limy, limy) * tz
    if clamp_detach:
        # the reference backward treats the clamped x/y as constants and
        # passes the unclamped ones through with unit derivative
        inx = (txtz >= -limx) & (txtz <= limx)
        iny = (tytz >= -limy) & (tytz <= limy)
        tx = torch.where(inx, t[:, 0] + (cx - t[:, 0]).detach(), cx.detach())
        ty = torch.where(iny, t[:, 1] + (cy - t[:, 1]).detach(), cy.detach())
    else:
        tx, ty = cx, cy
    z0 = torch.zeros_like(tz)
    Jm = torch.stack([torch.stack([fx / tz, z0, z0], 1),
                      torch.stack([z0, fy / tz, z0], 1),
                      torch.stack([-(fx * tx) / (tz * tz), -(fy * ty) / (tz * tz), z0], 1)], 1)
    Wm = torch.stack([torch.stack([V[0], V[1], V[2]]), torch.stack([V[4], V[5], V[6]]),
                      torch.stack([V[8], V[9], V[10]])], 0)
    Tm = _mm3(Wm.unsqueeze(0), Jm)
    Vrk = torch.stack([torch.stack([c6[:, 0], c6[:, 1], c6[:, 2]], 1),
                       torch.stack([c6[:, 1], c6[:, 3], c6[:, 4]], 1),
                       torch.stack([c6[:, 2], c6[:, 4], c6[:, 5]], 1)], 1)
    cov = _mm3(_mm3(Tm.transpose(1, 2), Vrk), Tm)
    return cov[:, 0, 0] + 0.3, cov[:, 1, 0], cov[:, 1, 1] + 0.3


def sh_rgb(D, means, campos, shs):
    """computeColorFromSH (forward.cu:28-80); shs [N,K,3] with DC first."""
    d = means - campos.view(1, 3)
    d = d / torch.sqrt((d * d).sum(1, keepdim=True))
    x, y, z = d[:, 0:1], d[:, 1:2], d[:, 2:3]
    sh = shs
    res = SH_C0 * sh[:, 0]
    if D > 0:
        res = res - SH_C1 * y * sh[:, 1] + SH_C1 * z * sh[:, 2] - SH_C1 * x * sh[:, 3]
        if D > 1:
            xx, yy, zz, xy, yz, xz = x * x, y * y, z * z, x * y, y * z, x * z
            res = (res + SH_C2[0] * xy * sh[:, 4] + SH_C2[1] * yz * sh[:, 5]
                   + SH_C2[2] * (2.0 * zz - xx - yy) * sh[:, 6] + SH_C2[3] * xz * sh[:, 7]
                   + SH_C2[4] * (xx - yy) * sh[:, 8])
            if D > 2:
                res = (res + SH_C3[0] * y * (3.0 * xx - yy) * sh[:, 9] + SH_C3[1] * xy * z * sh[:, 10]
                       + SH_C3[2] * y * (4.0 * zz - xx - yy) * sh[:, 11]
                       + SH_C3[3] * z * (2.0 * zz - 3.0 * xx - 3.0 * yy) * sh[:, 12]
                       + SH_C3[4] * x * (4.0 * zz - xx - yy) * sh[:, 13]
                       + SH_C3[5] * z * (xx - yy) * sh[:, 14] + SH_C3[6] * x * (xx - 3.0 * yy) * sh[:, 15])
    res = res + 0.5
    return res


def ndc2pix(v, S):
    return (((v.double() + 1.0) * S - 1.0) * 0.5).to(f32)


def preprocess_forward(means3D, scales, rotations, shs, opacities, viewmatrix, projmatrix, campos,
                       tanfovx, tanfovy, H, W, D, scale_modifier=1.0):
    """Returns dict(means2D, depths, radii, conic_opacity, rgb, clamped) with
    zeros for culled Gaussians (reference preprocessCUDA forward.cu:164-284)."""
    with torch.no_grad():
        V = viewmatrix.reshape(-1).to(f32)
        Pm = projmatrix.reshape(-1).to(f32)
        P = means3D.shape[0]
        op = opacities.reshape(-1)
        fx = np.float32(W) / (np.float32(2.0) * np.float32(tanfovx))
        fy = np.float32(H) / (np.float32(2.0) * np.float32(tanfovy))
        fx, fy = float(fx), float(fy)
        pv = _xform3(means3D, V)
        ok = pv[:, 2] > 0.2
        ph = _xform4(means3D, Pm)
        pw = 1.0 / (ph[:, 3] + 1e-7)
        pp = ph[:, :3] * pw[:, None]
        c6 = cov3d(scales, rotations, scale_modifier)
        a, b, c = _cov2d(means3D, V, fx, fy, float(np.float32(tanfovx)), float(np.float32(tanfovy)), c6)
        det = a * c - b * b
        ok &= det != 0
        dinv = 1.0 / det
        conic = torch.stack([c * dinv, -b * dinv, a * dinv], 1)
        opt = torch.log(op / _c(1.0 / 255.0))
        ext = torch.sqrt(2.0 * opt).double()
        ext = torch.where(torch.isnan(ext), torch.full_like(ext, 3.33), torch.clamp(ext, max=3.33)).to(f32)
        mid = 0.5 * (a + c)
        lam = mid + torch.sqrt(torch.clamp(mid * mid - det, min=0.01))
        rad = ext * torch.sqrt(lam)
        ok &= rad > 0
        px, py = ndc2pix(pp[:, 0], W), ndc2pix(pp[:, 1], H)
        ex = torch.minimum(ext * torch.sqrt(a), rad)
        ey = torch.minimum(ext * torch.sqrt(c), rad)
        gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
        x0 = torch.clamp(torch.floor((px - ex) / TILE), 0, gx)
        y0 = torch.clamp(torch.floor((py - ey) / TILE), 0, gy)
        x1 = torch.clamp(torch.ceil((px + ex) / TILE), 0, gx)
        y1 = torch.clamp(torch.ceil((py + ey) / TILE), 0, gy)
        ok &= ((x1 - x0) * (y1 - y0)) != 0
        ok &= ~torch.isnan(rad)
        rgb_raw = sh_rgb(D, means3D, campos.reshape(-1).to(f32), shs)
        clamped = rgb_raw < 0
        rgb = torch.clamp(rgb_raw, min=0.0)
        z = torch.zeros
        out = dict(
            means2D=torch.where(ok[:, None], torch.stack([px, py], 1), z(P, 2)),
            depths=torch.where(ok, pv[:, 2], z(P)),
            radii=torch.where(ok, torch.ceil(torch.nan_to_num(rad)).to(torch.int32), z(P, dtype=torch.int32)),
            conic_opacity=torch.where(ok[:, None], torch.cat([conic, op[:, None]], 1), z(P, 4)),
            rgb=torch.where(ok[:, None], rgb, z(P, 3)),
            clamped=torch.where(ok[:, None], clamped, z(P, 3, dtype=torch.bool)),
            radius_float=torch.where(ok, rad, z(P)),
        )
        return out


def preprocess_backward(means3D, scales, rotations, shs, opacities, viewmatrix, projmatrix, campos,
                        tanfovx, tanfovy, H, W, D, radii, g_means2D, g_conic_opacity, g_rgb,
                        scale_modifier=1.0, create_graph_inputs=None):
    """Gradients w.r.t. (means3D, scales, rotations, shs, opacities) given the
    render gradients in the reference's conventions (NDC-scaled means2D
    gradient, half off-diagonal conic gradient).  Autograd of a
    differentiable restatement of the forward; Gaussians with radius 0 get
    zero gradient (reference backward.cu:158, 371)."""
    V = viewmatrix.reshape(-1).to(f32)
    Pm = projmatrix.reshape(-1).to(f32)
    leaves = [t.detach().clone().requires_grad_(True) for t in (means3D, scales, rotations, shs, opacities)]
    m, s, q, sh, op = leaves
    vis = (radii > 0)
    fx = float(np.float32(W) / (np.float32(2.0) * np.float32(tanfovx)))
    fy = float(np.float32(H) / (np.float32(2.0) * np.float32(tanfovy)))
    ph = _xform4(m, Pm)
    pw = 1.0 / (ph[:, 3] + 1e-7)
    ndc = ph[:, :2] * pw[:, None]
    c6 = cov3d(s, q, scale_modifier)
    a, b, c = _cov2d(m, V, fx, fy, float(np.float32(tanfovx)), float(np.float32(tanfovy)), c6, clamp_detach=True)
    det = a * c - b * b
    conic = torch.stack([c / det, -b / det, a / det], 1)
    rgb_raw = sh_rgb(D, m, campos.reshape(-1).to(f32), sh)
    rgb = torch.clamp(rgb_raw, min=0.0)
    gm = g_means2D[:, :2] * vis[:, None]
    gc = g_conic_opacity[:, :3] * torch.tensor([1.0, 2.0, 1.0]) * vis[:, None]
    gr = g_rgb * vis[:, None]
    L = ((ndc * gm).sum() + (torch.nan_to_num(conic) * gc).sum() + (rgb * gr).sum()
         + (op.reshape(-1) * g_conic_opacity[:, 3]).sum())
    grads = torch.autograd.grad(L, leaves, allow_unused=True)
    out = []
    for g, leaf in zip(grads, leaves):
        g = torch.zeros_like(leaf) if g is None else torch.nan_to_num(g)
        out.append(g)
    # opacity gradient passes through for every Gaussian (reference copies column 3)
    dm, ds, dq, dsh, dop = out
    mask = vis.to(f32)
    return dm * mask[:, None], ds * mask[:, None], dq * mask[:, None], dsh * mask[:, None, None], dop


# ---------------------------------------------------------------------------
# Binning
# ---------------------------------------------------------------------------

def tile_rect_int(means2D, radii, gx, gy):
    """Reference getRect (r/auxiliary.h:66-76), float32 arithmetic, truncation."""
    px = means2D[:, 0].astype(np.float32)
    py = means2D[:, 1].astype(np.float32)
    r = radii.astype(np.float32)
    T = np.float32(TILE)
    x0 = np.trunc((px - r) / T)
    y0 = np.trunc((py - r) / T)
    x1 = np.trunc((((px + r) + T) - np.float32(1)) / T)
    y1 = np.trunc((((py + r) + T) - np.float32(1)) / T)
    clip = lambda v, g: np.minimum(g, np.maximum(0, v.astype(np.int64)))
    return clip(x0, gx), clip(y0, gy), clip(x1, gx), clip(y1, gy)


def binning(means2D, depths, radii, H, W, compute_locally=None):
    """Per-tile Gaussian lists in (depth bits, index) order.  Returns
    (point_list int64 [R], ranges int64 [T,2], counts int64 [P])."""
    m = np.asarray(means2D, np.float32)
    d = np.asarray(depths, np.float32)
    r = np.asarray(radii, np.int64)
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = gx * gy
    mask = np.ones(T, bool) if compute_locally is None else np.asarray(compute_locally, bool).reshape(-1)
    x0, y0, x1, y1 = tile_rect_int(m, r, gx, gy)
    vis = r > 0
    idx_l, tile_l = [], []
    for i in np.nonzero(vis)[0]:
        for ty in range(y0[i], y1[i]):
            for tx in range(x0[i], x1[i]):
                t = ty * gx + tx
                if mask[t]:
                    idx_l.append(i)
                    tile_l.append(t)
    idx = np.asarray(idx_l, np.int64)
    tile = np.asarray(tile_l, np.int64)
    counts = np.bincount(idx, minlength=len(r)) if len(idx) else np.zeros(len(r), np.int64)
    if len(idx) == 0:
        return idx, np.zeros((T, 2), np.int64), counts
    dbits = d.view(np.uint32)[idx].astype(np.int64)
    order = np.lexsort((idx, dbits, tile))
    pl = idx[order]
    ts = tile[order]
    ranges = np.zeros((T, 2), np.int64)
    starts = np.searchsorted(ts, np.arange(T), side="left")
    ends = np.searchsorted(ts, np.arange(T), side="right")
    ranges[:, 0] = np.where(ends > starts, starts, 0)
    ranges[:, 1] = np.where(ends > starts, ends, 0)
    return pl, ranges, counts


# ---------------------------------------------------------------------------
# Blend
# ---------------------------------------------------------------------------

def _tile_pixels(t, gx, H, W):
    tx, ty = t % gx, t // gx
    ys, xs = torch.meshgrid(torch.arange(16) + ty * 16, torch.arange(16) + tx * 16, indexing="ij")
    xs, ys = xs.reshape(-1), ys.reshape(-1)
    inside = (xs < W) & (ys < H)
    return xs[inside], ys[inside]


def _pair_terms(ids, means2D, conic_opacity, xs, ys):
    xy = means2D[ids]
    co = conic_opacity[ids]
    dx = xy[None, :, 0] - xs[:, None].to(f32)
    dy = xy[None, :, 1] - ys[:, None].to(f32)
    power = -0.5 * (co[None, :, 0] * dx * dx + co[None, :, 2] * dy * dy) - co[None, :, 1] * dx * dy
    G = torch.exp(power)
    alpha = torch.clamp(co[None, :, 3] * G, max=0.99)
    ok = ~(power > 0) & ~(alpha < 1.0 / 255.0)
    return dx, dy, power, G, alpha, ok, co


def _transmittance(alpha, ok):
    """Sequential front-to-back transmittance with the 1e-4 stop.  Returns
    (contrib mask, T_before [npx,n], T_final [npx], last_contributor [npx])."""
    a = torch.where(ok, alpha, torch.zeros_like(alpha))
    one_m = 1 - a
    Tcum = torch.cumprod(one_m, dim=1)  # T after each entry (skipped entries multiply by 1)
    stop = ok & (Tcum < 1e-4)
    first_stop = torch.where(stop.any(1), stop.float().argmax(1), torch.full((alpha.shape[0],), alpha.shape[1]))
    n = alpha.shape[1]
    pos = torch.arange(n)[None, :]
    contrib = ok & (pos < first_stop[:, None])
    Tb = torch.cat([torch.ones(alpha.shape[0], 1), Tcum[:, :-1]], 1)
    last = torch.where(contrib.any(1), n - 1 - torch.flip(contrib, [1]).float().argmax(1), torch.full_like(first_stop, -1))
    T_final = torch.where(last >= 0, Tcum.gather(1, last.clamp(min=0)[:, None])[:, 0], torch.ones(alpha.shape[0]))
    return contrib, Tb, T_final, (last + 1).to(torch.int64)


def render_forward(means2D, conic_opacity, rgb, bg, point_list, ranges, H, W, compute_locally=None, P=None):
    """Returns dict(color [3,H,W], final_T [H*W], n_contrib [H*W], out_observe [P],
    n_render, n_consider, n_contrib_tile [T])."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = gx * gy
    P = means2D.shape[0] if P is None else P
    mask = np.ones(T, bool) if compute_locally is None else np.asarray(compute_locally, bool).reshape(-1)
    color = torch.zeros(3, H, W)
    final_T = torch.ones(H * W)
    n_contrib = torch.zeros(H * W, dtype=torch.int64)
    obs = torch.zeros(P, dtype=torch.int64)
    n_render = torch.zeros(T, dtype=torch.int64)
    n_consider = torch.zeros(T, dtype=torch.int64)
    n_ctile = torch.zeros(T, dtype=torch.int64)
    pl = torch.as_tensor(point_list, dtype=torch.int64)
    for t in range(T):
        if not mask[t]:
            continue
        s, e = int(ranges[t][0]), int(ranges[t][1])
        xs, ys = _tile_pixels(t, gx, H, W)
        pix = ys * W + xs
        n_render[t] = e - s
        if e == s:
            color[:, ys, xs] = bg.view(3, 1)
            continue
        ids = pl[s:e]
        dx, dy, power, G, alpha, ok, co = _pair_terms(ids, means2D, conic_opacity, xs, ys)
        contrib, Tb, Tf, last = _transmittance(alpha, ok)
        w = torch.where(contrib, alpha * Tb, torch.zeros_like(alpha))
        c = (w.double() @ rgb[ids].double()).float()  # [npx,3]; float64 sum: the same on every host CPU
        color[:, ys, xs] = (c + Tf[:, None] * bg.view(1, 3)).t()
        final_T[pix] = Tf
        n_contrib[pix] = last
        o = (contrib & (Tb > 0.5)).sum(0)
        obs.index_add_(0, ids, o)
        n_consider[t] = last.sum()
        n_ctile[t] = contrib.sum()
    return dict(color=color, final_T=final_T, n_contrib=n_contrib, out_observe=obs, n_render=n_render,
                n_consider=n_consider, n_contrib_tile=n_ctile)


def render_backward(means2D, conic_opacity, rgb, bg, point_list, ranges, H, W, dL_dpix, compute_locally=None):
    """Closed form of the reference backward (r/backward.cu:324-530) per tile.
    Returns the [P,16] record laid out as the product's (means2D xy at 0:2,
    |means2D| xy at 4:6, conic00/01/11/opacity at 8:12, rgb at 12:15)."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = gx * gy
    P = means2D.shape[0]
    mask = np.ones(T, bool) if compute_locally is None else np.asarray(compute_locally, bool).reshape(-1)
    rec = torch.zeros(P, 16, dtype=torch.float64)
    pl = torch.as_tensor(point_list, dtype=torch.int64)
    for t in range(T):
        if not mask[t]:
            continue
        s, e = int(ranges[t][0]), int(ranges[t][1])
        if e == s:
            continue
        xs, ys = _tile_pixels(t, gx, H, W)
        ids = pl[s:e]
        dx, dy, power, G, alpha, ok, co = _pair_terms(ids, means2D, conic_opacity, xs, ys)
        contrib, Tb, Tf, last = _transmittance(alpha, ok)
        dpix = dL_dpix[:, ys, xs].t()  # [npx,3]
        c = rgb[ids]  # [n,3]
        a = torch.where(contrib, alpha, torch.zeros_like(alpha)).double()
        Tb64 = Tb.double()
        w = a * Tb64
        # colour accumulated strictly behind entry j: S_j = sum_{k>j} c_k a_k T_k
        wc = w[:, :, None] * c.double()[None]                 # [npx,n,3]
        S = torch.flip(torch.cumsum(torch.flip(wc, [1]), 1), [1]) - wc
        one_m = (1 - a)
        dL_dalpha = ((c.double()[None] * Tb64[:, :, None] - S / one_m[:, :, None]) * dpix.double()[:, None, :]).sum(2)
        bgdot = (bg.double().view(1, 3) * dpix.double()).sum(1)
        dL_dalpha = dL_dalpha - (Tf.double()[:, None] / one_m) * bgdot[:, None]
        dL_dalpha = torch.where(contrib, dL_dalpha, torch.zeros_like(dL_dalpha))
        Gd, dxd, dyd = G.double(), dx.double(), dy.double()
        cod = co.double()
        dL_dG = cod[None, :, 3] * dL_dalpha
        gdx, gdy = Gd * dxd, Gd * dyd
        dG_ddx = -gdx * cod[None, :, 0] - gdy * cod[None, :, 1]
        dG_ddy = -gdy * cod[None, :, 2] - gdx * cod[None, :, 1]
        gmx = dL_dG * dG_ddx * (0.5 * W)
        gmy = dL_dG * dG_ddy * (0.5 * H)
        rec[:, 0].index_add_(0, ids, gmx.sum(0))
        rec[:, 1].index_add_(0, ids, gmy.sum(0))
        rec[:, 4].index_add_(0, ids, gmx.abs().sum(0))
        rec[:, 5].index_add_(0, ids, gmy.abs().sum(0))
        rec[:, 8].index_add_(0, ids, (-0.5 * gdx * dxd * dL_dG).sum(0))
        rec[:, 9].index_add_(0, ids, (-0.5 * gdx * dyd * dL_dG).sum(0))
        rec[:, 10].index_add_(0, ids, (-0.5 * gdy * dyd * dL_dG).sum(0))
        rec[:, 11].index_add_(0, ids, (Gd * dL_dalpha).sum(0))
        dcol = (w[:, :, None] * dpix.double()[:, None, :]).sum(0)  # [n,3]
        rec[:, 12:15].index_add_(0, ids, dcol)
    return rec.to(f32)


# ---------------------------------------------------------------------------
# Loss
# ---------------------------------------------------------------------------

def ssim_window():
    g = torch.tensor([math.exp(-((x - 5) ** 2) / float(2 * 1.5 ** 2)) for x in range(11)], dtype=f32)
    g = g / g.sum()
    return (g[:, None] @ g[None, :]).float()


def band_loss_sums(img, gt):
    """(sum |img-gt|, sum SSIM-map) over a [C,Hb,W] band with zero padding at
    the band edges; gt uint8 is divided by 255 and clamped."""
    if gt.dtype == torch.uint8:
        gt = torch.clamp(gt.to(f32) / 255.0, 0.0, 1.0)
    C = img.shape[0]
    w = ssim_window().expand(C, 1, 11, 11).contiguous()
    conv = lambda x: F.conv2d(x, w, padding=5, groups=C)
    mu1, mu2 = conv(img), conv(gt)
    mu1_sq, mu2_sq, mu1_mu2 = mu1.pow(2), mu2.pow(2), mu1 * mu2
    s1 = conv(img * img) - mu1_sq
    s2 = conv(gt * gt) - mu2_sq
    s12 = conv(img * gt) - mu1_mu2
    C1, C2 = 0.01 ** 2, 0.03 ** 2
    ssim_map = ((2 * mu1_mu2 + C1) * (2 * s12 + C2)) / ((mu1_sq + mu2_sq + C1) * (s1 + s2 + C2))
    return torch.abs(img - gt).sum(), ssim_map.sum()


def loss_and_grad(img, gt, num_pixels, lambda_dssim=0.2):
    """loss = (1-l) * L1/N3 + l * (1 - SSIM/N3), N3 = num_pixels*3; returns
    (loss, l1_sum, ssim_sum, dL/dimg)."""
    x = img.detach().clone().requires_grad_(True)
    l1, ss = band_loss_sums(x, gt)
    n3 = num_pixels * 3
    loss = (1.0 - lambda_dssim) * (l1 / n3) + lambda_dssim * (1.0 - ss / n3)
    (g,) = torch.autograd.grad(loss, [x])
    return loss.detach(), l1.detach(), ss.detach(), g


# ---------------------------------------------------------------------------
# Whole step
# ---------------------------------------------------------------------------

def train_step(scene_params, cam, gt, sh_degree=3, bg=None, lambda_dssim=0.2, compute_locally=None, reg_weight=0.0):
    """One camera: activations -> preprocess -> binning -> blend -> loss ->
    backward -> gradients w.r.t. the raw parameters.  reg_weight adds the
    min-scale regulariser of loss_distribution.py:314-322 over the Gaussians
    the exchange would send (radius > 0, non-empty tile rect)."""
    xyz, scaling, rotation, opacity, fdc, frest = scene_params
    bg = torch.zeros(3) if bg is None else bg
    H, W = cam.image_height, cam.image_width
    raw = [t.detach().clone().requires_grad_(True) for t in (xyz, scaling, rotation, opacity, fdc, frest)]
    s_act = torch.exp(raw[1])
    q_act = F.normalize(raw[2])
    o_act = torch.sigmoid(raw[3])
    shs = torch.cat((raw[4], raw[5]), 1)
    pre = preprocess_forward(raw[0].detach(), s_act.detach(), q_act.detach(), shs.detach(), o_act.detach(),
                             cam.world_view_transform, cam.full_proj_transform, cam.camera_center,
                             cam.tanfovx, cam.tanfovy, H, W, sh_degree)
    pl, ranges, counts = binning(pre["means2D"].numpy(), pre["depths"].numpy(), pre["radii"].numpy(), H, W,
                                 compute_locally)
    fwd = render_forward(pre["means2D"], pre["conic_opacity"], pre["rgb"], bg, pl, ranges, H, W, compute_locally)
    loss, l1, ss, dimg = loss_and_grad(fwd["color"], gt, H * W, lambda_dssim)
    rec = render_backward(pre["means2D"], pre["conic_opacity"], pre["rgb"], bg, pl, ranges, H, W, dimg,
                          compute_locally)
    dm, ds, dq, dsh, dop = preprocess_backward(raw[0].detach(), s_act.detach(), q_act.detach(), shs.detach(),
                                               o_act.detach(), cam.world_view_transform, cam.full_proj_transform,
                                               cam.camera_center, cam.tanfovx, cam.tanfovy, H, W, sh_degree,
                                               pre["radii"], rec[:, 0:2], rec[:, 8:12], rec[:, 12:15])
    torch.autograd.backward([raw[0], s_act, q_act, o_act, shs], [dm, ds, dq, dop.reshape(o_act.shape), dsh],
                            retain_graph=True)
    if reg_weight:
        gxn, gyn = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
        sent = torch.as_tensor(route_bool(pre["means2D"].numpy(), pre["radii"].numpy(), H, W, [0, gxn * gyn])[:, 0])
        vis = sent & (pre["radii"] > 0)
        if int(vis.sum()) > 0:
            reg = reg_weight * torch.sort(s_act[vis], dim=-1)[0][..., 0].mean()
            reg.backward()
            loss = loss + reg.detach()
    grads = [t.grad if t.grad is not None else torch.zeros_like(t) for t in raw]
    return dict(pre=pre, point_list=pl, ranges=ranges, counts=counts, fwd=fwd, loss=loss, l1_sum=l1,
                ssim_sum=ss, dimg=dimg, rec=rec, grads=grads)


# ---------------------------------------------------------------------------
# Routing
# ---------------------------------------------------------------------------

def route_bool(means2D, radii, H, W, dist_global_strategy, avoid_pixel_all2all=False):
    """Reference getTouchedIdsBool (f/rasterize_points.cu:212-256): bool [P, ws]."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    x0, y0, x1, y1 = tile_rect_int(np.asarray(means2D, np.float32), np.asarray(radii, np.int64), gx, gy)
    tmin = y0 * gx + x0
    tmax = (y1 - 1) * gx + x1 - 1
    dist = np.asarray(dist_global_strategy, np.int64)
    ws = len(dist) - 1
    out = np.zeros((len(tmin), ws), bool)
    for rk in range(ws):
        lo, hi = dist[rk], dist[rk + 1]
        if avoid_pixel_all2all:
            lo, hi = lo - (gx + 1), hi + (gx + 1)
        out[:, rk] = (tmax >= tmin) & ~((tmax < lo) | (tmin >= hi))
    return out


def route_rect_bool(means2D, radii, H, W, rectangles, avoid_pixel_all2all=False):
    """Reference getTouchedIdsBoolAdjustMode6 (f/rasterize_points.cu:291-335):
    rank rk renders tile rows [y_l, y_r) and columns [x_l, x_r)
    (rectangles[rk]); the square tile rect is tested without rejecting an
    empty one first.  bool [P, ws]."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    x0, y0, x1, y1 = tile_rect_int(np.asarray(means2D, np.float32), np.asarray(radii, np.int64), gx, gy)
    rects = np.asarray(rectangles, np.int64).reshape(-1, 4)
    out = np.zeros((len(x0), len(rects)), bool)
    for rk, (yl, yr, xl, xr) in enumerate(rects):
        if avoid_pixel_all2all:
            yl = yl - 1 if yl > 0 else yl
            xl = xl - 1 if xl > 0 else xl
            yr, xr = yr + 1, xr + 1
        out[:, rk] = ~((y1 <= yl) | (yr <= y0) | (x1 <= xl) | (xr <= x0))
    return out


# ---------------------------------------------------------------------------
# Full (non-distributed) rasterizer: rasterize_gaussians / _simp / mark_visible
# ---------------------------------------------------------------------------

def tile_rect_float(means2D, rects, gx, gy):
    """Reference getRect with float half-extents (f/cuda_rasterizer/
    auxiliary.h:63-73): floor / ceil of (mean -+ extent) / 16, clamped."""
    m = torch.as_tensor(np.asarray(means2D, np.float32))
    e = torch.as_tensor(np.asarray(rects, np.float32))
    T = torch.tensor(float(TILE), dtype=f32)
    clip = lambda v, g: v.to(torch.int64).clamp(0, g).numpy()  # noqa: E731
    return (clip(torch.floor((m[:, 0] - e[:, 0]) / T), gx), clip(torch.floor((m[:, 1] - e[:, 1]) / T), gy),
            clip(torch.ceil((m[:, 0] + e[:, 0]) / T), gx), clip(torch.ceil((m[:, 1] + e[:, 1]) / T), gy))


def tile_reached(conic_opacity, means2D, tx, ty):
    """Reference exact tile test (f/cuda_rasterizer/rasterizer_impl.cu:52-97,
    153-170), float32, vectorised over (Gaussian, tile) pairs: the exponent
    factor 0.5 d^T conic d at the point of the tile's pixel-centre rectangle
    the test picks, compared with ln(opacity * 255).  The FMAs are the ones
    nvcc forms from the reference expressions (first product of each sum
    fused), evaluated with fma32."""
    co = torch.as_tensor(conic_opacity, dtype=f32)
    m = torch.as_tensor(means2D, dtype=f32)
    tx = torch.as_tensor(tx, dtype=torch.int64)
    ty = torch.as_tensor(ty, dtype=torch.int64)
    span = torch.tensor(float(TILE - 1), dtype=f32)
    x0, x1 = (tx * TILE).to(f32), ((tx + 1) * TILE - 1).to(f32)
    y0, y1 = (ty * TILE).to(f32), ((ty + 1) * TILE - 1).to(f32)
    mx, my = m[:, 0], m[:, 1]
    gap_x, gap_y = x0 - mx, y0 - my
    before_x, before_y = gap_x > 0, gap_y > 0
    out_x, out_y = before_x | (mx > x1), before_y | (my > y1)
    cx, cy = torch.where(before_x, x0, x1), torch.where(before_y, y0, y1)
    sx, sy = torch.copysign(span.expand_as(gap_x), gap_x), torch.copysign(span.expand_as(gap_y), gap_y)
    ex, ey = mx - cx, my - cy
    rx = 1.0 / ((span * span) * co[:, 0])
    ry = 1.0 / ((span * span) * co[:, 2])
    sat = lambda v: torch.where(torch.isnan(v), torch.zeros_like(v), v.clamp(0.0, 1.0))  # noqa: E731
    ux = sat(fma32(sx * co[:, 0], ex, (sx * co[:, 1]) * ey) * rx)
    uy = sat(fma32(sy * co[:, 1], ex, (sy * co[:, 2]) * ey) * ry)
    zero = torch.zeros_like(ux)
    qx = fma32(torch.where(out_y, ux, zero), sx, cx)
    qy = fma32(torch.where(out_x, uy, zero), sy, cy)
    dx, dy = mx - qx, my - qy
    half = torch.full_like(dx, 0.5)
    f = fma32(half, fma32(co[:, 0] * dx, dx, (co[:, 2] * dy) * dy), (co[:, 1] * dx) * dy)
    f = torch.where(out_x | out_y, f, zero)
    thr = torch.log(co[:, 3] / torch.tensor(1.0 / 255.0, dtype=f32))
    return (f <= thr).numpy()


def full_binning(means2D, depths, radii, rects, conic_opacity, H, W):
    """Per-tile lists of the full rasterizer (rasterizer_impl.cu:119-191,
    336-430): each Gaussian with radius > 0 over its float rectangle, only
    the tiles that pass the exact tile test, in (depth bits, index) order.
    Returns (point_list int64 [R], ranges int64 [T,2], counts int64 [P])."""
    m = np.asarray(means2D, np.float32)
    d = np.asarray(depths, np.float32)
    r = np.asarray(radii, np.int64)
    co = np.asarray(conic_opacity, np.float32)
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    T = gx * gy
    x0, y0, x1, y1 = tile_rect_float(m, rects, gx, gy)
    idx_l, tx_l, ty_l = [], [], []
    for i in np.nonzero(r > 0)[0]:
        for ty in range(y0[i], y1[i]):
            for tx in range(x0[i], x1[i]):
                idx_l.append(i)
                tx_l.append(tx)
                ty_l.append(ty)
    idx = np.asarray(idx_l, np.int64)
    if len(idx):
        keep = tile_reached(co[idx], m[idx], np.asarray(tx_l), np.asarray(ty_l))
        idx = idx[keep]
        tile = (np.asarray(ty_l) * gx + np.asarray(tx_l))[keep]
    counts = np.bincount(idx, minlength=len(r)) if len(idx) else np.zeros(len(r), np.int64)
    if len(idx) == 0:
        return idx, np.zeros((T, 2), np.int64), counts
    order = np.lexsort((idx, d.view(np.uint32)[idx].astype(np.int64), tile))
    pl, ts = idx[order], tile[order]
    ranges = np.zeros((T, 2), np.int64)
    starts = np.searchsorted(ts, np.arange(T), side="left")
    ends = np.searchsorted(ts, np.arange(T), side="right")
    ranges[:, 0] = np.where(ends > starts, starts, 0)
    ranges[:, 1] = np.where(ends > starts, ends, 0)
    return pl, ranges, counts


def render_stats(means2D, conic_opacity, point_list, ranges, H, W, P):
    """Statistics of rasterize_gaussians (flag_max_count) and
    rasterize_gaussians_simp (f/cuda_rasterizer/forward.cu:402-440, 566-590):
    per pixel, +1 for the contributing Gaussian of largest alpha*T (the first
    in list order on ties); over every (pixel, Gaussian) blend, the sum of
    alpha*T and the count.  Returns (max_count, accum_w, accum_n), float64 /
    int64 [P]."""
    gx, gy = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    mx = torch.zeros(P, dtype=torch.float64)
    aw = torch.zeros(P, dtype=torch.float64)
    an = torch.zeros(P, dtype=torch.int64)
    pl = torch.as_tensor(point_list, dtype=torch.int64)
    m2 = torch.as_tensor(means2D, dtype=f32)
    co = torch.as_tensor(conic_opacity, dtype=f32)
    for t in range(gx * gy):
        s, e = int(ranges[t][0]), int(ranges[t][1])
        if e == s:
            continue
        xs, ys = _tile_pixels(t, gx, H, W)
        ids = pl[s:e]
        _, _, _, _, alpha, ok, _ = _pair_terms(ids, m2, co, xs, ys)
        contrib, Tb, _, _ = _transmittance(alpha, ok)
        w = torch.where(contrib, alpha * Tb, torch.zeros_like(alpha))
        aw.index_add_(0, ids, w.double().sum(0))
        an.index_add_(0, ids, contrib.sum(0))
        has = contrib.any(1)
        best = torch.where(contrib, w, torch.full_like(w, -1.0)).argmax(1)
        mx.index_add_(0, ids[best[has]], torch.ones(int(has.sum()), dtype=torch.float64))
    return mx, aw, an


def mark_visible(means3D, viewmatrix):
    """Reference checkFrustum / in_frustum (f/cuda_rasterizer/
    rasterizer_impl.cu:100-114, auxiliary.h:158-185): view depth > 0.2."""
    p = torch.as_tensor(means3D, dtype=f32)
    return (_xform3(p, torch.as_tensor(viewmatrix, dtype=f32).reshape(-1))[:, 2] > 0.2).numpy()


def fma32(a, b, c):
    """Correctly rounded float32 fused multiply-add of float32 tensors.
    a*b is exact in float64 (2 x 24 significant bits); s + c is formed in
    float64 with its exact rounding error (Knuth's TwoSum), and a float64 sum
    that sits exactly halfway between two float32 values is moved one float64
    step toward the error's sign before the final rounding, so the double
    rounding cannot go the wrong way.  Exact for results in the float32
    normal range."""
    a, b, c = a.double(), b.double(), c.double()
    s = a * b
    t = s + c
    bp = t - s
    err = (s - (t - bp)) + (c - bp)
    half = (t.view(torch.int64) & ((1 << 29) - 1)) == (1 << 28)
    up = torch.nextafter(t, torch.full_like(t, float("inf")))
    down = torch.nextafter(t, torch.full_like(t, float("-inf")))
    t = torch.where(half & (err > 0), up, torch.where(half & (err < 0), down, t))
    return t.float()


def adam_update(param, grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps):
    """Reference adamUpdateCUDA (f/cuda_rasterizer/adam.cu:10-38) on [N, M]
    float32 tensors, in place, for the rows with visible[g].  The moment
    updates are the fused multiply-adds the reference build makes of
    f/cuda_rasterizer/adam.cu:30-31 -- fma(1-b1, g, b1*m) and
    fma((1-b2)*g, g, b2*v) -- so the result is bit-exact."""
    f = lambda x: torch.tensor(x, dtype=f32)
    b1, b2, lr, eps = f(b1), f(b2), f(lr), f(eps)
    v = visible.bool()
    g = grad[v]
    m = fma32((f(1.0) - b1).expand_as(g), g, b1 * exp_avg[v])
    s = fma32((f(1.0) - b2) * g, g, b2 * exp_avg_sq[v])
    # float32 square root correctly rounded: from float64, where one rounding
    # to float32 is exact (53 >= 2*24 + 2 bits); torch's vectorised float32
    # sqrt on the CPU need not be
    step = (-lr * m) / (torch.sqrt(s.double()).float() + eps)
    param[v] = param[v] + step
    exp_avg[v] = m
    exp_avg_sq[v] = s


def densification_stats(max_radii2D, xyz_gradient_accum, denom, radii, grad_means2D):
    """One camera's densification statistics, in place, as the reference
    updates them (train_internal.py:365-367 max_radii2D over the visibility
    filter; scene/gaussian_model.py:792-794 add_densification_stats): vis =
    radii > 0, grad_means2D [P, >=2] the viewspace gradient of every
    Gaussian."""
    vis = radii > 0
    max_radii2D[vis] = torch.max(max_radii2D[vis], radii[vis].to(max_radii2D.dtype))
    xyz_gradient_accum[vis] += torch.norm(grad_means2D[vis, :2], dim=-1, keepdim=True)
    denom[vis] += 1
