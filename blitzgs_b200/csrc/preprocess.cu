// EWA preprocess, forward and backward, one thread per Gaussian.
//
// Forward follows the reference preprocessCUDA
// (submodule/diff-gaussian-rasterization_f/cuda_rasterizer/forward.cu:164-284,
// host side rasterizer_impl.cu:982-1067) with three B200-side differences
// that do not change any output bit:
//   * no per-call cudaMalloc/cudaMemset/cudaFree of temporaries;
//   * every output element is written by the kernel (zeros for culled
//     Gaussians), so the caller needs no zero-fill pass;
//   * SH coefficients are read through a (dc, rest) pointer pair with a
//     per-Gaussian stride, so both the [P,16,3] tensor of the operator API and
//     the model's separate _features_dc / _features_rest tensors are read in
//     place (no torch.cat and no .contiguous() split copies); the
//     contiguous [P,16,3] case is read with 16-byte vector loads.
// Backward computes, in one kernel, the gradients the reference's
// computeCov2DCUDA and preprocessCUDA backward produce (backward.cu:146-400),
// from a matrix-form derivation of its own (written out above bwd_compute),
// and recomputes the 3D covariance and the clamp flags instead of reading
// them back from saved buffers.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "scan.cuh"

namespace blitz {

// Load the SH coefficients of Gaussian i into registers.  16 coefficient
// triplets at most (degree 3).
struct ShRegs {
  float dc[3];
  float rest[45];
};

__device__ __forceinline__ void load_sh(const PreprocessParams& p, int64_t i, int nrest,
                                        ShRegs& s) {
  const float* dc = p.dc + i * p.dc_stride;
  const float* rest = p.rest + i * p.rest_stride;
  if (p.sh_packed16) {
    // Contiguous [P,16,3]: 48 floats = 12 x float4, dc is the first triplet.
    const float4* v = reinterpret_cast<const float4*>(dc);
    float buf[48];
#pragma unroll
    for (int k = 0; k < 12; ++k) {
      float4 q = __ldg(v + k);
      buf[4 * k + 0] = q.x;
      buf[4 * k + 1] = q.y;
      buf[4 * k + 2] = q.z;
      buf[4 * k + 3] = q.w;
    }
    s.dc[0] = buf[0];
    s.dc[1] = buf[1];
    s.dc[2] = buf[2];
#pragma unroll
    for (int k = 0; k < 45; ++k) s.rest[k] = buf[3 + k];
  } else {
    s.dc[0] = __ldg(dc + 0);
    s.dc[1] = __ldg(dc + 1);
    s.dc[2] = __ldg(dc + 2);
#pragma unroll
    for (int k = 0; k < 45; ++k) s.rest[k] = (k < nrest * 3) ? __ldg(rest + k) : 0.f;
  }
}

// Activations of the raw model parameters, in the float arithmetic PyTorch's
// CUDA kernels use for torch.exp, torch.sigmoid and F.normalize
// (scene/gaussian_model.py:248-276 applies them before the rasterizer), so
// the activated values are bit-identical to the reference pipeline's.
__device__ __forceinline__ float act_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float quat_norm(float4 q) {
  // ||q|| as PyTorch's CUDA norm over a contiguous [P,4] row computes it:
  // squares rounded individually, then (x0^2 + x2^2) + (x1^2 + x3^2), then a
  // correctly rounded sqrt (bit-identical on 4M random quaternions; checked
  // by tests/test_gpu_parity.py).
  const float a = __fmul_rn(q.x, q.x), b = __fmul_rn(q.y, q.y), c = __fmul_rn(q.z, q.z), d = __fmul_rn(q.w, q.w);
  return __fsqrt_rn(__fadd_rn(__fadd_rn(a, c), __fadd_rn(b, d)));
}

struct Activated {
  float sx, sy, sz;
  float4 q;    // normalised rotation
  float nrm;   // max(||q_raw||, 1e-12)
  float o;
};

__device__ __forceinline__ Activated activate(const PreprocessParams& p, int64_t i) {
  Activated a;
  float sx = __ldg(p.scales + 3 * i + 0), sy = __ldg(p.scales + 3 * i + 1), sz = __ldg(p.scales + 3 * i + 2);
  float4 q = __ldg(reinterpret_cast<const float4*>(p.rotations) + i);
  // the operator-API backward passes no opacities (it never needs them)
  float o = p.opacities ? __ldg(p.opacities + i) : 0.f;
  if (p.raw) {
    sx = expf(sx);
    sy = expf(sy);
    sz = expf(sz);
    const float n = p.rot_norm ? __ldg(p.rot_norm + i) : quat_norm(q);
    a.nrm = fmaxf(n, 1e-12f);
    q = make_float4(q.x / a.nrm, q.y / a.nrm, q.z / a.nrm, q.w / a.nrm);
    o = act_sigmoid(o);
  } else {
    a.nrm = 1.f;
  }
  a.sx = sx;
  a.sy = sy;
  a.sz = sz;
  a.q = q;
  a.o = o;
  return a;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
//
// Two phases inside one persistent kernel.  In a training view only a few
// percent of the Gaussians survive the frustum cull, so a thread-per-Gaussian
// kernel spends its time waiting on one 12-byte xyz load per thread.
//   Phase A (streaming cull): each block takes chunks of kPreChunk Gaussians;
//     every thread loads xyz (and the scales of Gaussians in front of the near
//     plane) of kPreUnroll Gaussians at once and applies a conservative
//     screen-space bound.  Gaussians it rejects are certain to get radius 0
//     from the full computation; their rows are written here.
//   Phase B (full computation): the survivors are queued in shared memory and
//     processed a full block at a time, so every lane does useful work.
// Outputs are those of the reference preprocessCUDA bit for bit; phase A only
// decides who can skip the full computation.

constexpr int kPreThreads = 256;
constexpr int kPreUnroll = 8;
constexpr int kPreChunk = kPreThreads * kPreUnroll;
constexpr int kPreQueue = kPreChunk + kPreThreads;  // < kPreThreads carried over + one chunk
constexpr int kPreMaskSmem = 32 * 1024;             // tiles whose mask is staged in shared memory

// Everything the full computation produces for one Gaussian.
struct PreResult {
  float2 pimg;
  float depth;
  int radius;
  float4 conic_op;
  V3 rgb;
  bool clamp3[3];
  float cov3d[6];
  float smin;   // smallest activated scale (regulariser)
  float2 rect;  // half-extents of the screen rectangle (full rasterizer)
};

// Squared Frobenius norm of the rotation matrix built from q.
__device__ __forceinline__ float rot_frob2(float4 q) {
  const float r00 = 1.f - 2.f * (q.z * q.z + q.w * q.w), r01 = 2.f * (q.y * q.z - q.x * q.w), r02 = 2.f * (q.y * q.w + q.x * q.z);
  const float r10 = 2.f * (q.y * q.z + q.x * q.w), r11 = 1.f - 2.f * (q.y * q.y + q.w * q.w), r12 = 2.f * (q.z * q.w - q.x * q.y);
  const float r20 = 2.f * (q.y * q.w - q.x * q.z), r21 = 2.f * (q.z * q.w + q.x * q.y), r22 = 1.f - 2.f * (q.y * q.y + q.z * q.z);
  return r00 * r00 + r01 * r01 + r02 * r02 + r10 * r10 + r11 * r11 + r12 * r12 + r20 * r20 + r21 * r21 + r22 * r22;
}

// Conservative screen-space bound.  The tile rect of the full computation uses
// half-extents <= my_radius = extent * sqrt(lambda) with extent <= 3.33,
// lambda <= trace(cov2D) + 0.1 and trace(cov2D) <= s_max^2 ||R||_F^2
// ||J||_F^2 ||W||_F^2 + 0.6 (W the view rotation, R the rotation matrix, S the
// scales), where |t.x/t.z| is clamped to 1.3 tan(fov) inside J.  If even that
// radius keeps the rect outside the tile grid, the full computation would cull
// the Gaussian too.  NaNs never make it return true.
struct CullBound {
  float wf;    // ||W||_F^2
  float jnum;  // ||J||_F^2 * z^2
  float gw, gh;
  // Magnitude bounds of the affine rows phase A evaluates: for a point with
  // max(|x|,|y|,|z|) = m, the terms of each row sum in absolute value to at
  // most lin * m + off (zw: view z and clip w; xy: clip x and clip y).
  float zw_lin, zw_off, xy_lin, xy_off;
};

// Rounding bound for a 4-term affine row a*x + b*y + c*z + d evaluated in
// float32, with or without FMA contraction: each of its at most six
// operations rounds a partial result bounded by S = |a x| + |b y| + |c z| + |d|
// by at most u = 2^-24 relative, so two evaluations of the same row in
// different orders differ by at most 12 u S.  16 u S leaves room.
constexpr float kAffineErr = 16.0f / 16777216.0f;

__device__ __forceinline__ CullBound make_cull_bound(const PreprocessParams& p, const float* Vs, const float* Ps) {
  CullBound c;
  c.wf = Vs[0] * Vs[0] + Vs[1] * Vs[1] + Vs[2] * Vs[2] + Vs[4] * Vs[4] + Vs[5] * Vs[5] + Vs[6] * Vs[6] + Vs[8] * Vs[8] +
         Vs[9] * Vs[9] + Vs[10] * Vs[10];
  const float cx = 1.3f * p.tanfovx, cy = 1.3f * p.tanfovy;
  c.jnum = p.focal_x * p.focal_x * (1.f + cx * cx) + p.focal_y * p.focal_y * (1.f + cy * cy);
  c.gw = (float)(p.grid_x * kTileX);
  c.gh = (float)(p.grid_y * kTileY);
  c.zw_lin = fmaxf(fabsf(Vs[2]) + fabsf(Vs[6]) + fabsf(Vs[10]), fabsf(Ps[3]) + fabsf(Ps[7]) + fabsf(Ps[11]));
  c.zw_off = fmaxf(fabsf(Vs[14]), fabsf(Ps[15]));
  c.xy_lin = fmaxf(fabsf(Ps[0]) + fabsf(Ps[4]) + fabsf(Ps[8]), fabsf(Ps[1]) + fabsf(Ps[5]) + fabsf(Ps[9]));
  c.xy_off = fmaxf(fabsf(Ps[12]), fabsf(Ps[13]));
  return c;
}

__device__ __forceinline__ bool off_grid(const CullBound& c, float2 pimg, float z, float smax, float rf) {
  const float jf = c.jnum / (z * z);
  const float rb = 3.34f * sqrtf((smax * smax * rf * jf * c.wf + 0.8f) * 1.01f) + 2.f;
  return pimg.x + rb < -1.f || pimg.x - rb > c.gw + 1.f || pimg.y + rb < -1.f || pimg.y - rb > c.gh + 1.f;
}

// The reference per-Gaussian computation (forward.cu:164-284) for one
// Gaussian that passed phase A.
__device__ __forceinline__ void preprocess_one(const PreprocessParams& p, const float* Vs, const float* Ps,
                                               const CullBound& cb, int64_t i, PreResult& r) {
  const float3 p_orig = make_float3(__ldg(p.means3D + 3 * i + 0), __ldg(p.means3D + 3 * i + 1),
                                    __ldg(p.means3D + 3 * i + 2));
  r.pimg = make_float2(0.f, 0.f);
  r.depth = 0.f;
  r.radius = 0;
  r.conic_op = make_float4(0.f, 0.f, 0.f, 0.f);
  r.rgb = {0.f, 0.f, 0.f};
  r.clamp3[0] = r.clamp3[1] = r.clamp3[2] = false;
#pragma unroll
  for (int k = 0; k < 6; ++k) r.cov3d[k] = 0.f;
  r.smin = 0.f;
  r.rect = make_float2(0.f, 0.f);

  do {
    // near-plane test (reference in_frustum, auxiliary.h:156-185)
    const float3 p_view = xform_point3(p_orig, Vs);
    if (p_view.z <= 0.2f) {
      if (p.prefiltered) atomicOr(p.error_flag, kErrPrefilteredCulled);
      break;
    }
    const float4 p_hom = xform_point4(p_orig, Ps);
    const float p_w = 1.0f / (p_hom.w + 0.0000001f);
    const float3 p_proj = make_float3(p_hom.x * p_w, p_hom.y * p_w, p_hom.z * p_w);
    const float2 pimg = make_float2(ndc_to_pix(p_proj.x, p.W), ndc_to_pix(p_proj.y, p.H));

    const Activated act = activate(p, i);
    r.smin = fminf(act.sx, fminf(act.sy, act.sz));
    // the bound again, now with the rotation's own ||R||_F^2
    const float smax = fabsf(p.scale_modifier) * fmaxf(fabsf(act.sx), fmaxf(fabsf(act.sy), fabsf(act.sz)));
    if (off_grid(cb, pimg, p_view.z, smax, rot_frob2(act.q))) break;

    cov3d_from_scale_rot(act.sx, act.sy, act.sz, p.scale_modifier, act.q, r.cov3d);
    const float3 cov = cov2d_ewa(p_orig, p.focal_x, p.focal_y, p.tanfovx, p.tanfovy, r.cov3d, Vs);

    const float det = (cov.x * cov.z - cov.y * cov.y);
    if (det == 0.0f) break;
    const float det_inv = 1.f / det;
    const float3 conic = make_float3(cov.z * det_inv, -cov.y * det_inv, cov.x * det_inv);

    // Opacity-aware extent: min(3.33, sqrt(2 ln(255 alpha))).  The mixed
    // double/float min resolves to fmin in double, so a NaN (alpha < 1/255)
    // yields 3.33 and such Gaussians are not culled by opacity.
    const float opacity = act.o;
    constexpr float alpha_threshold = 1.0f / 255.0f;
    const float opacity_power_threshold = logf(opacity / alpha_threshold);
    const float extent = fmin(3.33, (double)sqrtf(2.0f * opacity_power_threshold));

    const float mid = 0.5f * (cov.x + cov.z);
    const float lambda = mid + sqrtf(fmaxf(0.01f, mid * mid - det));
    const float my_radius = extent * sqrtf(lambda);
    if (my_radius <= 0.0f) break;

    const float extent_x = fminf(extent * sqrtf(cov.x), my_radius);
    const float extent_y = fminf(extent * sqrtf(cov.z), my_radius);
    if (tile_rect_f_count(pimg, make_float2(extent_x, extent_y), p.grid_x, p.grid_y) == 0) break;

    ShRegs s;
    load_sh(p, i, p.M, s);
    r.rgb = sh_to_rgb(p.D, p_orig, p.campos, s.dc, s.rest, r.clamp3);

    r.depth = p_view.z;
    r.radius = (int)ceilf(my_radius);
    r.pimg = pimg;
    r.conic_op = make_float4(conic.x, conic.y, conic.z, opacity);
    r.rect = make_float2(extent_x, extent_y);
  } while (0);
}

__device__ __forceinline__ void store_one(const PreprocessParams& p, int64_t i, const PreResult& r) {
  reinterpret_cast<float2*>(p.out_means2D)[i] = r.pimg;
  p.out_depths[i] = r.depth;
  p.out_radii[i] = r.radius;
  reinterpret_cast<float4*>(p.out_conic_opacity)[i] = r.conic_op;
  p.out_rgb[3 * i + 0] = r.rgb.x;
  p.out_rgb[3 * i + 1] = r.rgb.y;
  p.out_rgb[3 * i + 2] = r.rgb.z;
  if (p.out_clamped) {
    p.out_clamped[3 * i + 0] = r.clamp3[0];
    p.out_clamped[3 * i + 1] = r.clamp3[1];
    p.out_clamped[3 * i + 2] = r.clamp3[2];
  }
  if (p.out_cov3D) {
#pragma unroll
    for (int k = 0; k < 6; ++k) p.out_cov3D[6 * i + k] = r.cov3d[k];
  }
  if (p.out_rects) reinterpret_cast<float2*>(p.out_rects)[i] = r.rect;
}

// Rows of a Gaussian rejected in phase A: zeros, like the reference's
// zero-initialised outputs.  With listed_rows_only, only radii (and counts)
// are written: the caller reads the other outputs through the visible list.
__device__ __forceinline__ void store_culled(const PreprocessParams& p, int64_t i) {
  p.out_radii[i] = 0;
  if (p.counts_out) p.counts_out[i] = 0u;
  if (p.listed_rows_only) return;
  reinterpret_cast<float2*>(p.out_means2D)[i] = make_float2(0.f, 0.f);
  p.out_depths[i] = 0.f;
  reinterpret_cast<float4*>(p.out_conic_opacity)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  p.out_rgb[3 * i + 0] = 0.f;
  p.out_rgb[3 * i + 1] = 0.f;
  p.out_rgb[3 * i + 2] = 0.f;
  if (p.out_clamped) {
    p.out_clamped[3 * i + 0] = false;
    p.out_clamped[3 * i + 1] = false;
    p.out_clamped[3 * i + 2] = false;
  }
  if (p.out_cov3D) {
#pragma unroll
    for (int k = 0; k < 6; ++k) p.out_cov3D[6 * i + k] = 0.f;
  }
  if (p.out_rects) reinterpret_cast<float2*>(p.out_rects)[i] = make_float2(0.f, 0.f);
}

// Per-thread running sums of one block, reduced once at the end of a kernel.
struct FwdAcc {
  double reg_v = 0.0, reg_c = 0.0;      // regulariser: sum of min scales, count
  unsigned long long r = 0ull, n = 0ull;  // tile instances, Gaussians with a tile
};

// Phase A for the kPreUnroll Gaussians base + u*kPreThreads of this thread:
// keep[u] is false only for Gaussians the full computation is certain to cull
// (their rows are written here).  Every test is conservative, so fast
// approximate arithmetic is enough: the view depth and the clip coordinates
// are evaluated here in an order of our own, so each test widens its
// threshold by the rounding bound kAffineErr of the affine rows (at city
// coordinates, |x| ~ 1000, that is ~1e-3 in depth); the exact tests are
// repeated in phase B with the reference's expressions.
__device__ __forceinline__ void cull_phase(const PreprocessParams& p, const float* Vs, const float* Ps,
                                           const CullBound& cb, int64_t base, bool (&keep)[kPreUnroll]) {
  // Without a rotation load, ||R||_F^2 <= 9: every entry of R is bounded by
  // |q|^2 <= 1 when q was normalised here.  A caller-supplied norm or an
  // operator-API rotation can have any length, so those load q.
  const bool load_q = !p.raw || p.rot_norm;
  const float abs_mod = fabsf(p.scale_modifier);
  // per-thread base pointers: Gaussian base + u * kPreThreads sits at a
  // compile-time offset from them
  const int64_t rem = p.P - base;  // Gaussians from base on
  const float* xb = p.means3D + 3 * base;
  const float* sb = p.scales + 3 * base;
  // xyz and the scales in one round trip (the scales of Gaussians behind the
  // camera are read for nothing, which costs less than a second round trip)
  float3 x[kPreUnroll], sc[kPreUnroll];
#pragma unroll
  for (int u = 0; u < kPreUnroll; ++u) {
    x[u] = make_float3(0.f, 0.f, 0.f);
    sc[u] = make_float3(0.f, 0.f, 0.f);
    if (u * kPreThreads < rem) {
      const int o = 3 * u * kPreThreads;
      x[u] = make_float3(__ldg(xb + o + 0), __ldg(xb + o + 1), __ldg(xb + o + 2));
      sc[u] = make_float3(__ldg(sb + o + 0), __ldg(sb + o + 1), __ldg(sb + o + 2));
    }
  }
#pragma unroll
  for (int u = 0; u < kPreUnroll; ++u) {
    const bool in = u * kPreThreads < rem;
    const float m = fmaxf(fabsf(x[u].x), fmaxf(fabsf(x[u].y), fabsf(x[u].z)));
    const float z = Vs[2] * x[u].x + Vs[6] * x[u].y + Vs[10] * x[u].z + Vs[14];
    // a Gaussian the caller culls is skipped before any test (forward.cu:196-203)
    const bool culled = in && p.culling && p.culling[base + u * kPreThreads];
    // the exact near test (z <= 0.2 culls) runs in phase B; here only what
    // is behind it by more than the rounding bound is dropped and reported
    keep[u] = in && !culled && z > 0.2f - kAffineErr * fmaf(cb.zw_lin, m, cb.zw_off);
    if (in && !culled && !keep[u] && p.prefiltered) atomicOr(p.error_flag, kErrPrefilteredCulled);
    if (keep[u]) {
      float m = fmaxf(fabsf(sc[u].x), fmaxf(fabsf(sc[u].y), fabsf(sc[u].z)));
      if (p.raw) m = __expf(fmaxf(sc[u].x, fmaxf(sc[u].y, sc[u].z)));  // exp is increasing: exp(max) = max(exp)
      const float smax = abs_mod * m * 1.0001f;
      float rf = 9.001f;
      if (load_q) {
        const int64_t i = base + u * kPreThreads;
        float4 q = __ldg(reinterpret_cast<const float4*>(p.rotations) + i);
        if (p.raw) {
          const float inv = 1.f / fmaxf(__ldg(p.rot_norm + i), 1e-12f);
          q = make_float4(q.x * inv, q.y * inv, q.z * inv, q.w * inv);
        }
        rf = rot_frob2(q) * 1.0001f + 1e-6f;
      }
      const float hx = Ps[0] * x[u].x + Ps[4] * x[u].y + Ps[8] * x[u].z + Ps[12];
      const float hy = Ps[1] * x[u].x + Ps[5] * x[u].y + Ps[9] * x[u].z + Ps[13];
      const float hw = Ps[3] * x[u].x + Ps[7] * x[u].y + Ps[11] * x[u].z + Ps[15];
      const float pw = __fdividef(1.f, hw + 0.0000001f);
      const float nx = hx * pw, ny = hy * pw;
      const float2 pimg = make_float2(((nx + 1.f) * (float)p.W - 1.f) * 0.5f, ((ny + 1.f) * (float)p.H - 1.f) * 0.5f);
      // pixel distance between this pimg and the reference's: the rounding
      // bounds of hx, hy and hw carried through x / w (a vanishing or
      // negative w gives an infinite or NaN margin, which keeps the Gaussian)
      const float ew = kAffineErr * fmaf(cb.zw_lin, m, cb.zw_off);
      const float exy = kAffineErr * fmaf(cb.xy_lin, m, cb.xy_off);
      const float ex = 0.5f * (float)p.W * fabsf(pw) * (exy + fabsf(nx) * ew);
      const float ey = 0.5f * (float)p.H * fabsf(pw) * (exy + fabsf(ny) * ew);
      const float jf = __fdividef(cb.jnum, z * z);
      const float v = (smax * smax * rf * jf * cb.wf + 0.8f) * 1.01f;
      const float rb = 3.34f * (v * rsqrtf(v)) * 1.0001f + 2.f;
      const float rx = rb + ex, ry = rb + ey;
      keep[u] = !(pimg.x + rx < -1.f || pimg.x - rx > cb.gw + 1.f || pimg.y + ry < -1.f || pimg.y - ry > cb.gh + 1.f);
    }
    if (in && !keep[u]) store_culled(p, base + u * kPreThreads);
  }
}

// Phase B for one Gaussian (valid) or a filler lane: full computation, the
// fused tile count and regulariser, the block-aggregated visible-list slot
// (three barriers: every thread of the block must call this together), and
// the row stores.  With scan_state the block's slots follow the ordered
// prefix of the listed counts of the rounds before `round` (the list keeps
// the candidates' order); without it they come from one atomic per block.
__device__ __forceinline__ void full_phase(const PreprocessParams& p, const float* Vs, const float* Ps,
                                           const CullBound& cb, int64_t i, bool valid, const bool* s_mask,
                                           bool use_smem, int* s_wc, int* s_base, FwdAcc& acc,
                                           int64_t round = -1, unsigned long long* scan_state = nullptr,
                                           unsigned* status = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  PreResult res;
  preprocess_one(p, Vs, Ps, cb, i, res);
  uint32_t cnt = 0;
  if (valid && res.radius > 0 && (p.counts_out || p.reg_sums)) {
    int2 lo, hi;
    tile_rect_int(res.pimg, res.radius, p.grid_x, p.grid_y, lo, hi);
    // min-scale regulariser (gaussian_renderer/loss_distribution.py:314-322):
    // Gaussians the exchange sends (radius > 0 and a non-empty square tile
    // rect, the get_local2j_ids test) contribute their smallest scale.
    if (p.reg_sums && (hi.y - 1) * p.grid_x + hi.x - 1 >= lo.y * p.grid_x + lo.x) {
      acc.reg_v += res.smin;
      acc.reg_c += 1.0;
    }
    // tile count of the binning (the sizing pass before duplicateWithKeys,
    // rasterizer_impl.cu), restricted to the tiles this rank renders
    if (p.counts_out) {
      if (!p.compute_locally) {
        cnt = (uint32_t)((hi.x - lo.x) * (hi.y - lo.y));
      } else {
        for (int y = lo.y; y < hi.y; ++y)
          for (int xx = lo.x; xx < hi.x; ++xx) {
            const int t = y * p.grid_x + xx;
            cnt += (use_smem ? s_mask[t] : p.compute_locally[t]) ? 1u : 0u;
          }
      }
    }
  }
  acc.r += cnt;
  acc.n += cnt > 0u ? 1ull : 0ull;
  if (p.vis_list_out) {
    // block-aggregated slots: one atomic per block and round
    const bool listed = valid && res.radius > 0;
    const unsigned m = __ballot_sync(0xffffffffu, listed);
    if (lane == 0) s_wc[warp] = __popc(m);
    __syncthreads();
    if (warp == 0) {
      // exclusive prefix of the warps' counts, the block total, the block's base
      const int c = lane < kPreThreads / 32 ? s_wc[lane] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int tot = __shfl_sync(0xffffffffu, incl, 31);
      if (lane < kPreThreads / 32) s_wc[lane] = incl - c;
      int b = 0;
      if (scan_state) {
        b = (int)scan_exclusive(scan_state, round, 1, 0, (unsigned long long)tot, status);
        if (lane == 0 && tot) atomicAdd(p.vis_count_out, tot);
      } else if (lane == 0 && tot) {
        b = atomicAdd(p.vis_count_out, tot);
      }
      if (lane == 0) *s_base = b;
    }
    __syncthreads();
    uint32_t dest = 0u;
    if (listed) {
      const uint32_t slot = (uint32_t)(*s_base + s_wc[warp] + __popc(m & ((1u << lane) - 1u)));
      p.vis_list_out[slot] = (uint32_t)i;
      if (p.slot_of_out) p.slot_of_out[i] = slot;
      if (p.x_ranks) {
        // exchange record: conic+opacity | means2D | rgb | depth | radius bits | min scale
        float4* r4 = reinterpret_cast<float4*>(p.x_records + 12 * (int64_t)slot);
        r4[0] = res.conic_op;
        r4[1] = make_float4(res.pimg.x, res.pimg.y, res.rgb.x, res.rgb.y);
        r4[2] = make_float4(res.rgb.z, res.depth, __int_as_float(res.radius), res.smin);
        // destinations: the reference getTouchedIdsBool test on the square
        // tile rect (rasterize_points.cu:212-256) against each rank's rows
        int2 lo, hi;
        tile_rect_int(res.pimg, res.radius, p.grid_x, p.grid_y, lo, hi);
        const int tmin = lo.y * p.grid_x + lo.x;
        const int tmax = (hi.y - 1) * p.grid_x + hi.x - 1;
        if (tmax >= tmin)
          for (int r = 0; r < p.x_ranks; ++r)
            if (!(tmax < __ldg(p.x_tile_lo + r) || tmin >= __ldg(p.x_tile_hi + r))) dest |= 1u << r;
        p.x_mask[slot] = dest;
      }
    }
    if (p.x_ranks) {
      // per-destination row counts: one atomic per warp and rank
      for (int r = 0; r < p.x_ranks; ++r) {
        const unsigned b = __ballot_sync(0xffffffffu, (dest >> r) & 1u);
        if (lane == 0 && b) atomicAdd(p.x_counts + r, __popc(b));
      }
    }
    __syncthreads();  // s_wc / s_base are rewritten next round
  }
  if (valid) {
    store_one(p, i, res);
    if (p.counts_out) p.counts_out[i] = cnt;
  }
}

// One atomic per block and counter.
__device__ __forceinline__ void flush_totals(const PreprocessParams& p, FwdAcc acc) {
  __shared__ double s_rd[2][kPreThreads / 32];
  __shared__ unsigned long long s_rt[2][kPreThreads / 32];
  if (!p.reg_sums && !p.totals_out) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc.reg_v += __shfl_xor_sync(0xffffffffu, acc.reg_v, o);
    acc.reg_c += __shfl_xor_sync(0xffffffffu, acc.reg_c, o);
    acc.r += __shfl_xor_sync(0xffffffffu, acc.r, o);
    acc.n += __shfl_xor_sync(0xffffffffu, acc.n, o);
  }
  if (lane == 0) {
    s_rd[0][warp] = acc.reg_v;
    s_rd[1][warp] = acc.reg_c;
    s_rt[0][warp] = acc.r;
    s_rt[1][warp] = acc.n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double bv = 0.0, bc = 0.0;
    unsigned long long br = 0ull, bn = 0ull;
    for (int w = 0; w < kPreThreads / 32; ++w) {
      bv += s_rd[0][w];
      bc += s_rd[1][w];
      br += s_rt[0][w];
      bn += s_rt[1][w];
    }
    if (p.reg_sums && bc > 0) {
      atomicAdd(p.reg_sums + 0, bv);
      atomicAdd(p.reg_sums + 1, bc);
    }
    if (p.totals_out && (br | bn)) {
      atomicAdd(p.totals_out + 0, br);
      atomicAdd(p.totals_out + 1, bn);
    }
  }
}

__device__ __forceinline__ void load_camera(const PreprocessParams& p, float* Vs, float* Ps) {
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    Vs[k] = __ldg(p.viewmatrix + k);
    Ps[k] = __ldg(p.projmatrix + k);
  }
}

// Stage the compute_locally tile mask in shared memory when counts are asked
// for and it fits.  Returns whether it was staged (no barrier here).
__device__ __forceinline__ bool stage_mask(const PreprocessParams& p, bool* s_mask) {
  const int n_tiles = p.grid_x * p.grid_y;
  const bool use_smem = p.counts_out && p.compute_locally && n_tiles <= kPreMaskSmem;
  if (use_smem)
    for (int t = threadIdx.x; t < n_tiles; t += kPreThreads) s_mask[t] = p.compute_locally[t];
  return use_smem;
}

// Single-kernel form (no scratch): persistent blocks run phase A over chunks
// and phase B over the survivors queued in shared memory, a full block at a
// time.
__global__ void __launch_bounds__(kPreThreads, 2) preprocess_fwd_kernel(PreprocessParams p) {
  extern __shared__ bool s_mask[];  // n_tiles bytes when the tile mask is staged
  __shared__ uint32_t s_queue[kPreQueue];
  __shared__ int s_qn, s_base;
  __shared__ int s_wc[kPreThreads / 32];

  const int tid = threadIdx.x, lane = tid & 31;
  const bool use_smem = stage_mask(p, s_mask);
  if (tid == 0) s_qn = 0;
  float Vs[16], Ps[16];
  load_camera(p, Vs, Ps);
  const CullBound cb = make_cull_bound(p, Vs, Ps);
  FwdAcc acc;
  const int64_t n_chunks = (p.P + kPreChunk - 1) / kPreChunk;
  __syncthreads();

  for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
    const bool last = chunk + gridDim.x >= n_chunks;
    const int64_t base = chunk * kPreChunk + tid;
    bool keep[kPreUnroll];
    cull_phase(p, Vs, Ps, cb, base, keep);
#pragma unroll
    for (int u = 0; u < kPreUnroll; ++u) {
      const unsigned m = __ballot_sync(0xffffffffu, keep[u]);
      int wbase = 0;
      if (lane == 0 && m) wbase = atomicAdd(&s_qn, __popc(m));
      wbase = __shfl_sync(0xffffffffu, wbase, 0);
      if (keep[u]) s_queue[wbase + __popc(m & ((1u << lane) - 1u))] = (uint32_t)(base + u * kPreThreads);
    }
    __syncthreads();
    const int qn = s_qn;
    __syncthreads();  // everyone has read s_qn before anyone changes it
    if (qn < kPreThreads && !(last && qn > 0)) continue;

    const int n_proc = last ? qn : (qn / kPreThreads) * kPreThreads;
    for (int r0 = 0; r0 < n_proc; r0 += kPreThreads) {
      const bool valid = r0 + tid < n_proc;
      full_phase(p, Vs, Ps, cb, s_queue[valid ? r0 + tid : r0], valid, s_mask, use_smem, s_wc, &s_base, acc);
    }
    // carry the remainder (< kPreThreads entries) to the front of the queue;
    // sources sit at >= n_proc >= kPreThreads > destinations
    const int rem = qn - n_proc;
    const uint32_t carry = tid < rem ? s_queue[n_proc + tid] : 0u;
    __syncthreads();
    if (tid < rem) s_queue[tid] = carry;
    if (tid == 0) s_qn = rem;
    __syncthreads();
  }
  flush_totals(p, acc);
}

// Two-kernel form (caller scratch).  Phase A alone, at high occupancy: one
// chunk per block, chunks taken in ticket order; survivors are appended to
// the candidate list at the ordered prefix of the survivor counts of the
// chunks before (scan.cuh), so the list is in ascending index order.
template <bool ORDERED>
__global__ void __launch_bounds__(kPreThreads, 4) preprocess_cull_kernel(PreprocessParams p, uint32_t* cand,
                                                                          int* cand_count, int* ticket,
                                                                          unsigned long long* chunk_state,
                                                                          unsigned* status) {
  __shared__ int s_off[kPreUnroll][kPreThreads / 32];
  __shared__ int s_base, s_chunk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (ORDERED && tid == 0) s_chunk = atomicAdd(ticket, 1);
  float Vs[16], Ps[16];
  load_camera(p, Vs, Ps);
  const CullBound cb = make_cull_bound(p, Vs, Ps);
  if (ORDERED) __syncthreads();
  const int64_t chunk = ORDERED ? s_chunk : blockIdx.x;
  const int64_t base = chunk * kPreChunk + tid;
  bool keep[kPreUnroll];
  cull_phase(p, Vs, Ps, cb, base, keep);
  unsigned m[kPreUnroll];
#pragma unroll
  for (int u = 0; u < kPreUnroll; ++u) {
    m[u] = __ballot_sync(0xffffffffu, keep[u]);
    if (lane == 0) s_off[u][warp] = __popc(m[u]);
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive prefix over the (u, warp) counts in index order, two per lane
    static_assert(kPreUnroll * (kPreThreads / 32) == 64, "two (u, warp) counts per lane");
    int* flat = &s_off[0][0];
    const int c0 = flat[2 * lane], c1 = flat[2 * lane + 1];
    int incl = c0 + c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    flat[2 * lane] = incl - c0 - c1;
    flat[2 * lane + 1] = incl - c1;
    if (ORDERED) {
      const int b = (int)scan_exclusive(chunk_state, chunk, 1, 0, (unsigned long long)tot, status);
      if (lane == 0) {
        s_base = b;
        if (tot) atomicAdd(cand_count, tot);
      }
    } else if (lane == 0) {
      s_base = tot ? atomicAdd(cand_count, tot) : 0;
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kPreUnroll; ++u)
    if (keep[u]) cand[s_base + s_off[u][warp] + __popc(m[u] & ((1u << lane) - 1u))] = (uint32_t)(base + u * kPreThreads);
}

// Phase B over the candidate list: persistent blocks take rounds of
// kPreThreads candidates in ticket order; the visible list is written in
// candidate order (ordered prefix over the rounds, scan.cuh).
template <bool ORDERED>
__global__ void __launch_bounds__(kPreThreads, 2) preprocess_full_kernel(PreprocessParams p, const uint32_t* cand,
                                                                          const int* cand_count, int* ticket,
                                                                          unsigned long long* round_state,
                                                                          unsigned* status) {
  extern __shared__ bool s_mask[];
  __shared__ int s_base, s_round;
  __shared__ int s_wc[kPreThreads / 32];
  const int tid = threadIdx.x;
  const bool use_smem = stage_mask(p, s_mask);
  float Vs[16], Ps[16];
  load_camera(p, Vs, Ps);
  const CullBound cb = make_cull_bound(p, Vs, Ps);
  FwdAcc acc;
  const int n = *cand_count;
  const int n_rounds = (n + kPreThreads - 1) / kPreThreads;
  if (!ORDERED) __syncthreads();
  for (int k = 0;; ++k) {
    int round;
    if (ORDERED) {
      if (tid == 0) s_round = atomicAdd(ticket, 1);
      __syncthreads();
      round = s_round;
      __syncthreads();  // everyone has read s_round before it is rewritten
    } else {
      round = blockIdx.x + k * gridDim.x;
    }
    if (round >= n_rounds) break;
    const int r0 = round * kPreThreads;
    const bool valid = r0 + tid < n;
    full_phase(p, Vs, Ps, cb, cand[valid ? r0 + tid : r0], valid, s_mask, use_smem, s_wc, &s_base, acc, round,
               ORDERED ? round_state : nullptr, status);
  }
  flush_totals(p, acc);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
//
// Derived in matrix form, math convention (column vectors; R(q) the rotation
// of the quaternion q = (r, x, y, z); S = diag(mod * s)).  The forward chain of
// one Gaussian with centre m is
//   t = W m + w                      view-space centre (W the view rotation)
//   J = [ fx/tz  0      -fx cx/tz^2 ]   EWA Jacobian at the clamped centre,
//       [ 0      fy/tz  -fy cy/tz^2 ]   cx, cy = t.x, t.y clamped to +-1.3 tan(fov) tz
//   L = R(q) S,  Sigma = L L^T         3D covariance
//   T = J W,     A = T Sigma T^T + 0.3 I     2D covariance
//   Q = A^-1 (the conic),  p = ndc(P [m; 1]) the screen centre
//   c = max(0, sum_k B_k(d / |d|) f_k + 0.5),  d = m - campos  (SH colour)
// and reverse mode through it gives, for an upstream G_Q that is symmetric
// (its off-diagonal entry is the gradient of each of the two symmetric
// entries of Q),
//   G_A = -adj(A) G_Q adj(A) / (det(A)^2 + 1e-7)
//   G_Sigma = T^T G_A T,   G_T = 2 G_A T Sigma,   G_J = G_T W^T
//   dL/dt through the four non-zero entries of J,  dL/dm += W^T dL/dt
//   G_L = 2 G_Sigma L,  dL/ds_j = sum_i R_ij (G_L)_ij,  G_R = G_L S,
//   dL/dq = sum_ij (G_R)_ij dR_ij/dq
// The gradient conventions are the operator contract of the reference
// rasterizer (submodule/diff-gaussian-rasterization_f/cuda_rasterizer/
// backward.cu:146-400): the clamped cx, cy carry gradient to t.x, t.y only
// where the clamp is inactive and are held constant in tz; the scale gradient
// is the gradient with respect to mod * s (equal to the true one at mod = 1,
// the training value); the quaternion gradient is with respect to the
// quaternion the kernel was given; a clamped colour channel passes nothing.

// Row k of the 3x3 part of a column-major 4x4 M (math convention).
__device__ __forceinline__ float3 mat_row(const float* M, int k) { return make_float3(M[k], M[4 + k], M[8 + k]); }

__device__ __forceinline__ float dot3(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }

__device__ __forceinline__ float3 lin2(float a, float3 u, float b, float3 v) {
  return make_float3(a * u.x + b * v.x, a * u.y + b * v.y, a * u.z + b * v.z);
}

// Symmetric 3x3 matrix.
struct Sym3 {
  float xx, xy, xz, yy, yz, zz;
};

__device__ __forceinline__ float3 sym_mul(const Sym3& S, float3 v) {
  return make_float3(S.xx * v.x + S.xy * v.y + S.xz * v.z, S.xy * v.x + S.yy * v.y + S.yz * v.z,
                     S.xz * v.x + S.yz * v.y + S.zz * v.z);
}

template <bool ACC>
__device__ __forceinline__ void put(float* dst, float v) {
  if (ACC)
    *dst += v;
  else
    *dst = v;
}

// Per-Gaussian backward results, held in registers until the block stores them.
struct BwdOut {
  float mean[3];
  float scale[3];
  float4 rot;
  float op;
  float dc[3];
  float rest[45];
};

__device__ __forceinline__ void bwd_zero(BwdOut& o) {
#pragma unroll
  for (int k = 0; k < 3; ++k) o.mean[k] = o.scale[k] = o.dc[k] = 0.f;
  o.rot = make_float4(0.f, 0.f, 0.f, 0.f);
  o.op = 0.f;
#pragma unroll
  for (int k = 0; k < 45; ++k) o.rest[k] = 0.f;
}

// SH colour part: dL/d(coefficients) into out.dc / out.rest, and the
// gradient with respect to the unit view direction (returned).  Each basis
// function B_k of degree <= 3 enters with its value and its Cartesian
// gradient in (x, y, z); the coefficient gradient is B_k dL/dc and the
// direction gradient sums grad(B_k) (f_k . dL/dc).
__device__ __forceinline__ float3 sh_backward(int D, float3 u, const ShRegs& s, const float dR[3], BwdOut& out) {
  const float x = u.x, y = u.y, z = u.z;
  float3 g = make_float3(0.f, 0.f, 0.f);
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) out.dc[ch] = kSH0 * dR[ch];
  // coefficient k (1-based past DC) with basis value b and gradient (bx, by, bz)
  auto term = [&](int k, float b, float bx, float by, float bz) {
    const float* f = s.rest + 3 * (k - 1);
    float* o = out.rest + 3 * (k - 1);
    o[0] = b * dR[0];
    o[1] = b * dR[1];
    o[2] = b * dR[2];
    const float w = f[0] * dR[0] + f[1] * dR[1] + f[2] * dR[2];
    g.x += w * bx;
    g.y += w * by;
    g.z += w * bz;
  };
  if (D > 0) {
    term(1, -kSH1 * y, 0.f, -kSH1, 0.f);
    term(2, kSH1 * z, 0.f, 0.f, kSH1);
    term(3, -kSH1 * x, -kSH1, 0.f, 0.f);
    if (D > 1) {
      const float xx = x * x, yy = y * y, zz = z * z;
      term(4, kSH2[0] * x * y, kSH2[0] * y, kSH2[0] * x, 0.f);
      term(5, kSH2[1] * y * z, 0.f, kSH2[1] * z, kSH2[1] * y);
      term(6, kSH2[2] * (2.f * zz - xx - yy), -2.f * kSH2[2] * x, -2.f * kSH2[2] * y, 4.f * kSH2[2] * z);
      term(7, kSH2[3] * x * z, kSH2[3] * z, 0.f, kSH2[3] * x);
      term(8, kSH2[4] * (xx - yy), 2.f * kSH2[4] * x, -2.f * kSH2[4] * y, 0.f);
      if (D > 2) {
        term(9, kSH3[0] * y * (3.f * xx - yy), 6.f * kSH3[0] * x * y, 3.f * kSH3[0] * (xx - yy), 0.f);
        term(10, kSH3[1] * x * y * z, kSH3[1] * y * z, kSH3[1] * x * z, kSH3[1] * x * y);
        term(11, kSH3[2] * y * (4.f * zz - xx - yy), -2.f * kSH3[2] * x * y, kSH3[2] * (4.f * zz - xx - 3.f * yy),
             8.f * kSH3[2] * y * z);
        term(12, kSH3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy), -6.f * kSH3[3] * x * z, -6.f * kSH3[3] * y * z,
             kSH3[3] * (6.f * zz - 3.f * xx - 3.f * yy));
        term(13, kSH3[4] * x * (4.f * zz - xx - yy), kSH3[4] * (4.f * zz - 3.f * xx - yy), -2.f * kSH3[4] * x * y,
             8.f * kSH3[4] * x * z);
        term(14, kSH3[5] * z * (xx - yy), 2.f * kSH3[5] * x * z, -2.f * kSH3[5] * y * z, kSH3[5] * (xx - yy));
        term(15, kSH3[6] * x * (xx - 3.f * yy), 3.f * kSH3[6] * (xx - yy), -6.f * kSH3[6] * x * y, 0.f);
      }
    }
  }
  return g;
}

// Gradients of one visible Gaussian (radius > 0) given its upstream
// gradients gco (conic00, conic01, conic11, opacity).
// up = row of the upstream gradients (i, or the list position).
__device__ __forceinline__ void bwd_compute(const PreprocessBwdParams& p, int64_t i, int64_t up, float4 gco,
                                            BwdOut& out) {
  const PreprocessParams& f = p.f;
  float V[16], Pm[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    V[k] = __ldg(f.viewmatrix + k);
    Pm[k] = __ldg(f.projmatrix + k);
  }
  const float3 m = make_float3(__ldg(f.means3D + 3 * i + 0), __ldg(f.means3D + 3 * i + 1),
                               __ldg(f.means3D + 3 * i + 2));
  const Activated act = activate(f, i);
  const float sx = act.sx, sy = act.sy, sz = act.sz;
  const float qr = act.q.x, qx = act.q.y, qy = act.q.z, qz = act.q.w;

  // L = R(q) S; Sigma = L L^T
  const float Rm[3][3] = {{1.f - 2.f * (qy * qy + qz * qz), 2.f * (qx * qy - qr * qz), 2.f * (qx * qz + qr * qy)},
                          {2.f * (qx * qy + qr * qz), 1.f - 2.f * (qx * qx + qz * qz), 2.f * (qy * qz - qr * qx)},
                          {2.f * (qx * qz - qr * qy), 2.f * (qy * qz + qr * qx), 1.f - 2.f * (qx * qx + qy * qy)}};
  const float sm[3] = {f.scale_modifier * sx, f.scale_modifier * sy, f.scale_modifier * sz};
  float Lm[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int j = 0; j < 3; ++j) Lm[a][j] = Rm[a][j] * sm[j];
  Sym3 Sg;
  Sg.xx = Lm[0][0] * Lm[0][0] + Lm[0][1] * Lm[0][1] + Lm[0][2] * Lm[0][2];
  Sg.xy = Lm[0][0] * Lm[1][0] + Lm[0][1] * Lm[1][1] + Lm[0][2] * Lm[1][2];
  Sg.xz = Lm[0][0] * Lm[2][0] + Lm[0][1] * Lm[2][1] + Lm[0][2] * Lm[2][2];
  Sg.yy = Lm[1][0] * Lm[1][0] + Lm[1][1] * Lm[1][1] + Lm[1][2] * Lm[1][2];
  Sg.yz = Lm[1][0] * Lm[2][0] + Lm[1][1] * Lm[2][1] + Lm[1][2] * Lm[2][2];
  Sg.zz = Lm[2][0] * Lm[2][0] + Lm[2][1] * Lm[2][1] + Lm[2][2] * Lm[2][2];

  // view-space centre, clamp masks, Jacobian entries, T = J W
  const float3 t = xform_point3(m, V);
  const float limx = 1.3f * f.tanfovx, limy = 1.3f * f.tanfovy;
  const float ux = t.x / t.z, uy = t.y / t.z;
  const float free_x = (ux < -limx || ux > limx) ? 0.f : 1.f;
  const float free_y = (uy < -limy || uy > limy) ? 0.f : 1.f;
  const float cx = fminf(limx, fmaxf(-limx, ux)) * t.z;
  const float cy = fminf(limy, fmaxf(-limy, uy)) * t.z;
  const float iz = 1.f / t.z, iz2 = iz * iz;
  const float fx = f.focal_x, fy = f.focal_y;
  const float3 w0 = mat_row(V, 0), w1 = mat_row(V, 1), w2 = mat_row(V, 2);
  const float3 T0 = lin2(fx * iz, w0, -fx * cx * iz2, w2);
  const float3 T1 = lin2(fy * iz, w1, -fy * cy * iz2, w2);

  // A = T Sigma T^T + 0.3 I, with U = T Sigma
  const float3 U0 = sym_mul(Sg, T0), U1 = sym_mul(Sg, T1);
  const float a00 = dot3(U0, T0) + 0.3f, a01 = dot3(U0, T1), a11 = dot3(U1, T1) + 0.3f;

  // G_A = -adj(A) G_Q adj(A) / (det^2 + 1e-7); adj(A) = [a11 -a01; -a01 a00]
  const float q00 = gco.x, q01 = gco.y, q11 = gco.z;
  const float det = a00 * a11 - a01 * a01;
  const float inv = 1.f / (det * det + 1e-7f);
  float g00 = 0.f, g01 = 0.f, g11 = 0.f;
  if (inv != 0.f) {
    const float k00 = a11 * q00 - a01 * q01, k01 = a11 * q01 - a01 * q11;  // row 0 of adj(A) G_Q
    const float k10 = a00 * q01 - a01 * q00, k11 = a00 * q11 - a01 * q01;  // row 1
    g00 = -(k00 * a11 - k01 * a01) * inv;
    g01 = -(k01 * a00 - k00 * a01) * inv;
    g11 = -(k11 * a00 - k10 * a01) * inv;
  }

  // Y = G_A T (2x3); G_Sigma = T^T Y; G_T = 2 Y Sigma
  const float3 Y0 = lin2(g00, T0, g01, T1), Y1 = lin2(g01, T0, g11, T1);
  Sym3 GS;
  GS.xx = T0.x * Y0.x + T1.x * Y1.x;
  GS.xy = T0.x * Y0.y + T1.x * Y1.y;
  GS.xz = T0.x * Y0.z + T1.x * Y1.z;
  GS.yy = T0.y * Y0.y + T1.y * Y1.y;
  GS.yz = T0.y * Y0.z + T1.y * Y1.z;
  GS.zz = T0.z * Y0.z + T1.z * Y1.z;
  const float3 GT0 = sym_mul(Sg, Y0), GT1 = sym_mul(Sg, Y1);  // halves of the rows of G_T
  // the four live entries of G_J = G_T W^T
  const float gj00 = 2.f * dot3(GT0, w0), gj02 = 2.f * dot3(GT0, w2);
  const float gj11 = 2.f * dot3(GT1, w1), gj12 = 2.f * dot3(GT1, w2);
  const float dtx = free_x * -fx * iz2 * gj02;
  const float dty = free_y * -fy * iz2 * gj12;
  const float dtz = -iz2 * (fx * gj00 + fy * gj11) + 2.f * iz2 * iz * (fx * cx * gj02 + fy * cy * gj12);
  float3 dm = make_float3(dtx * w0.x + dty * w1.x + dtz * w2.x, dtx * w0.y + dty * w1.y + dtz * w2.y,
                          dtx * w0.z + dty * w1.z + dtz * w2.z);

  // screen centre: p = (h.x, h.y) / (h.w + 1e-7), upstream already in NDC units
  {
    const float* gm2 = p.g_means2D + up * p.g_means2D_stride;
    const float gx = gm2[0], gy = gm2[1];
    const float4 h = xform_point4(m, Pm);
    const float u = 1.0f / (h.w + 0.0000001f);
    const float v = (gx * h.x + gy * h.y) * u * u;
    const float3 px = mat_row(Pm, 0), py = mat_row(Pm, 1), pw = mat_row(Pm, 3);
    dm.x += u * (gx * px.x + gy * py.x) - v * pw.x;
    dm.y += u * (gx * px.y + gy * py.y) - v * pw.y;
    dm.z += u * (gx * px.z + gy * py.z) - v * pw.z;
  }

  // SH colour through the unit direction d / |d|
  {
    ShRegs s;
    load_sh(f, i, f.M, s);
    bool clamp3[3];
    (void)sh_to_rgb(f.D, m, f.campos, s.dc, s.rest, clamp3);
    const float* gc = p.g_colors + up * p.g_colors_stride;
    const float dR[3] = {clamp3[0] ? 0.f : gc[0], clamp3[1] ? 0.f : gc[1], clamp3[2] ? 0.f : gc[2]};
    const float3 d = make_float3(m.x - f.campos[0], m.y - f.campos[1], m.z - f.campos[2]);
    const float len = sqrtf(d.x * d.x + d.y * d.y + d.z * d.z);
    const float3 dir = make_float3(d.x / len, d.y / len, d.z / len);
    const float3 gu = sh_backward(f.D, dir, s, dR, out);
    // d(d/|d|)/dd = (I - dir dir^T) / |d|
    const float proj = dot3(dir, gu);
    dm.x += (gu.x - dir.x * proj) / len;
    dm.y += (gu.y - dir.y * proj) / len;
    dm.z += (gu.z - dir.z * proj) / len;
  }
  out.mean[0] = dm.x;
  out.mean[1] = dm.y;
  out.mean[2] = dm.z;

  // scale and quaternion: G_L = 2 G_Sigma L, G_R = G_L S
  {
    float GR[3][3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float3 gl = sym_mul(GS, make_float3(Lm[0][j], Lm[1][j], Lm[2][j]));  // column j of G_Sigma L
      out.scale[j] = 2.f * (Rm[0][j] * gl.x + Rm[1][j] * gl.y + Rm[2][j] * gl.z);
      GR[0][j] = 2.f * gl.x * sm[j];
      GR[1][j] = 2.f * gl.y * sm[j];
      GR[2][j] = 2.f * gl.z * sm[j];
    }
    // dR/dq for R(q) above, contracted with G_R
    const float s01 = GR[0][1] + GR[1][0], s02 = GR[0][2] + GR[2][0], s12 = GR[1][2] + GR[2][1];
    const float d10 = GR[1][0] - GR[0][1], d02 = GR[0][2] - GR[2][0], d21 = GR[2][1] - GR[1][2];
    out.rot.x = 2.f * (qz * d10 + qy * d02 + qx * d21);
    out.rot.y = 2.f * (qy * s01 + qz * s02 + qr * d21) - 4.f * qx * (GR[1][1] + GR[2][2]);
    out.rot.z = 2.f * (qx * s01 + qr * d02 + qz * s12) - 4.f * qy * (GR[0][0] + GR[2][2]);
    out.rot.w = 2.f * (qr * d10 + qx * s02 + qy * s12) - 4.f * qz * (GR[0][0] + GR[1][1]);
  }
  out.op = gco.w;
  if (f.raw) {
    // min-scale regulariser: d(loss)/d(min-axis scale) for Gaussians the
    // exchange sends (radius > 0 and a non-empty square tile rect)
    float gmin = 0.f;
    if (p.reg_scale && p.means2D) {
      const float2 m2 = reinterpret_cast<const float2*>(p.means2D)[i];
      int2 lo, hi;
      tile_rect_int(m2, __ldg(p.radii + i), f.grid_x, f.grid_y, lo, hi);
      if ((hi.y - 1) * f.grid_x + hi.x - 1 >= lo.y * f.grid_x + lo.x) gmin += *p.reg_scale;
    }
    // per-row gradient of the smallest scale (the multi-GPU step: summed over
    // the ranks that received this Gaussian)
    if (p.g_minscale) gmin += __ldg(p.g_minscale + up * p.g_minscale_stride);
    // to the first smallest axis (static indexing keeps `out` in registers)
    if (sx <= sy && sx <= sz)
      out.scale[0] += gmin;
    else if (sy <= sz)
      out.scale[1] += gmin;
    else
      out.scale[2] += gmin;
    // chain through the activations: exp, normalize (with its 1e-12 clamp), sigmoid
    out.scale[0] *= sx;
    out.scale[1] *= sy;
    out.scale[2] *= sz;
    const float4 g = out.rot, q = act.q;
    if (act.nrm > 1e-12f) {
      const float dot = q.x * g.x + q.y * g.y + q.z * g.z + q.w * g.w;
      out.rot = make_float4((g.x - q.x * dot) / act.nrm, (g.y - q.y * dot) / act.nrm, (g.z - q.z * dot) / act.nrm,
                            (g.w - q.w * dot) / act.nrm);
    } else {
      out.rot = make_float4(g.x / act.nrm, g.y / act.nrm, g.z / act.nrm, g.w / act.nrm);
    }
    out.op = gco.w * (1.f - act.o) * act.o;
  }
}

// Backward over a compact list of visible Gaussians (raw mode): every lane
// does useful work; gradients are added into pre-zeroed (or accumulating)
// outputs.
template <bool ACC>
__device__ __forceinline__ void list_one(const PreprocessBwdParams& p, const PreprocessParams& f, int64_t j) {
  const int64_t g = p.vis_list[j];
  const int64_t up = p.upstream_by_slot ? j : g;
  const float4 gco = *reinterpret_cast<const float4*>(p.g_conic_opacity + up * p.g_conic_stride);
  BwdOut o;
  bwd_zero(o);
  bwd_compute(p, g, up, gco, o);
  const int64_t i = p.out_by_slot ? j : g;  // output row
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    put<ACC>(p.g_means3D + 3 * i + k, o.mean[k]);
    put<ACC>(p.g_scales + 3 * i + k, o.scale[k]);
  }
  float4* r = reinterpret_cast<float4*>(p.g_rotations) + i;
  if (ACC) {
    float4 a = *r;
    a.x += o.rot.x;
    a.y += o.rot.y;
    a.z += o.rot.z;
    a.w += o.rot.w;
    *r = a;
  } else {
    *r = o.rot;
  }
  if (p.g_opacities) put<ACC>(p.g_opacities + i, o.op);
  float* gd = p.g_dc + i * p.g_dc_stride;
  float* gr = p.g_rest + i * p.g_rest_stride;
#pragma unroll
  for (int k = 0; k < 3; ++k) put<ACC>(gd + k, o.dc[k]);
#pragma unroll
  for (int k = 0; k < 45; ++k)
    if (k < f.M * 3) put<ACC>(gr + k, o.rest[k]);
}

template <bool ACC>
__global__ void __launch_bounds__(128) preprocess_bwd_list_kernel(PreprocessBwdParams p) {
  const PreprocessParams& f = p.f;
  const int64_t n = *p.vis_count;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    list_one<ACC>(p, f, j);
  }
}

constexpr int kBwdBlock = 128;

// Store one W-float row per thread of the block into the contiguous rows
// [base, base+n) of dst, staged through shared memory (odd pitch: no bank
// conflicts) so every warp store covers consecutive addresses.
template <int W, bool ACC>
__device__ __forceinline__ void store_rows(float* __restrict__ dst, int n, const float* row, float* stage) {
  constexpr int PITCH = W | 1;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < W; ++k) stage[threadIdx.x * PITCH + k] = row[k];
  __syncthreads();
  for (int e = threadIdx.x; e < n * W; e += kBwdBlock) {
    const int r = e / W, c = e - r * W;
    const float v = stage[r * PITCH + c];
    if (ACC)
      dst[e] += v;
    else
      dst[e] = v;
  }
}

template <bool ACC>
__global__ void __launch_bounds__(kBwdBlock) preprocess_bwd_kernel(PreprocessBwdParams p) {
  __shared__ float stage[kBwdBlock * 49];
  const PreprocessParams& f = p.f;
  const int64_t base = (int64_t)blockIdx.x * kBwdBlock;
  const int64_t i = base + threadIdx.x;
  const int n = (int)((f.P - base) < kBwdBlock ? (f.P - base) : kBwdBlock);
  const bool valid = i < f.P;

  float4 gco = make_float4(0.f, 0.f, 0.f, 0.f);
  bool vis = false;
  if (valid) {
    vis = __ldg(p.radii + i) > 0;
    gco = *reinterpret_cast<const float4*>(p.g_conic_opacity + i * p.g_conic_stride);
  }
  if (ACC && !__syncthreads_or(vis)) return;  // nothing to add in this block

  BwdOut o;
  bwd_zero(o);
  o.op = gco.w;  // the reference copies column 3 for every Gaussian
  if (vis) bwd_compute(p, i, i, gco, o);
  if (valid && p.g_opacities) put<ACC>(p.g_opacities + i, o.op);

  if (valid) {
    float4* r = reinterpret_cast<float4*>(p.g_rotations) + i;
    if (ACC) {
      float4 a = *r;
      a.x += o.rot.x;
      a.y += o.rot.y;
      a.z += o.rot.z;
      a.w += o.rot.w;
      *r = a;
    } else {
      *r = o.rot;
    }
  }
  store_rows<3, ACC>(p.g_means3D + 3 * base, n, o.mean, stage);
  store_rows<3, ACC>(p.g_scales + 3 * base, n, o.scale, stage);
  const bool packed = p.g_dc_stride == 48 && p.g_rest_stride == 48 && p.g_rest == p.g_dc + 3 && f.M == 15;
  if (packed) {
    float row[48];
#pragma unroll
    for (int k = 0; k < 3; ++k) row[k] = o.dc[k];
#pragma unroll
    for (int k = 0; k < 45; ++k) row[3 + k] = o.rest[k];
    store_rows<48, ACC>(p.g_dc + 48 * base, n, row, stage);
  } else if (p.g_dc_stride == 3 && p.g_rest_stride == 45 && f.M == 15) {
    store_rows<3, ACC>(p.g_dc + 3 * base, n, o.dc, stage);
    store_rows<45, ACC>(p.g_rest + 45 * base, n, o.rest, stage);
  } else if (valid) {
    float* gd = p.g_dc + i * p.g_dc_stride;
    float* gr = p.g_rest + i * p.g_rest_stride;
#pragma unroll
    for (int k = 0; k < 3; ++k) put<ACC>(gd + k, o.dc[k]);
#pragma unroll
    for (int k = 0; k < 45; ++k)
      if (k < f.M * 3) put<ACC>(gr + k, o.rest[k]);
  }
}

// Blocks of `kernel` that are resident on the current device at once (SMs x
// blocks per SM), for persistent grids.  Evaluated once per process: every
// device of a run is the same model.
template <typename K>
int resident_blocks(K kernel, int threads, size_t smem) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  return std::max(sms, 1) * std::max(per_sm, 1);
}

// Scratch of the two-kernel form: counters, the ordered-scan state of the
// cull chunks and of the full kernel's rounds, and the candidate list.
struct PreScratch {
  int* cand_count;
  int* cull_ticket;
  int* round_ticket;
  unsigned* status;  // scan.cuh status bits
  unsigned long long* chunk_state;
  unsigned long long* round_state;
  uint32_t* cand;
  size_t zero_bytes;  // bytes [256, zero_bytes) must be zero before the launch
};

static int64_t pre_chunks(int64_t P) { return (P + kPreChunk - 1) / kPreChunk; }
static int64_t pre_rounds(int64_t P) { return (P + kPreThreads - 1) / kPreThreads; }

static PreScratch pre_scratch_layout(void* base, int64_t P) {
  char* b = static_cast<char*>(base);
  PreScratch s;
  s.status = reinterpret_cast<unsigned*>(b + kPreStatusOffset);  // bytes [0, 256): never cleared here
  s.cand_count = reinterpret_cast<int*>(b + 256);
  s.cull_ticket = reinterpret_cast<int*>(b + 260);
  s.round_ticket = reinterpret_cast<int*>(b + 264);
  size_t off = 384;
  s.chunk_state = reinterpret_cast<unsigned long long*>(b + off);
  off += 8 * (size_t)std::max<int64_t>(pre_chunks(P), 1);
  s.round_state = reinterpret_cast<unsigned long long*>(b + off);
  off += 8 * (size_t)std::max<int64_t>(pre_rounds(P), 1);
  s.zero_bytes = off;
  s.cand = reinterpret_cast<uint32_t*>(b + off);
  return s;
}

size_t preprocess_scratch_bytes(int64_t P) {
  return pre_scratch_layout(nullptr, P).zero_bytes + sizeof(uint32_t) * (size_t)std::max<int64_t>(P, 1);
}

int launch_preprocess_fwd(const PreprocessParams& p, cudaStream_t st, void* scratch, size_t scratch_bytes,
                          int grid_share, unsigned* status) {
  if (p.totals_out) cudaMemsetAsync(p.totals_out, 0, 2 * sizeof(unsigned long long), st);
  if (p.P <= 0) return (int)cudaGetLastError();
  const int n_tiles = p.grid_x * p.grid_y;
  const size_t smem = (p.counts_out && p.compute_locally && n_tiles <= kPreMaskSmem) ? (size_t)n_tiles : 0;
  const int64_t n_chunks = pre_chunks(p.P);
  if (scratch && scratch_bytes >= preprocess_scratch_bytes(p.P)) {
    // cull pass over every Gaussian, then the full computation over the
    // candidates (persistent grid: the count is only known on the device)
    PreScratch s = pre_scratch_layout(scratch, p.P);
    if (status) s.status = status;
    static const int resident_full = resident_blocks(preprocess_full_kernel<false>, kPreThreads, kPreMaskSmem);
    // launches that run side by side (grid_share of them) split the device
    const int64_t blocks = std::min<int64_t>((p.P + kPreThreads - 1) / kPreThreads,
                                             std::max(resident_full / std::max(grid_share, 1), 1));
    if (p.ordered_list) {
      cudaMemsetAsync(static_cast<char*>(scratch) + 256, 0, s.zero_bytes - 256, st);
      preprocess_cull_kernel<true><<<(unsigned)n_chunks, kPreThreads, 0, st>>>(p, s.cand, s.cand_count, s.cull_ticket,
                                                                               s.chunk_state, s.status);
      preprocess_full_kernel<true><<<(unsigned)blocks, kPreThreads, smem, st>>>(p, s.cand, s.cand_count,
                                                                                s.round_ticket, s.round_state,
                                                                                s.status);
    } else {
      cudaMemsetAsync(s.cand_count, 0, sizeof(int), st);
      preprocess_cull_kernel<false><<<(unsigned)n_chunks, kPreThreads, 0, st>>>(p, s.cand, s.cand_count, nullptr,
                                                                                nullptr, s.status);
      preprocess_full_kernel<false><<<(unsigned)blocks, kPreThreads, smem, st>>>(p, s.cand, s.cand_count, nullptr,
                                                                                 nullptr, s.status);
    }
    return (int)cudaGetLastError();
  }
  // persistent grid: as many blocks as fit on the device at once
  static const int resident = resident_blocks(preprocess_fwd_kernel, kPreThreads, kPreMaskSmem);
  const int64_t blocks = std::min<int64_t>(n_chunks, resident);
  preprocess_fwd_kernel<<<(unsigned)blocks, kPreThreads, smem, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_preprocess_bwd(const PreprocessBwdParams& p, bool accumulate, cudaStream_t st) {
  if (p.f.P <= 0) return 0;
  if (p.vis_list) {
    // listed Gaussians only: add onto the outputs when accumulating, else
    // store (the caller zero-filled every row)
    // persistent grid-stride launch: the list length is only known on the
    // device, and one block per possible entry would be mostly empty blocks
    static const int res_acc = resident_blocks(preprocess_bwd_list_kernel<true>, 128, 0);
    static const int res_set = resident_blocks(preprocess_bwd_list_kernel<false>, 128, 0);
    const int64_t need = (p.f.P + 127) / 128;
    if (accumulate)
      preprocess_bwd_list_kernel<true><<<(unsigned)std::min<int64_t>(need, res_acc), 128, 0, st>>>(p);
    else
      preprocess_bwd_list_kernel<false><<<(unsigned)std::min<int64_t>(need, res_set), 128, 0, st>>>(p);
    return (int)cudaGetLastError();
  }
  const int threads = kBwdBlock;
  const int64_t blocks = (p.f.P + threads - 1) / threads;
  if (accumulate)
    preprocess_bwd_kernel<true><<<(unsigned)blocks, threads, 0, st>>>(p);
  else
    preprocess_bwd_kernel<false><<<(unsigned)blocks, threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
