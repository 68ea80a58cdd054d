// Shared device math for the BlitzGS B200 splatting path.
//
// Bit-exactness contract: the culling decision, integer radius, screen-space
// mean and view depth of every Gaussian must equal the reference rasterizer's
// bit for bit, because they decide tile rectangles and the per-tile depth
// order.  nvcc contracts a*b+c into FMA; two programs get the same bits only
// if they present the compiler the same expression shapes.  Every helper
// below therefore evaluates its formula in the same association order as the
// reference (submodule/diff-gaussian-rasterization_f/cuda_rasterizer/
// forward.cu:28-284 and auxiliary.h:43-194, which use glm's column-major
// mat3 product Result[c][r] = A[0][r]*B[c][0] + A[1][r]*B[c][1] + A[2][r]*B[c][2]),
// including multiplications by the structural zeros of the Jacobian, which
// the compiler may not fold without fast-math.  No fast-math flags are used.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace blitz {

constexpr int kTileX = 16;   // tile width in pixels (reference config.h BLOCK_X)
constexpr int kTileY = 16;   // tile height in pixels (reference config.h BLOCK_Y)
constexpr int kTilePix = kTileX * kTileY;

// Real spherical-harmonics basis constants for degrees 0..3 (standard values;
// the reference lists the same constants in auxiliary.h:21-38).
__device__ __constant__ static const float kSH0 = 0.28209479177387814f;
__device__ __constant__ static const float kSH1 = 0.4886025119029199f;
__device__ __constant__ static const float kSH2[5] = {
    1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
    -1.0925484305920792f, 0.5462742152960396f};
__device__ __constant__ static const float kSH3[7] = {
    -0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
    0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
    -0.5900435899266435f};

struct V3 {
  float x, y, z;
};

// Column-major 3x3 matrix: m[c][r] is column c, row r.
struct M3 {
  float m[3][3];
  __device__ __forceinline__ float* operator[](int c) { return m[c]; }
  __device__ __forceinline__ const float* operator[](int c) const { return m[c]; }
};

__device__ __forceinline__ M3 make_m3(float c00, float c01, float c02, float c10,
                                      float c11, float c12, float c20, float c21,
                                      float c22) {
  M3 r;
  r.m[0][0] = c00; r.m[0][1] = c01; r.m[0][2] = c02;
  r.m[1][0] = c10; r.m[1][1] = c11; r.m[1][2] = c12;
  r.m[2][0] = c20; r.m[2][1] = c21; r.m[2][2] = c22;
  return r;
}

__device__ __forceinline__ M3 m3_mul(const M3& a, const M3& b) {
  M3 r;
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int rr = 0; rr < 3; ++rr)
      r.m[c][rr] = a.m[0][rr] * b.m[c][0] + a.m[1][rr] * b.m[c][1] + a.m[2][rr] * b.m[c][2];
  return r;
}

__device__ __forceinline__ M3 m3_t(const M3& a) {
  M3 r;
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int rr = 0; rr < 3; ++rr) r.m[c][rr] = a.m[rr][c];
  return r;
}

// Affine transform by a 4x4 matrix stored column-major (row-vector convention
// of the camera tensors: world_view_transform and full_proj_transform).
__device__ __forceinline__ float3 xform_point3(const float3& p, const float* M) {
  return make_float3(M[0] * p.x + M[4] * p.y + M[8] * p.z + M[12],
                     M[1] * p.x + M[5] * p.y + M[9] * p.z + M[13],
                     M[2] * p.x + M[6] * p.y + M[10] * p.z + M[14]);
}

__device__ __forceinline__ float4 xform_point4(const float3& p, const float* M) {
  return make_float4(M[0] * p.x + M[4] * p.y + M[8] * p.z + M[12],
                     M[1] * p.x + M[5] * p.y + M[9] * p.z + M[13],
                     M[2] * p.x + M[6] * p.y + M[10] * p.z + M[14],
                     M[3] * p.x + M[7] * p.y + M[11] * p.z + M[15]);
}

__device__ __forceinline__ float3 xform_vec_t(const float3& p, const float* M) {
  return make_float3(M[0] * p.x + M[1] * p.y + M[2] * p.z,
                     M[4] * p.x + M[5] * p.y + M[6] * p.z,
                     M[8] * p.x + M[9] * p.y + M[10] * p.z);
}

// NDC -> pixel.  The reference evaluates this in double precision (double
// literals in auxiliary.h:43-46) and rounds the result to float once.
__device__ __forceinline__ float ndc_to_pix(float v, int S) {
  return ((v + 1.0) * S - 1.0) * 0.5;
}

// Square tile rectangle used by binning, routing and touch counting: integer
// radius, truncating division (reference auxiliary.h:48-58).
__device__ __forceinline__ void tile_rect_int(float2 p, int radius, int gx, int gy,
                                              int2& rmin, int2& rmax) {
  rmin.x = min(gx, max(0, (int)((p.x - radius) / kTileX)));
  rmin.y = min(gy, max(0, (int)((p.y - radius) / kTileY)));
  rmax.x = min(gx, max(0, (int)((p.x + radius + kTileX - 1) / kTileX)));
  rmax.y = min(gy, max(0, (int)((p.y + radius + kTileY - 1) / kTileY)));
}

// Axis-aligned rectangle used only by the preprocess "touches any tile"
// cull: float half-extents, floor/ceil (reference auxiliary.h:60-70).
__device__ __forceinline__ int tile_rect_f_count(float2 p, float2 e, int gx, int gy) {
  int x0 = min(gx, max(0, (int)floorf((p.x - e.x) / kTileX)));
  int y0 = min(gy, max(0, (int)floorf((p.y - e.y) / kTileY)));
  int x1 = min(gx, max(0, (int)ceilf((p.x + e.x) / kTileX)));
  int y1 = min(gy, max(0, (int)ceilf((p.y + e.y) / kTileY)));
  return (x1 - x0) * (y1 - y0);
}

// power = -0.5 (c00 dx^2 + c11 dy^2) - c01 dx dy, rounded as the reference
// kernel rounds it: nvcc fuses the first product of each sum into an FMA when
// every product has one use,
//   sum = fma(c00 dx, dx, (c11 dy) dy),  power = fma(-0.5, sum, -(c01 dx) dy).
// Spelled out so that the rounding cannot change with the code around it (a
// product shared between two uses would be fused the other way round).  The
// forward and the backward both call this, so their skip decisions agree bit
// for bit.
__device__ __forceinline__ float pair_power(float4 co, float2 d) {
  const float sum = __fmaf_rn(__fmul_rn(co.x, d.x), d.x, __fmul_rn(__fmul_rn(co.z, d.y), d.y));
  return __fmaf_rn(-0.5f, sum, -__fmul_rn(__fmul_rn(co.y, d.x), d.y));
}

// The same rectangle as tile bounds [rmin, rmax).
__device__ __forceinline__ void tile_rect_f(float2 p, float2 e, int gx, int gy, int2& rmin, int2& rmax) {
  rmin.x = min(gx, max(0, (int)floorf((p.x - e.x) / kTileX)));
  rmin.y = min(gy, max(0, (int)floorf((p.y - e.y) / kTileY)));
  rmax.x = min(gx, max(0, (int)ceilf((p.x + e.x) / kTileX)));
  rmax.y = min(gy, max(0, (int)ceilf((p.y + e.y) / kTileY)));
}

// Exact tile test of the full rasterizer: does Gaussian (mean m, conic and
// opacity co) reach alpha >= 1/255 anywhere on tile (tx, ty)?  thr is
// ln(255 * opacity).  The exponent factor 0.5 d^T conic d is evaluated at
// one point of the tile's pixel-centre rectangle: the mean itself when it
// lies inside (factor 0), else the corner on the mean's side moved along the
// rectangle's edges towards the minimiser of the factor on each edge line,
// clamped to the edge (the method of rasterizer_impl.cu:52-97; the same
// float operations in the same order, with the products fused into FMAs the
// way nvcc fuses that expression, so the emitted tile set is bit-identical).
__device__ __forceinline__ bool tile_reached(float4 co, float2 m, float thr, int tx, int ty) {
  constexpr float kSpanX = (float)(kTileX - 1), kSpanY = (float)(kTileY - 1);
  const float x0 = (float)(tx * kTileX), x1 = (float)((tx + 1) * kTileX - 1);
  const float y0 = (float)(ty * kTileY), y1 = (float)((ty + 1) * kTileY - 1);
  const float gap_x = x0 - m.x, gap_y = y0 - m.y;  // > 0: the mean lies before the tile
  const bool before_x = gap_x > 0.f, before_y = gap_y > 0.f;
  const bool out_x = before_x || m.x > x1, out_y = before_y || m.y > y1;
  if (!out_x && !out_y) return 0.f <= thr;
  const float cx = before_x ? x0 : x1, cy = before_y ? y0 : y1;  // starting corner
  const float sx = copysignf(kSpanX, gap_x), sy = copysignf(kSpanY, gap_y);  // edge vectors from it
  const float ex = m.x - cx, ey = m.y - cy;
  // position along each edge (0..1) of the factor's minimum on that edge line
  const float rx = __frcp_rn(__fmul_rn(kSpanX * kSpanX, co.x));
  const float ry = __frcp_rn(__fmul_rn(kSpanY * kSpanY, co.z));
  const float ux = __saturatef(__fmul_rn(__fmaf_rn(__fmul_rn(sx, co.x), ex, __fmul_rn(__fmul_rn(sx, co.y), ey)), rx));
  const float uy = __saturatef(__fmul_rn(__fmaf_rn(__fmul_rn(sy, co.y), ex, __fmul_rn(__fmul_rn(sy, co.z), ey)), ry));
  const float qx = __fmaf_rn(out_y ? ux : 0.f, sx, cx);
  const float qy = __fmaf_rn(out_x ? uy : 0.f, sy, cy);
  const float dx = m.x - qx, dy = m.y - qy;
  const float f = __fmaf_rn(0.5f, __fmaf_rn(__fmul_rn(co.x, dx), dx, __fmul_rn(__fmul_rn(co.z, dy), dy)),
                            __fmul_rn(__fmul_rn(co.y, dx), dy));
  return f <= thr;
}

// ln(255 * opacity) as the full rasterizer's binning computes it.
__device__ __forceinline__ float tile_reach_threshold(float opacity) {
  return logf(__fdiv_rn(opacity, 1.0f / 255.0f));
}

// 3D covariance (upper triangle) from scale and an (unnormalised) quaternion
// (r, x, y, z): Sigma = (S R)^T (S R).  The reference normalises the
// quaternion in PyTorch before the kernel, not inside it (forward.cu:136).
__device__ __forceinline__ void cov3d_from_scale_rot(float sx, float sy, float sz, float mod,
                                                     float4 q, float* cov) {
  M3 S = make_m3(1.f, 0.f, 0.f, 0.f, 1.f, 0.f, 0.f, 0.f, 1.f);
  S.m[0][0] = mod * sx;
  S.m[1][1] = mod * sy;
  S.m[2][2] = mod * sz;
  const float r = q.x, x = q.y, y = q.z, z = q.w;
  M3 R = make_m3(1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y),
                 2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x),
                 2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y));
  M3 M = m3_mul(S, R);
  M3 Sig = m3_mul(m3_t(M), M);
  cov[0] = Sig.m[0][0];
  cov[1] = Sig.m[0][1];
  cov[2] = Sig.m[0][2];
  cov[3] = Sig.m[1][1];
  cov[4] = Sig.m[1][2];
  cov[5] = Sig.m[2][2];
}

// EWA projection of a 3D covariance to the 2D screen covariance (with the
// +0.3 px^2 low-pass), following Zwicker et al. 2002 eq. 29/31 with the
// +-1.3 tan(fov) clamp of the view-space position.
__device__ __forceinline__ float3 cov2d_ewa(const float3& mean, float fx, float fy, float tanx,
                                            float tany, const float* cov3d, const float* V) {
  float3 t = xform_point3(mean, V);
  const float limx = 1.3f * tanx;
  const float limy = 1.3f * tany;
  const float txtz = t.x / t.z;
  const float tytz = t.y / t.z;
  t.x = min(limx, max(-limx, txtz)) * t.z;
  t.y = min(limy, max(-limy, tytz)) * t.z;
  M3 J = make_m3(fx / t.z, 0.0f, -(fx * t.x) / (t.z * t.z), 0.0f, fy / t.z,
                 -(fy * t.y) / (t.z * t.z), 0, 0, 0);
  M3 W = make_m3(V[0], V[4], V[8], V[1], V[5], V[9], V[2], V[6], V[10]);
  M3 T = m3_mul(W, J);
  M3 Vrk = make_m3(cov3d[0], cov3d[1], cov3d[2], cov3d[1], cov3d[3], cov3d[4], cov3d[2],
                   cov3d[4], cov3d[5]);
  M3 cov = m3_mul(m3_mul(m3_t(T), m3_t(Vrk)), T);
  cov.m[0][0] += 0.3f;
  cov.m[1][1] += 0.3f;
  return make_float3(cov.m[0][0], cov.m[0][1], cov.m[1][1]);
}

// View-dependent colour from degree-<=3 SH: dc is the 3-float DC term, sh the
// 15x3 higher-order terms.  Adds the +0.5 offset and reports per-channel
// clamping at zero.
struct ShIn {
  const float* dc;   // 3 floats
  const float* sh;   // M*3 floats (M = coefficients beyond DC)
};

__device__ __forceinline__ V3 sh_to_rgb(int deg, const float3& pos, const float* campos,
                                        const float* dc, const float* sh, bool* clamp3) {
  V3 dir = {pos.x - campos[0], pos.y - campos[1], pos.z - campos[2]};
  // glm::length(v) = sqrt(dot(v, v)); dot = v.x*v.x + v.y*v.y + v.z*v.z
  float len = sqrtf(dir.x * dir.x + dir.y * dir.y + dir.z * dir.z);
  dir.x = dir.x / len;
  dir.y = dir.y / len;
  dir.z = dir.z / len;
  V3 res = {kSH0 * dc[0], kSH0 * dc[1], kSH0 * dc[2]};
  if (deg > 0) {
    const float x = dir.x, y = dir.y, z = dir.z;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float v = (&res.x)[c];
      v = v - kSH1 * y * sh[0 * 3 + c] + kSH1 * z * sh[1 * 3 + c] - kSH1 * x * sh[2 * 3 + c];
      (&res.x)[c] = v;
    }
    if (deg > 1) {
      const float xx = x * x, yy = y * y, zz = z * z;
      const float xy = x * y, yz = y * z, xz = x * z;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        float v = (&res.x)[c];
        v = v + kSH2[0] * xy * sh[3 * 3 + c] + kSH2[1] * yz * sh[4 * 3 + c] +
            kSH2[2] * (2.0f * zz - xx - yy) * sh[5 * 3 + c] + kSH2[3] * xz * sh[6 * 3 + c] +
            kSH2[4] * (xx - yy) * sh[7 * 3 + c];
        (&res.x)[c] = v;
      }
      if (deg > 2) {
#pragma unroll
        for (int c = 0; c < 3; ++c) {
          float v = (&res.x)[c];
          v = v + kSH3[0] * y * (3.0f * xx - yy) * sh[8 * 3 + c] +
              kSH3[1] * xy * z * sh[9 * 3 + c] +
              kSH3[2] * y * (4.0f * zz - xx - yy) * sh[10 * 3 + c] +
              kSH3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy) * sh[11 * 3 + c] +
              kSH3[4] * x * (4.0f * zz - xx - yy) * sh[12 * 3 + c] +
              kSH3[5] * z * (xx - yy) * sh[13 * 3 + c] +
              kSH3[6] * x * (xx - 3.0f * yy) * sh[14 * 3 + c];
          (&res.x)[c] = v;
        }
      }
    }
  }
  res.x += 0.5f;
  res.y += 0.5f;
  res.z += 0.5f;
  clamp3[0] = res.x < 0;
  clamp3[1] = res.y < 0;
  clamp3[2] = res.z < 0;
  res.x = fmaxf(res.x, 0.0f);
  res.y = fmaxf(res.y, 0.0f);
  res.z = fmaxf(res.z, 0.0f);
  return res;
}

__device__ __forceinline__ uint32_t float_bits(float f) { return __float_as_uint(f); }

}  // namespace blitz
