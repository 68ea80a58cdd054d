// Eval-side kernels of the full (non-distributed) rasterizer:
//   mark_visible   -- GaussianRasterizer.markVisible (_C.mark_visible,
//                     rasterizer_impl.cu:100-114, 257-268);
//   depth render   -- rasterize_gaussians_depth (forward.cu:614-845).
// The colour forward, rasterize_gaussians_simp and flag_max_count run on the
// training blend (blend.cu, its STATS variant) over the full rasterizer's
// tile lists (binning.cu with rects).
#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

__global__ void __launch_bounds__(256) mark_visible_kernel(int64_t P, const float* __restrict__ means3D,
                                                           const float* __restrict__ viewmatrix,
                                                           bool* __restrict__ present) {
  __shared__ float Vs[16];
  if (threadIdx.x < 16) Vs[threadIdx.x] = viewmatrix[threadIdx.x];
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float3 x = make_float3(means3D[3 * i], means3D[3 * i + 1], means3D[3 * i + 2]);
  present[i] = xform_point3(x, Vs).z > 0.2f;
}

// Inverse of a column-major 4x4 matrix by cofactors (2x2 minors of the two
// row pairs), in float as the reference computes its inverse: the matrix is
// ill-conditioned in its depth row (znear 0.01), so a more accurate inverse
// would move every ray away from the reference's by ~7e-4 relative.  A
// singular matrix yields non-finite entries, as any inverse.
__device__ void invert4(const float* mf, float* inv) {
  auto at = [&](int r, int c) { return mf[c * 4 + r]; };
  // minors of rows (0,1) and rows (2,3), columns (i,j)
  const float s0 = at(0, 0) * at(1, 1) - at(1, 0) * at(0, 1);
  const float s1 = at(0, 0) * at(1, 2) - at(1, 0) * at(0, 2);
  const float s2 = at(0, 0) * at(1, 3) - at(1, 0) * at(0, 3);
  const float s3 = at(0, 1) * at(1, 2) - at(1, 1) * at(0, 2);
  const float s4 = at(0, 1) * at(1, 3) - at(1, 1) * at(0, 3);
  const float s5 = at(0, 2) * at(1, 3) - at(1, 2) * at(0, 3);
  const float c5 = at(2, 2) * at(3, 3) - at(3, 2) * at(2, 3);
  const float c4 = at(2, 1) * at(3, 3) - at(3, 1) * at(2, 3);
  const float c3 = at(2, 1) * at(3, 2) - at(3, 1) * at(2, 2);
  const float c2 = at(2, 0) * at(3, 3) - at(3, 0) * at(2, 3);
  const float c1 = at(2, 0) * at(3, 2) - at(3, 0) * at(2, 2);
  const float c0 = at(2, 0) * at(3, 1) - at(3, 0) * at(2, 1);
  const float det = s0 * c5 - s1 * c4 + s2 * c3 + s3 * c2 - s4 * c1 + s5 * c0;
  const float id = 1.0f / det;
  float r[4][4];  // r[row][col] of the inverse
  r[0][0] = (at(1, 1) * c5 - at(1, 2) * c4 + at(1, 3) * c3) * id;
  r[0][1] = (-at(0, 1) * c5 + at(0, 2) * c4 - at(0, 3) * c3) * id;
  r[0][2] = (at(3, 1) * s5 - at(3, 2) * s4 + at(3, 3) * s3) * id;
  r[0][3] = (-at(2, 1) * s5 + at(2, 2) * s4 - at(2, 3) * s3) * id;
  r[1][0] = (-at(1, 0) * c5 + at(1, 2) * c2 - at(1, 3) * c1) * id;
  r[1][1] = (at(0, 0) * c5 - at(0, 2) * c2 + at(0, 3) * c1) * id;
  r[1][2] = (-at(3, 0) * s5 + at(3, 2) * s2 - at(3, 3) * s1) * id;
  r[1][3] = (at(2, 0) * s5 - at(2, 2) * s2 + at(2, 3) * s1) * id;
  r[2][0] = (at(1, 0) * c4 - at(1, 1) * c2 + at(1, 3) * c0) * id;
  r[2][1] = (-at(0, 0) * c4 + at(0, 1) * c2 - at(0, 3) * c0) * id;
  r[2][2] = (at(3, 0) * s4 - at(3, 1) * s2 + at(3, 3) * s0) * id;
  r[2][3] = (-at(2, 0) * s4 + at(2, 1) * s2 - at(2, 3) * s0) * id;
  r[3][0] = (-at(1, 0) * c3 + at(1, 1) * c1 - at(1, 2) * c0) * id;
  r[3][1] = (at(0, 0) * c3 - at(0, 1) * c1 + at(0, 2) * c0) * id;
  r[3][2] = (-at(3, 0) * s3 + at(3, 1) * s1 - at(3, 2) * s0) * id;
  r[3][3] = (at(2, 0) * s3 - at(2, 1) * s1 + at(2, 2) * s0) * id;
  for (int c = 0; c < 4; ++c)
    for (int rr = 0; rr < 4; ++rr) inv[c * 4 + rr] = r[rr][c];
}

constexpr int kDepthBatch = kTilePix;

// One CTA per tile, one thread per pixel; the tile's list is walked front to
// back in batches of kDepthBatch Gaussians staged in shared memory.
//
// Per pixel the ray runs from the camera centre through the point the
// inverse projection maps the pixel's NDC position (z = 99/99.99, the far
// end of znear 0.01 / zfar 100) to; as in the reference, the homogeneous w
// of that point is not divided out.  For each blended Gaussian the ray is
// intersected with its 3-sigma ellipsoid (rotation and scales as given):
// a t^2 + b t + c = 0 in the Gaussian's frame, t* = -b / 2a the closest
// approach, depth = t* / |ray|.  The colour blend is the usual one, with one
// difference kept from the reference: a Gaussian whose depth is negative
// still adds its colour, but neither attenuates T nor competes for the
// largest weight.
__global__ void __launch_bounds__(kTilePix) depth_render_kernel(DepthParams p) {
  __shared__ float s_inv[16];
  __shared__ int s_id[kDepthBatch];
  __shared__ float4 s_co[kDepthBatch];
  __shared__ float2 s_xy[kDepthBatch];
  // per Gaussian, for the ray-ellipsoid test: the world -> Gaussian rotation
  // (9), 1/(3 s)^2 per axis (3), the camera centre in the Gaussian frame
  // scaled by 1/(3 s)^2 (3) and the constant term c of the quadratic (1).
  // All of it depends on the Gaussian and the camera only, not the pixel.
  __shared__ float s_g[kDepthBatch][16];
  const int tile = blockIdx.x;
  const int tx = tile % p.grid_x, ty = tile / p.grid_x;
  const int px = tx * kTileX + (threadIdx.x % kTileX), py = ty * kTileY + (threadIdx.x / kTileX);
  const bool inside = px < p.W && py < p.H;
  if (threadIdx.x == 0) invert4(p.projmatrix, s_inv);
  __syncthreads();

  const float2 pixf = make_float2((float)px, (float)py);
  const float3 o = make_float3(p.campos[0], p.campos[1], p.campos[2]);
  // pixel -> NDC -> (non-divided) world point on the far plane
  const float nx = (float)((double)((2 * pixf.x + 1) / p.W - 1) * 1.0000001);
  const float ny = (float)((double)((2 * pixf.y + 1) / p.H - 1) * 1.0000001);
  const float nz = (float)((100.0 - 100.0 * 0.01) / (100.0 - 0.01));
  const float4 far_pt = xform_point4(make_float3(nx, ny, nz), s_inv);
  const float3 ray = make_float3(far_pt.x - o.x, far_pt.y - o.y, far_pt.z - o.z);
  const float ray_len = sqrtf(ray.x * ray.x + ray.y * ray.y + ray.z * ray.z);
  const float inv_len = 1.0f / ray_len;
  const float3 u = make_float3(ray.x * inv_len, ray.y * inv_len, ray.z * inv_len);

  const uint2 range = p.ranges[tile];
  const int n = (int)(range.y - range.x);
  bool done = !inside;
  float T = 1.f, C0 = 0.f, C1 = 0.f, C2 = 0.f;
  float w_max = 0.f, depth_max = 0.f, disc_max = 0.f;
  int id_max = 0;
  float3 hit = make_float3(0.f, 0.f, 0.f);

  for (int base = 0; base < n; base += kDepthBatch) {
    if (__syncthreads_count(done) == kTilePix) break;
    const int k = base + threadIdx.x;
    if (k < n) {
      const int id = (int)p.point_list[range.x + k];
      s_id[threadIdx.x] = id;
      s_xy[threadIdx.x] = reinterpret_cast<const float2*>(p.means2D)[id];
      s_co[threadIdx.x] = reinterpret_cast<const float4*>(p.conic_opacity)[id];
      float* g = s_g[threadIdx.x];
      const float4 q = reinterpret_cast<const float4*>(p.rotations)[id];
      const float qr = q.x, qx = q.y, qy = q.z, qz = q.w;
      // the transpose of the rotation built from q (quaternion as given)
      const float R[9] = {1.f - 2.f * (qy * qy + qz * qz), 2.f * (qx * qy + qr * qz), 2.f * (qx * qz - qr * qy),
                          2.f * (qx * qy - qr * qz), 1.f - 2.f * (qx * qx + qz * qz), 2.f * (qy * qz + qr * qx),
                          2.f * (qx * qz + qr * qy), 2.f * (qy * qz - qr * qx), 1.f - 2.f * (qx * qx + qy * qy)};
      const float v[3] = {o.x - p.means3D[3 * (int64_t)id + 0], o.y - p.means3D[3 * (int64_t)id + 1],
                          o.z - p.means3D[3 * (int64_t)id + 2]};
      float c = -1.f;
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const float s3 = p.scales[3 * (int64_t)id + r] * 3.0f;
        const float is2 = 1.0f / (s3 * s3);
        const float ro = R[3 * r] * v[0] + R[3 * r + 1] * v[1] + R[3 * r + 2] * v[2];  // rotated origin
        g[r * 3 + 0] = R[3 * r];
        g[r * 3 + 1] = R[3 * r + 1];
        g[r * 3 + 2] = R[3 * r + 2];
        g[9 + r] = is2;
        g[12 + r] = ro * is2;
        c += ro * ro * is2;
      }
      g[15] = c;
    }
    __syncthreads();
    const int cnt = min(kDepthBatch, n - base);
    for (int j = 0; !done && j < cnt; ++j) {
      const float2 xy = s_xy[j];
      const float4 co = s_co[j];
      const float2 d = make_float2(xy.x - pixf.x, xy.y - pixf.y);
      const float power = pair_power(co, d);
      if (power > 0.0f) continue;
      const float alpha = fminf(0.99f, co.w * expf(power));
      if (alpha < 1.0f / 255.0f) continue;
      const float test_T = T * (1 - alpha);
      if (test_T < 0.0001f) {
        done = true;
        continue;
      }
      const int id = s_id[j];
      C0 += p.rgb[3 * (int64_t)id + 0] * alpha * T;
      C1 += p.rgb[3 * (int64_t)id + 1] * alpha * T;
      C2 += p.rgb[3 * (int64_t)id + 2] * alpha * T;
      const float* g = s_g[j];
      const float w[3] = {u.x, u.y, u.z};
      float a = 0.f, bh = 0.f;  // a t^2 + 2 bh t + c: the ray in the Gaussian's 3-sigma frame
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const float rd = g[3 * r] * w[0] + g[3 * r + 1] * w[1] + g[3 * r + 2] * w[2];  // rotated direction
        a += rd * rd * g[9 + r];
        bh += rd * g[12 + r];
      }
      const float b = 2 * bh, c = g[15];
      const float t_star = -b / 2 / a;
      const float depth = t_star / ray_len;
      if (depth < 0) continue;
      if (w_max < alpha * T) {
        w_max = alpha * T;
        depth_max = depth;
        disc_max = b * b - 4 * a * c;
        id_max = id;
        hit = make_float3(o.x + t_star * u.x, o.y + t_star * u.y, o.z + t_star * u.z);
      }
      T = test_T;
    }
  }
  if (inside) {
    const int64_t HW = (int64_t)p.H * p.W, pix = (int64_t)p.W * py + px;
    p.out_color[pix] = C0 + T * p.bg[0];
    p.out_color[HW + pix] = C1 + T * p.bg[1];
    p.out_color[2 * HW + pix] = C2 + T * p.bg[2];
    p.out_pts[pix] = hit.x;
    p.out_pts[HW + pix] = hit.y;
    p.out_pts[2 * HW + pix] = hit.z;
    p.out_depth[pix] = depth_max;
    p.accum_alpha[pix] = T;
    p.discriminants[pix] = disc_max;
    p.gidx[pix] = id_max;
  }
}

}  // namespace

int launch_depth_render(const DepthParams& p, cudaStream_t st) {
  const int n_tiles = p.grid_x * p.grid_y;
  if (n_tiles <= 0) return 0;
  depth_render_kernel<<<n_tiles, kTilePix, 0, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_mark_visible(int64_t P, const float* means3D, const float* viewmatrix, bool* present, cudaStream_t st) {
  if (P <= 0) return 0;
  mark_visible_kernel<<<(unsigned)((P + 255) / 256), 256, 0, st>>>(P, means3D, viewmatrix, present);
  return (int)cudaGetLastError();
}

}  // namespace blitz
