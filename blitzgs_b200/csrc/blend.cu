// Per-tile alpha blending, forward and backward.
//
// Forward semantics follow the reference renderCUDA
// (submodule/diff-gaussian-rasterization_r/cuda_rasterizer/forward.cu:263-413):
// one pixel per thread, front-to-back over the tile's depth-sorted list;
//   power = -0.5 (c00 dx^2 + c11 dy^2) - c01 dx dy   (skip if > 0)
//   alpha = min(0.99, o exp(power))                   (skip if < 1/255)
//   stop before the Gaussian that would take T below 1e-4.
// The per-pair arithmetic is written in the reference's expression order so
// that skip/stop decisions and n_contrib match bit for bit.
//
// Work decomposition (B200-side; no output bit changes in the forward):
//   * the unit of work is a warp strip: 8x4 pixels of a 16x16 tile.  Each
//     warp walks its tile's list on its own, 32 entries at a time: lane i
//     loads entry i, tests a conservative bounding box of the Gaussian's
//     alpha >= 1/255 region against the strip's 32 pixel centres, and the
//     survivors are compacted (ballot + popc) into the warp's shared-memory
//     batch.  About half of the (strip, Gaussian) pairs of a tile list miss
//     the strip and never enter the per-pixel loop, and no warp waits at a
//     block barrier for the tile's slowest warp;
//   * the forward stops a warp as soon as its 32 pixels are saturated;
//     the backward starts each warp at its own largest n_contrib;
//   * the forward can record, per strip, the Gaussians that contributed to
//     at least one of its pixels (ids and list positions, in list order);
//     the backward then replays only those -- the same pairs in the same
//     order -- instead of walking and box-testing the whole tile list (22%
//     off the backward for 3% on the forward);
//   * the list walk is software-pipelined: list entries are loaded two
//     batches ahead and the Gaussians' position and conic one batch ahead,
//     so the dependent L2 loads of a batch overlap the previous batch's
//     pixel loop (8% off the forward);
//   * a per-Gaussian log-domain threshold rejects, before the exp, every pair
//     whose alpha is provably below 1/255 (margin 1e-3 in the exponent, far
//     above the few-ulp error of logf/expf), so most pairs cost ~8 FP32
//     instructions instead of ~30;
//   * colours are staged with the geometry instead of being re-read from
//     global memory for every (pixel, Gaussian) pair;
//   * out_observe counts are kept per lane as a bitmask over the batch and
//     reduced over the warp once per batch, then flushed with one atomic per
//     (warp, Gaussian);
//   * the per-tile statistics (n_render, n_consider, n_contrib) are reduced
//     in the epilogue instead of three extra kernels.
// Strip shape: 8x4 pixels overlap ~18% fewer ~12-pixel splats than 16x2.
// Tried and slower: 16x2 strips (13% slower forward, 19% slower backward);
// a tile-wide staging round shared by the 8 warps (23% slower forward, 35%
// slower backward than 8x4 strips); two pixels per
// thread (fewer instructions, but the occupancy loss cost more), a per-warp
// box test inside the pair loop, a guarded __expf in the backward, and a
// forward register cap for five CTAs per SM (48 registers, with small
// spills: 2-4% slower than four CTAs at 61).
//
// Backward follows the reference back-to-front replay (backward.cu:324-530)
// but replaces the 11 global atomics per (pixel, Gaussian) pair with a
// warp-level transpose reduction (13 shuffles for the 11 values) and one
// 11-lane RED instruction per (warp, Gaussian) -- or, when at most
// kDirectLanes pixels of the warp contribute, their own REDs.  T is
// recovered with one reciprocal of (1 - alpha) (fast division, 1 - alpha in
// [0.01, 1)) shared by the two divisions of the reference; the gradients
// differ from IEEE division by ~1e-7 relative.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

// Backward: a (warp, Gaussian) pair with at most this many contributing
// pixels adds their gradients with per-lane REDs instead of the reduction.
constexpr int kDirectLanes = 8;
// A warp strip: the kStripW x kStripH pixels of one warp (lane l: column
// l % kStripW, row l / kStripW); kStrips per tile, strip s at column
// s % kStripsX and row s / kStripsX of the tile's strip grid.
constexpr int kStripW = 8;
constexpr int kStripH = 4;
constexpr int kStripsX = kTileX / kStripW;
constexpr int kStrips = kStripsX * (kTileY / kStripH);
static_assert(kStripW * kStripH == 32, "a strip is one warp of pixels");

// Pixel of this lane in strip s of tile (tx, ty).
__device__ __forceinline__ int2 strip_pixel(int tx, int ty, int s, int lane) {
  return make_int2(tx * kTileX + (s % kStripsX) * kStripW + lane % kStripW,
                   ty * kTileY + (s / kStripsX) * kStripH + lane / kStripW);
}

// Top-left pixel of strip s of tile (tx, ty).
__device__ __forceinline__ float2 strip_origin(int tx, int ty, int s) {
  return make_float2((float)(tx * kTileX + (s % kStripsX) * kStripW), (float)(ty * kTileY + (s / kStripsX) * kStripH));
}

// exp-skip threshold: for power < thr, o*expf(power) < (1/255) * e^-1e-3.
__device__ __forceinline__ float skip_threshold(float o) {
  if (o > 0.f) return logf(1.0f / (255.0f * o)) - 1e-3f;
  if (o <= 0.f) return __int_as_float(0x7f800000);  // +inf: never contributes
  return __int_as_float(0xff800000);                  // NaN opacity: never pre-skip
}

// Conservative bounding box of the pixels where this Gaussian can reach
// alpha >= 1/255: the ellipse d^T C d <= 2 ln(255 o) (C = conic), inflated
// for the float error of the per-pixel power (more for ill-conditioned
// conics, whose terms cancel).  An empty box (xmin > xmax) means no pixel
// can pass; degenerate conics and NaN opacities get an infinite box (never
// culled).  Every (pixel, Gaussian) pair outside the box is skipped by the
// per-pixel test too, so skipping them wholesale changes no output.
__device__ __forceinline__ float4 alpha_box(float2 xy, float4 co) {
  const float inf = __int_as_float(0x7f800000);
  const float o = co.w;
  if (o < 1.0f / 255.0f) return make_float4(inf, -inf, inf, -inf);  // o * G <= o < 1/255 everywhere
  const float det = co.x * co.z - co.y * co.y;
  if (!(o >= 1.0f / 255.0f) || !(co.x > 0.f && co.z > 0.f && det > 0.f)) return make_float4(-inf, inf, -inf, inf);
  const float k = co.x * co.z / det;  // >= 1; large when the terms of the quadratic form cancel
  const float r2 = 2.f * logf(255.f * o) * (1.002f + 1e-5f * k) + 1e-3f;
  const float hx = sqrtf(r2 * co.z / det) + 0.01f;
  const float hy = sqrtf(r2 * co.x / det) + 0.01f;
  if (!(hx < 1e30f && hy < 1e30f)) return make_float4(-inf, inf, -inf, inf);
  return make_float4(xy.x - hx, xy.x + hx, xy.y - hy, xy.y + hy);
}

// Does the box miss the pixel centres [x0, x1] x [y0, y1]?
__device__ __forceinline__ bool box_misses(float4 b, float x0, float x1, float y0, float y1) {
  return b.y < x0 || b.x > x1 || b.w < y0 || b.z > y1;
}

__device__ __forceinline__ int block_sum_int(int v, int* s_red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  int t = 0;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

template <bool STATS>
__global__ void __launch_bounds__(kTilePix) blend_fwd_kernel(BlendFwdParams p) {
  const int tile = blockIdx.x;
  const int tx = tile % p.grid_x, ty = tile / p.grid_x;
  const int2 pxy = strip_pixel(tx, ty, threadIdx.x >> 5, threadIdx.x & 31);
  const int px = pxy.x, py = pxy.y;
  const bool inside = px < p.W && py < p.H;
  const int64_t HW = (int64_t)p.H * p.W;
  const int64_t pix = (int64_t)p.W * py + px;

  const bool local = p.compute_locally ? p.compute_locally[tile] : true;
  if (!local) {
    if (inside) {
      p.out_color[pix] = 0.f;
      p.out_color[HW + pix] = 0.f;
      p.out_color[2 * HW + pix] = 0.f;
      p.final_T[pix] = 1.f;
      p.n_contrib[pix] = 0u;
    }
    if (threadIdx.x == 0 && p.n_render) {
      p.n_render[tile] = 0;
      p.n_consider[tile] = 0;
      p.n_contrib_tile[tile] = 0;
    }
    if (p.strip_counts && threadIdx.x < kStrips) p.strip_counts[(int64_t)tile * kStrips + threadIdx.x] = 0;
    return;
  }

  // Warp w (strip w of the tile) walks the tile's list on its own, 32
  // entries at a time, keeps the Gaussians whose alpha box reaches its
  // pixels, and stops as soon as its 32 pixels are saturated.
  constexpr int kWarps = kTilePix / 32;
  __shared__ float4 s_a[kWarps][32];
  __shared__ float4 s_b[kWarps][32];
  __shared__ float4 s_c[kWarps][32];
  __shared__ int s_id[kWarps][32];
  __shared__ int s_red[32];
  __shared__ float s_w[STATS ? kWarps : 1][32];  // STATS: blend weights and counts per batch entry
  __shared__ int s_n[STATS ? kWarps : 1][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float2 so = strip_origin(tx, ty, warp);

  const uint2 range = p.ranges[tile];
  const int n = (int)(range.y - range.x);
  const float2 pixf = make_float2((float)px, (float)py);

  int* strip_ids = nullptr;
  int* strip_pos = nullptr;
  int n_act = 0;
  if (p.strip_ids) {
    const int64_t off = (int64_t)kStrips * range.x + (int64_t)warp * n;
    strip_ids = p.strip_ids + off;
    strip_pos = p.strip_pos + off;
  }

  bool done = !inside;
  float T = 1.0f;
  uint32_t last_contributor = 0, n2l = 0;
  float C0 = 0.f, C1 = 0.f, C2 = 0.f;
  float w_max = 0.f;  // STATS: largest blending weight so far and its Gaussian
  int id_max = -1;

  // software pipeline: list ids two batches ahead, Gaussian data one batch ahead
  int id_n = 0, id_nn = 0;
  float2 xy_n = make_float2(0.f, 0.f);
  float4 co_n = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane < n) {
    id_n = (int)p.point_list[range.x + lane];
    xy_n = reinterpret_cast<const float2*>(p.means2D)[id_n];
    co_n = reinterpret_cast<const float4*>(p.conic_opacity)[id_n];
  }
  if (lane + 32 < n) id_nn = (int)p.point_list[range.x + lane + 32];
  for (int base = 0; base < n; base += 32) {
    if (__all_sync(0xffffffffu, done)) break;
    const int k = base + lane;
    const int id = id_n;
    const float2 xy = xy_n;
    const float4 co = co_n;
    id_n = id_nn;
    if (k + 32 < n) {
      xy_n = reinterpret_cast<const float2*>(p.means2D)[id_n];
      co_n = reinterpret_cast<const float4*>(p.conic_opacity)[id_n];
    }
    if (k + 64 < n) id_nn = (int)p.point_list[range.x + k + 64];
    const bool keep =
        k < n && !box_misses(alpha_box(xy, co), so.x, so.x + (float)(kStripW - 1), so.y, so.y + (float)(kStripH - 1));
    const unsigned km = __ballot_sync(0xffffffffu, keep);
    if (!km) continue;
    if (keep) {
      const int slot = __popc(km & ((1u << lane) - 1u));
      s_id[warp][slot] = id;
      s_a[warp][slot] = make_float4(xy.x, xy.y, co.x, co.y);
      // 1-based list position, as the reference counts it
      s_b[warp][slot] = make_float4(co.z, co.w, skip_threshold(co.w), __int_as_float(k + 1));
      s_c[warp][slot] = make_float4(p.rgb[3 * (int64_t)id + 0], p.rgb[3 * (int64_t)id + 1],
                                    p.rgb[3 * (int64_t)id + 2], 0.f);
      if (STATS) {
        s_w[warp][slot] = 0.f;
        s_n[warp][slot] = 0;
      }
    }
    __syncwarp();
    const int kept = __popc(km);
    // per lane, bit j: this pixel blended batch entry j (act) while T > 0.5 (obs);
    // reduced over the warp after the loop instead of shared-memory atomics
    // that all lanes would aim at the same word
    unsigned act_bits = 0u, obs_bits = 0u;
    for (int j = 0; !done && j < kept; ++j) {
      const float4 ga = s_a[warp][j];
      const float4 gb = s_b[warp][j];
      const float2 d = {ga.x - pixf.x, ga.y - pixf.y};
      const float4 con_o = make_float4(ga.z, ga.w, gb.x, gb.y);
      const float power = pair_power(con_o, d);
      if (power < gb.z) continue;  // alpha provably < 1/255
      if (power > 0.0f) continue;
      const float alpha = min(0.99f, con_o.w * expf(power));
      if (alpha < 1.0f / 255.0f) continue;
      const float test_T = T * (1 - alpha);
      if (test_T < 0.0001f) {
        done = true;
        continue;
      }
      ++n2l;
      act_bits |= 1u << j;
      const float4 cth = s_c[warp][j];
      const float w = alpha * T;  // blending weight
      C0 += cth.x * w;
      C1 += cth.y * w;
      C2 += cth.z * w;
      if (STATS) {
        if (w_max < w) {
          w_max = w;
          id_max = s_id[warp][j];
        }
        if (p.accum_w) {
          atomicAdd(&s_w[warp][j], w);
          atomicAdd(&s_n[warp][j], 1);
        }
      } else if (T > 0.5) {
        obs_bits |= 1u << j;
      }
      T = test_T;
      last_contributor = (uint32_t)__float_as_int(gb.w);
    }
    __syncwarp();
    if (STATS) {
      if (p.accum_w && lane < kept && s_n[warp][lane] > 0) {
        atomicAdd(&p.accum_w[s_id[warp][lane]], s_w[warp][lane]);
        atomicAdd(&p.accum_n[s_id[warp][lane]], s_n[warp][lane]);
      }
    } else {
      // observation count of entry j = lanes with bit j; lane j flushes it
      unsigned todo = __reduce_or_sync(0xffffffffu, obs_bits);
      int my_obs = 0;
      while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1u;
        const int c = __popc(__ballot_sync(0xffffffffu, (obs_bits >> j) & 1u));
        if (lane == j) my_obs = c;
      }
      if (my_obs) atomicAdd(&p.out_observe[s_id[warp][lane]], my_obs);
    }
    if (strip_ids) {
      // append this batch's contributing Gaussians to the strip's list, in order
      const bool a = ((__reduce_or_sync(0xffffffffu, act_bits) >> lane) & 1u) != 0;
      const unsigned am = __ballot_sync(0xffffffffu, a);
      if (a) {
        const int at = n_act + __popc(am & ((1u << lane) - 1u));
        strip_ids[at] = s_id[warp][lane];
        strip_pos[at] = __float_as_int(s_b[warp][lane].w) - 1;  // 0-based list position
      }
      n_act += __popc(am);
    }
    __syncwarp();
  }
  if (strip_ids && lane == 0) p.strip_counts[(int64_t)tile * kStrips + warp] = n_act;

  if (inside) {
    p.final_T[pix] = T;
    p.n_contrib[pix] = last_contributor;
    p.out_color[pix] = C0 + T * p.bg[0];
    p.out_color[HW + pix] = C1 + T * p.bg[1];
    p.out_color[2 * HW + pix] = C2 + T * p.bg[2];
  }
  if (STATS) {
    if (p.max_count && id_max >= 0) atomicAdd(&p.max_count[id_max], 1.f);
    if (!p.n_render) return;  // (uniform across the block)
  }
  const int s1 = block_sum_int(inside ? (int)last_contributor : 0, s_red);
  if (threadIdx.x == 0) p.n_consider[tile] = s1;
  const int s2 = block_sum_int(inside ? (int)n2l : 0, s_red);
  if (threadIdx.x == 0) {
    p.n_contrib_tile[tile] = s2;
    p.n_render[tile] = n;
  }
}

// Position of reduced value m (0..10) in the 16-float per-Gaussian gradient
// record: [m.x m.y 0 0 | a.x a.y 0 0 | c00 c01 c11 op | r g b 0].
__constant__ int kSlot[11] = {0, 1, 4, 5, 8, 9, 10, 11, 12, 13, 14};

// Sum 11 per-lane values over the warp in 13 shuffles.  Each step halves the
// values a lane keeps, swapping half with the partner lane (an odd one out is
// summed by both partners), so lane L ends with the warp total of value
// reduce11_value(L).  Step xor 16: values 0-4 | 5-9, value 10 by both;
// xor 8: the first three of the five (with 10) | the last two and 10;
// xor 4: first | second, the third by both; xor 2: the pair | the third;
// xor 1: both.
__device__ __forceinline__ float warp_transpose_reduce11(const float v[11]) {
  const int lane = threadIdx.x & 31;
  float a[6];
  {
    const bool b = lane & 16;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const float send = b ? v[i] : v[5 + i];
      const float keep = b ? v[5 + i] : v[i];
      a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    a[5] = v[10] + __shfl_xor_sync(0xffffffffu, v[10], 16);
  }
  float c[3];
  {
    const bool b = lane & 8;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float send = b ? a[i] : a[3 + i];
      const float keep = b ? a[3 + i] : a[i];
      c[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  float e0, e1;
  {
    const bool b = lane & 4;
    const float send = b ? c[0] : c[1];
    const float keep = b ? c[1] : c[0];
    e0 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    e1 = c[2] + __shfl_xor_sync(0xffffffffu, c[2], 4);
  }
  float g;
  {
    const bool b = lane & 2;
    const float send = b ? e0 : e1;
    const float keep = b ? e1 : e0;
    g = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return g + __shfl_xor_sync(0xffffffffu, g, 1);
}

// The value whose total lane L holds after warp_transpose_reduce11, or -1
// where another lane holds the same total (one writer per value).
__device__ __forceinline__ int reduce11_value(int lane) {
  if (lane & 1) return -1;
  const int half = 5 * ((lane >> 4) & 1), hi = (lane >> 3) & 1, odd = (lane >> 2) & 1;
  if (lane & 2) {
    if (odd) return -1;
    if (hi) return half ? -1 : 10;
    return half + 2;
  }
  return half + 3 * hi + odd;
}

// Backward, one warp per CTA: CTA tile * kStrips + s replays strip s of the
// tile.  Each warp walks its tile's list back to front from its own largest
// n_contrib, 32 list entries at a time: lane i loads entry i, tests the
// Gaussian's alpha >= 1/255 box against the strip's pixels, and the
// survivors are compacted into the warp's shared-memory batch.  No block
// barrier: warps of a tile never wait for one another.
//
// With LISTS (the forward recorded, per strip, the Gaussians that contributed
// to at least one of its pixels: strip_ids / strip_pos, strip_counts) the
// warp walks only that list, back to front: the same (pixel, Gaussian) pairs
// in the same order, without the box tests and without the iterations in
// which no pixel of the strip contributes.
template <bool LISTS>
__device__ __forceinline__ void blend_bwd_strip(const BlendBwdParams& p, int gstrip, float4* s_a, float4* s_b,
                                                float4* s_c, int* s_id) {
  const int tile = gstrip / kStrips;
  const int strip = gstrip - tile * kStrips;
  if (p.compute_locally && !p.compute_locally[tile]) return;
  const int tx = tile % p.grid_x, ty = tile / p.grid_x;
  const int lane = threadIdx.x;
  const int2 pxy = strip_pixel(tx, ty, strip, lane);
  const int px = pxy.x, py = pxy.y;
  const bool inside = px < p.W && py < p.H;
  const int64_t HW = (int64_t)p.H * p.W;
  const int64_t pix = (int64_t)p.W * py + px;
  const float2 pixf = make_float2((float)px, (float)py);

  const float2 so = strip_origin(tx, ty, strip);

  const uint2 range = p.ranges[tile];
  const float T_final = inside ? p.final_T[pix] : 0.f;
  float T = T_final;
  const int last_contributor = inside ? (int)p.n_contrib[pix] : 0;
  float dpx[3] = {0.f, 0.f, 0.f};
  if (inside) {
    dpx[0] = p.dL_dpix[pix];
    dpx[1] = p.dL_dpix[HW + pix];
    dpx[2] = p.dL_dpix[2 * HW + pix];
  }
  const float bg_dot = p.bg[0] * dpx[0] + p.bg[1] * dpx[1] + p.bg[2] * dpx[2];

  // only list positions below the strip's largest n_contrib can contribute
  int n_eff = last_contributor;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n_eff = max(n_eff, __shfl_xor_sync(0xffffffffu, n_eff, o));

  // The pair loop sums the gradient values without their constant factors;
  // each total is scaled once: d(pixel)/d(ndc) = W/2, H/2 and the signs of
  // the mean gradients, -1/2 of the conic gradients.
  const float ddelx_dx = 0.5 * p.W;
  const float ddely_dy = 0.5 * p.H;
  const float kScale[11] = {-ddelx_dx, -ddely_dy, ddelx_dx, ddely_dy, -0.5f, -0.5f, -0.5f, 1.f, 1.f, 1.f, 1.f};
  // record slot and scale of the total this lane writes after the warp
  // reduction (slot -1: none)
  const int red_value = reduce11_value(lane);
  const int red_slot = red_value >= 0 ? kSlot[red_value] : -1;
  float red_scale = 1.f;
#pragma unroll
  for (int m = 0; m < 11; ++m) red_scale = red_value == m ? kScale[m] : red_scale;
  // The reference keeps the colour accumulated behind the current Gaussian
  // per channel and forms sum_ch (colour - accum) * dL/dpix; only the dot
  // product with dL/dpix is used, so it is carried as one scalar
  // (acc_d = sum_ch accum_ch * dL/dpix_ch, same linear recurrence).
  float acc_d = 0.f;
  float last_alpha = 0.f;
  float last_cd = 0.f;
  const float neg_bg = -T_final * bg_dot;  // background term of dL/dalpha, times 1/(1 - alpha)

  // software pipeline: list entries two batches ahead, Gaussian data one
  // batch ahead.  Walk mode: entries of the tile list from the strip's
  // largest n_contrib down; list mode: entries of the strip's recorded list.
  const int n_tile = (int)(range.y - range.x);
  const int* lst_id = nullptr;
  const int* lst_pos = nullptr;
  int n_walk = n_eff;
  if constexpr (LISTS) {
    const int64_t off = (int64_t)kStrips * range.x + (int64_t)strip * n_tile;
    lst_id = p.strip_ids + off;
    lst_pos = p.strip_pos + off;
    n_walk = p.strip_counts[(int64_t)tile * kStrips + strip];
  }
  auto entry = [&](int e, int& id, int& pos) {  // e-th entry of the walk, back to front
    if constexpr (LISTS) {
      id = __ldg(lst_id + e);
      pos = __ldg(lst_pos + e);
    } else {
      id = (int)p.point_list[range.x + e];
      pos = e;
    }
  };
  int id_n = 0, id_nn = 0, pos_n = 0, pos_nn = 0;
  float2 xy_n = make_float2(0.f, 0.f);
  float4 co_n = make_float4(0.f, 0.f, 0.f, 0.f);
  {
    const int e0 = n_walk - 1 - lane, e1 = e0 - 32;
    if (e0 >= 0) entry(e0, id_n, pos_n);
    if (e1 >= 0) entry(e1, id_nn, pos_nn);
    if (e0 >= 0) {
      xy_n = reinterpret_cast<const float2*>(p.means2D)[id_n];
      co_n = reinterpret_cast<const float4*>(p.conic_opacity)[id_n];
    }
  }
  for (int base = 0; base < n_walk; base += 32) {
    const int e = n_walk - 1 - (base + lane);  // walk entry, back to front
    const int id = id_n, k = pos_n;            // k: list position
    const float2 xy = xy_n;
    const float4 co = co_n;
    id_n = id_nn;
    pos_n = pos_nn;
    if (e - 32 >= 0) {
      xy_n = reinterpret_cast<const float2*>(p.means2D)[id_n];
      co_n = reinterpret_cast<const float4*>(p.conic_opacity)[id_n];
    }
    if (e - 64 >= 0) entry(e - 64, id_nn, pos_nn);
    bool keep = e >= 0;
    if constexpr (!LISTS)
      keep = keep && !box_misses(alpha_box(xy, co), so.x, so.x + (float)(kStripW - 1), so.y,
                                 so.y + (float)(kStripH - 1));
    const unsigned km = __ballot_sync(0xffffffffu, keep);
    if (!km) continue;
    __syncwarp();  // the previous batch is no longer read
    if (keep) {
      const int slot = __popc(km & ((1u << lane) - 1u));
      s_id[slot] = p.record_rows ? (int)__ldg(p.record_rows + id) : id;  // gradient record row
      s_a[slot] = make_float4(xy.x, xy.y, co.x, co.y);
      s_b[slot] = make_float4(co.z, co.w, skip_threshold(co.w), __int_as_float(k));  // list position
      s_c[slot] = make_float4(p.rgb[3 * (int64_t)id + 0], p.rgb[3 * (int64_t)id + 1], p.rgb[3 * (int64_t)id + 2],
                              0.f);
    }
    __syncwarp();
    const int kept = __popc(km);
    for (int j = 0; j < kept; ++j) {
      const float4 gb = s_b[j];
      const int pos = __float_as_int(gb.w);
      float g[11];
      bool contrib = false;
      if (pos < last_contributor) {
        const float4 ga = s_a[j];
        const float2 d = {ga.x - pixf.x, ga.y - pixf.y};
        const float4 con_o = make_float4(ga.z, ga.w, gb.x, gb.y);
        const float power = pair_power(con_o, d);
        if (power >= gb.z && !(power > 0.0f)) {
          const float4 cth = s_c[j];
          const float G = expf(power);
          const float alpha = min(0.99f, con_o.w * G);
          if (!(alpha < 1.0f / 255.0f)) {
            contrib = true;
            const float inv1ma = __fdividef(1.0f, 1.f - alpha);  // 1 - alpha in [0.01, 1)
            T = T * inv1ma;
            const float dchannel_dcolor = alpha * T;
            const float cd = cth.x * dpx[0] + cth.y * dpx[1] + cth.z * dpx[2];
            acc_d = fmaf(last_alpha, last_cd - acc_d, acc_d);
            last_alpha = alpha;
            last_cd = cd;
            const float dL_dalpha = (cd - acc_d) * T + neg_bg * inv1ma;
            const float dL_dG = con_o.w * dL_dalpha;
            const float gdx = G * d.x;
            const float gdy = G * d.y;
            g[0] = dL_dG * (gdx * con_o.x + gdy * con_o.y);  // x -W/2
            g[1] = dL_dG * (gdy * con_o.z + gdx * con_o.y);  // x -H/2
            g[2] = fabsf(g[0]);
            g[3] = fabsf(g[1]);
            const float gdx_dG = gdx * dL_dG;
            g[4] = gdx_dG * d.x;  // x -1/2
            g[5] = gdx_dG * d.y;
            g[6] = gdy * dL_dG * d.y;
            g[7] = G * dL_dalpha;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) g[8 + ch] = dchannel_dcolor * dpx[ch];
          }
        }
      }
      const unsigned cm = __ballot_sync(0xffffffffu, contrib);
      if (!cm) continue;
      if (__popc(cm) <= kDirectLanes) {
        // few contributing pixels: their own REDs cost fewer instructions
        // than the warp-wide transpose reduction
        if (contrib) {
          float* dst = p.grad_accum + 16 * (int64_t)s_id[j];
#pragma unroll
          for (int m = 0; m < 11; ++m) atomicAdd(dst + kSlot[m], g[m] * kScale[m]);
        }
        continue;
      }
      if (!contrib) {
#pragma unroll
        for (int m = 0; m < 11; ++m) g[m] = 0.f;
      }
      // value order for the reduction: m.x m.y |m.x| |m.y| c00 c01 c11 op r g b
      const float tot = warp_transpose_reduce11(g) * red_scale;
      if (red_slot >= 0 && tot != 0.f) atomicAdd(p.grad_accum + 16 * (int64_t)s_id[j] + red_slot, tot);
    }
  }
}

// One warp per CTA, CTA g replays strip g (tile g / kStrips).  (Persistent
// one-warp CTAs looping over the strips, with static or ticketed strip
// assignment, measured 45-55% slower on the city workload.)
template <bool LISTS>
__global__ void __launch_bounds__(32, 32) blend_bwd_kernel(BlendBwdParams p, int n_strips) {
  __shared__ float4 s_a[32];
  __shared__ float4 s_b[32];
  __shared__ float4 s_c[32];
  __shared__ int s_id[32];
  (void)n_strips;
  blend_bwd_strip<LISTS>(p, blockIdx.x, s_a, s_b, s_c, s_id);
}


}  // namespace

int launch_blend_fwd(const BlendFwdParams& p, cudaStream_t st) {
  const int n_tiles = p.grid_x * p.grid_y;
  if (n_tiles <= 0) return 0;
  if (p.max_count || p.accum_w)
    blend_fwd_kernel<true><<<n_tiles, kTilePix, 0, st>>>(p);
  else
    blend_fwd_kernel<false><<<n_tiles, kTilePix, 0, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_blend_bwd(const BlendBwdParams& p, cudaStream_t st) {
  const int n_tiles = p.grid_x * p.grid_y;
  if (n_tiles <= 0) return 0;
  const int n_strips = n_tiles * kStrips;
  if (p.strip_ids)
    blend_bwd_kernel<true><<<n_strips, 32, 0, st>>>(p, n_strips);
  else
    blend_bwd_kernel<false><<<n_strips, 32, 0, st>>>(p, n_strips);
  return (int)cudaGetLastError();
}

}  // namespace blitz
