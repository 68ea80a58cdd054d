// Routing mask: which image-row partitions (ranks) a Gaussian's square tile
// rect overlaps.
//
// Semantics are those of the reference getTouchedIdsBool
// (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:212-256,
// called through DivisionStrategyFinal.get_local2j_ids,
// gaussian_renderer/workload_division.py:682-704): the rect is flattened to
// the tile-id interval [min.y*gx + min.x, (max.y-1)*gx + max.x - 1] and tested
// against each rank's [dist[r], dist[r+1]) interval of tile ids (optionally
// widened by gx+1 on both sides).  An empty interval sends nothing.  The
// output is the dense bool [P, world_size] matrix the reference returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "scan.cuh"

namespace blitz {

namespace {

__global__ void __launch_bounds__(256) route_bool_kernel(RouteParams p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.P) return;
  bool* out = p.out_bool + i * p.world_size;
  const float2 m = reinterpret_cast<const float2*>(p.means2D)[i];
  int2 lo, hi;
  tile_rect_int(m, p.radii[i], p.grid_x, p.grid_y, lo, hi);
  const int tmin = lo.y * p.grid_x + lo.x;
  const int tmax = (hi.y - 1) * p.grid_x + hi.x - 1;
  for (int rk = 0; rk < p.world_size; ++rk) {
    bool hit = false;
    if (tmax >= tmin) {
      int l = p.dist_global_strategy[rk];
      int r = p.dist_global_strategy[rk + 1];
      if (p.avoid_pixel_all2all) {
        l -= p.grid_x + 1;
        r += p.grid_x + 1;
      }
      hit = !(tmax < l || tmin >= r);
    }
    out[rk] = hit;
  }
}

// One thread per row, 256-row tiles taken in ticket order; a row sent to k
// ranks takes k slots.  Its position in a destination's segment is the
// ordered count of the rows before it that go there: per-warp ballots, a
// block prefix over the warps, and the ordered prefix over the tiles before
// (scan.cuh, one counter per rank).  Rows keep their list order in every
// segment, so with an index-ordered list (the two-kernel preprocess) each
// segment is in ascending index order and the receivers see the same order
// on every run.  send_row records where each slot came from.
constexpr int kPackThreads = 256;
__global__ void __launch_bounds__(kPackThreads) exchange_pack_kernel(PackParams p) {
  __shared__ int s_tile;
  __shared__ int s_wcnt[kPackThreads / 32][32];  // rows per (warp, rank), then their exclusive prefix
  __shared__ int s_base[32];                      // tile's exclusive prefix per rank
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = atomicAdd(p.ticket, 1);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t j = tile * kPackThreads + tid;
  const bool in = j < p.n_rows;
  const uint32_t m = in ? __ldg(p.mask + j) : 0u;
  float4 r0, r1, r2;
  if (m) {
    const float4* src = reinterpret_cast<const float4*>(p.records + 12 * j);
    r0 = src[0];
    r1 = src[1];
    r2 = src[2];
  }
  for (int r = 0; r < p.n_ranks; ++r) {
    const unsigned b = __ballot_sync(0xffffffffu, (m >> r) & 1u);
    if (lane == 0) s_wcnt[warp][r] = __popc(b);
  }
  __syncthreads();
  if (warp == 0) {
    int tot = 0;
    if (lane < p.n_ranks)
      for (int w = 0; w < kPackThreads / 32; ++w) {
        const int c = s_wcnt[w][lane];
        s_wcnt[w][lane] = tot;
        tot += c;
      }
    // one warp-wide look-back per rank
    for (int r = 0; r < p.n_ranks; ++r) {
      const int t_r = __shfl_sync(0xffffffffu, tot, r);
      const int b = (int)scan_exclusive(p.scan_state, tile, p.n_ranks, r, (unsigned long long)t_r, p.status);
      if (lane == 0) s_base[r] = b;
    }
  }
  __syncthreads();
  for (int r = 0; r < p.n_ranks; ++r) {
    const bool mine = (m >> r) & 1u;
    const unsigned b = __ballot_sync(0xffffffffu, mine);
    if (mine) {
      const int64_t pos = p.dest_offset[r] + s_base[r] + s_wcnt[warp][r] + __popc(b & ((1u << lane) - 1u));
      float4* dst = reinterpret_cast<float4*>(p.send + 12 * pos);
      dst[0] = r0;
      dst[1] = r1;
      dst[2] = r2;
      p.send_row[pos] = p.row_base + (int)j;
    }
  }
}

// Rectangle form: rank rk renders tile rows [y_l, y_r) and columns
// [x_l, x_r) (rectangles[4*rk..]), optionally widened by one tile (the low
// bounds only while positive).  The reference tests the square tile rect
// without first rejecting an empty one, and so does this kernel: a Gaussian
// whose clamped rect is empty can still be routed.
__global__ void __launch_bounds__(256) route_bool_rect_kernel(RouteParams p, const int* __restrict__ rects) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= p.P) return;
  bool* out = p.out_bool + i * p.world_size;
  const float2 m = reinterpret_cast<const float2*>(p.means2D)[i];
  int2 lo, hi;
  tile_rect_int(m, p.radii[i], p.grid_x, p.grid_y, lo, hi);
  for (int rk = 0; rk < p.world_size; ++rk) {
    int yl = rects[4 * rk + 0], yr = rects[4 * rk + 1], xl = rects[4 * rk + 2], xr = rects[4 * rk + 3];
    if (p.avoid_pixel_all2all) {
      if (yl > 0) yl -= 1;
      if (xl > 0) xl -= 1;
      yr += 1;
      xr += 1;
    }
    out[rk] = !(hi.y <= yl || yr <= lo.y || hi.x <= xl || xr <= lo.x);
  }
}

}  // namespace

int launch_route_bool_rect(const RouteParams& p, const int* rectangles, cudaStream_t st) {
  if (p.P <= 0) return 0;
  const int threads = 256;
  route_bool_rect_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p, rectangles);
  return (int)cudaGetLastError();
}

namespace {

// Segment s and offset inside it of camera row r (segments are few: a
// linear scan over the run lengths).
__device__ __forceinline__ int64_t segment_row(const Segments& sg, int64_t r) {
  for (int s = 0; s < sg.n; ++s) {
    if (r < sg.count[s]) return sg.start[s] + r;
    r -= sg.count[s];
  }
  return -1;
}

// Received record [c00 c01 c11 op | x y | r g b | depth radius-bits minscale]
// -> the render's arrays; the min-scale regulariser's sum and count over the
// rows with radius > 0 are reduced per block and added in double.
__global__ void __launch_bounds__(256) exchange_unpack_kernel(UnpackParams p, int64_t n) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double ms = 0.0, cnt = 0.0;
  if (r < n) {
    const int64_t src = segment_row(p.seg, r);
    if (src >= 0) {
      const float4* v = reinterpret_cast<const float4*>(p.records + 12 * src);
      const float4 a = v[0], b = v[1], c = v[2];
      reinterpret_cast<float4*>(p.conic)[r] = a;
      reinterpret_cast<float2*>(p.means2D)[r] = make_float2(b.x, b.y);
      p.rgb[3 * r + 0] = b.z;
      p.rgb[3 * r + 1] = b.w;
      p.rgb[3 * r + 2] = c.x;
      p.depths[r] = c.y;
      const int rad = __float_as_int(c.z);
      p.radii[r] = rad;
      if (rad > 0) {
        ms = c.w;
        cnt = 1.0;
      }
    }
  }
  if (!p.reg) return;
  __shared__ double s_red[2][8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ms += __shfl_xor_sync(0xffffffffu, ms, o);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_red[0][threadIdx.x >> 5] = ms;
    s_red[1][threadIdx.x >> 5] = cnt;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, c = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      a += s_red[0][w];
      c += s_red[1][w];
    }
    if (c > 0.0) {
      atomicAdd(p.reg + 0, a);
      atomicAdd(p.reg + 1, c);
    }
  }
}

// Render-backward record [m.x m.y 0 0 | a.x a.y 0 0 | c00 c01 c11 op | r g b 0]
// of camera row r -> gradient record [c00 c01 c11 op | x y | r g b | |x| |y|
// dminscale] at its send row (dminscale = reg_scale for rows with radius > 0).
__global__ void __launch_bounds__(256) grad_records_pack_kernel(GradPackParams p, int64_t n) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int64_t dst = segment_row(p.seg, r);
  if (dst < 0) return;
  const float4* v = reinterpret_cast<const float4*>(p.rec16 + 16 * r);
  const float4 m = v[0], a = v[1], c = v[2], col = v[3];
  const float g_min = (p.reg_scale && __ldg(p.radii + r) > 0) ? *p.reg_scale : 0.f;
  float4* o = reinterpret_cast<float4*>(p.send + 12 * dst);
  o[0] = c;
  o[1] = make_float4(m.x, m.y, col.x, col.y);
  o[2] = make_float4(col.z, a.x, a.y, g_min);
}

}  // namespace

int launch_exchange_unpack(const UnpackParams& p, int64_t n, cudaStream_t st) {
  if (n <= 0) return 0;
  exchange_unpack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p, n);
  return (int)cudaGetLastError();
}

int launch_grad_records_pack(const GradPackParams& p, int64_t n, cudaStream_t st) {
  if (n <= 0) return 0;
  grad_records_pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p, n);
  return (int)cudaGetLastError();
}

size_t exchange_pack_scratch_bytes(int64_t n_rows, int n_ranks) {
  const int64_t tiles = std::max<int64_t>((n_rows + kPackThreads - 1) / kPackThreads, 1);
  return 384 + 8 * (size_t)tiles * (size_t)std::max(n_ranks, 1);
}

int launch_exchange_pack(PackParams p, void* scratch, cudaStream_t st) {
  if (p.n_rows <= 0) return 0;
  char* b = static_cast<char*>(scratch);
  p.status = reinterpret_cast<unsigned*>(b);  // bytes [0, 256): never cleared here
  p.ticket = reinterpret_cast<int*>(b + 256);
  p.scan_state = reinterpret_cast<unsigned long long*>(b + 384);
  cudaMemsetAsync(b + 256, 0, exchange_pack_scratch_bytes(p.n_rows, p.n_ranks) - 256, st);
  exchange_pack_kernel<<<(unsigned)((p.n_rows + kPackThreads - 1) / kPackThreads), kPackThreads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_route_bool(const RouteParams& p, cudaStream_t st) {
  if (p.P <= 0) return 0;
  const int threads = 256;
  route_bool_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
