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
#include "common.cuh"
#include "kernels.h"

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

// One thread per row; a row sent to k ranks takes k slots.  Positions within
// a (rank, camera) segment come from warp-aggregated atomics, so their order
// varies run to run; send_row records where each one came from.
__global__ void __launch_bounds__(256) exchange_pack_kernel(PackParams p) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
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
    const bool mine = (m >> r) & 1u;
    const unsigned b = __ballot_sync(0xffffffffu, mine);
    if (!b) continue;
    int base = 0;
    if (lane == __ffs(b) - 1) base = atomicAdd(p.cursor + r, __popc(b));
    base = __shfl_sync(0xffffffffu, base, __ffs(b) - 1);
    if (mine) {
      const int64_t pos = p.dest_offset[r] + base + __popc(b & ((1u << lane) - 1u));
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

int launch_exchange_pack(const PackParams& p, cudaStream_t st) {
  if (p.n_rows <= 0) return 0;
  const int threads = 256;
  exchange_pack_kernel<<<(unsigned)((p.n_rows + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_route_bool(const RouteParams& p, cudaStream_t st) {
  if (p.P <= 0) return 0;
  const int threads = 256;
  route_bool_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
