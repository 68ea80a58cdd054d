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

}  // namespace

int launch_route_bool(const RouteParams& p, cudaStream_t st) {
  if (p.P <= 0) return 0;
  const int threads = 256;
  route_bool_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
