// Tile binning: per-tile lists of Gaussian indices in front-to-back order.
//
// The reference (submodule/diff-gaussian-rasterization_r/cuda_rasterizer/
// rasterizer_impl.cu:602-665) emits one 64-bit key (tile << 32 | depth bits)
// per (Gaussian, tile) instance and radix-sorts all R instances over
// 32 + ceil(log2 T) bits (6 onesweep passes at 1152x864).  Its result is the
// per-tile list ordered by (depth bits, Gaussian index), because the sort is
// stable and instances are emitted in index order.
//
// Here the same order is produced with far fewer bytes moved:
//   1. bin_count: per Gaussian, the number of compute_locally tiles its
//      square rect touches (0 = not rendered) -> counts, totals {R, n_vis};
//   2. compact the visible Gaussians in index order (cub select);
//   3. stable sort of the n_vis depth keys (32 bits, over Gaussians, not
//      instances);
//   4. exclusive scan of the counts in depth order -> write offsets;
//   5. emit: each visible Gaussian writes its tile ids in depth order;
//   6. stable sort of the R instances by tile id only (ceil(log2 T) bits:
//      12 bits at 1152x864, two passes);
//   7. tile ranges from the sorted tile ids.
// Stable sorts in steps 3 and 6 make the final order (tile, depth, index),
// identical to the reference's.
#include <cub/cub.cuh>

#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

constexpr int kMaskSmem = 32 * 1024;  // tiles whose mask is staged in shared memory

__device__ __forceinline__ bool tile_on(const bool* s_mask, const bool* g_mask, int t, bool use_smem) {
  if (!g_mask) return true;
  return use_smem ? s_mask[t] : g_mask[t];
}

__global__ void __launch_bounds__(256) bin_count_kernel(BinParams p) {
  __shared__ bool s_mask[kMaskSmem];
  __shared__ unsigned long long s_tot[2];
  const int n_tiles = p.grid_x * p.grid_y;
  const bool use_smem = p.compute_locally && n_tiles <= kMaskSmem;
  if (threadIdx.x < 2) s_tot[threadIdx.x] = 0ull;
  if (use_smem)
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_mask[t] = p.compute_locally[t];
  __syncthreads();

  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t cnt = 0;
  if (i < p.P) {
    const int r = p.radii[i];
    if (r > 0) {
      const float2 m = reinterpret_cast<const float2*>(p.means2D)[i];
      int2 lo, hi;
      tile_rect_int(m, r, p.grid_x, p.grid_y, lo, hi);
      if (!p.compute_locally) {
        cnt = (uint32_t)((hi.x - lo.x) * (hi.y - lo.y));
      } else {
        for (int y = lo.y; y < hi.y; ++y)
          for (int x = lo.x; x < hi.x; ++x)
            cnt += tile_on(s_mask, p.compute_locally, y * p.grid_x + x, use_smem) ? 1u : 0u;
      }
    }
    p.counts[i] = cnt;
  }
  // block totals -> one atomic per block
  unsigned long long c = cnt, v = cnt > 0 ? 1ull : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    c += __shfl_xor_sync(0xffffffffu, c, o);
    v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  if ((threadIdx.x & 31) == 0 && (c | v)) {
    atomicAdd(&s_tot[0], c);
    atomicAdd(&s_tot[1], v);
  }
  __syncthreads();
  if (threadIdx.x == 0 && (s_tot[0] | s_tot[1])) {
    atomicAdd(&p.totals[0], s_tot[0]);
    atomicAdd(&p.totals[1], s_tot[1]);
  }
}

struct Positive {
  __host__ __device__ __forceinline__ bool operator()(const uint32_t& c) const { return c > 0; }
};

__global__ void gather_depth_keys(const uint32_t* __restrict__ vis_idx, const float* __restrict__ depths,
                                  uint32_t* __restrict__ keys, int64_t n) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n) keys[j] = float_bits(depths[vis_idx[j]]);
}

__global__ void gather_counts(const uint32_t* __restrict__ order, const uint32_t* __restrict__ counts,
                              uint32_t* __restrict__ out, int64_t n) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n) out[j] = counts[order[j]];
}

__global__ void __launch_bounds__(256) emit_kernel(BinParams p, const uint32_t* __restrict__ order,
                                                   const uint32_t* __restrict__ offsets, int64_t n_vis,
                                                   int64_t R, uint32_t* __restrict__ tile_keys,
                                                   uint32_t* __restrict__ vals, unsigned* err) {
  __shared__ bool s_mask[kMaskSmem];
  const int n_tiles = p.grid_x * p.grid_y;
  const bool use_smem = p.compute_locally && n_tiles <= kMaskSmem;
  if (use_smem)
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_mask[t] = p.compute_locally[t];
  __syncthreads();
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n_vis) return;
  const uint32_t i = order[j];
  int64_t off = offsets[j];
  const float2 m = reinterpret_cast<const float2*>(p.means2D)[i];
  int2 lo, hi;
  tile_rect_int(m, p.radii[i], p.grid_x, p.grid_y, lo, hi);
  for (int y = lo.y; y < hi.y; ++y)
    for (int x = lo.x; x < hi.x; ++x) {
      const int t = y * p.grid_x + x;
      if (!tile_on(s_mask, p.compute_locally, t, use_smem)) continue;
      if (off < R) {
        tile_keys[off] = (uint32_t)t;
        vals[off] = i;
      } else {
        atomicOr(err, kErrBinOverflow);
      }
      ++off;
    }
}

__global__ void tile_ranges_kernel(const uint32_t* __restrict__ keys, int64_t R, uint2* __restrict__ ranges,
                                   uint32_t n_tiles) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= R) return;
  const uint32_t t = keys[k];
  if (t >= n_tiles || (k > 0 && keys[k - 1] >= n_tiles)) return;  // never taken when counts are consistent
  if (k == 0)
    ranges[t].x = 0;
  else {
    const uint32_t prev = keys[k - 1];
    if (prev != t) {
      ranges[prev].y = (uint32_t)k;
      ranges[t].x = (uint32_t)k;
    }
  }
  if (k == R - 1) ranges[t].y = (uint32_t)R;
}

int tile_bits(int n_tiles) {
  int b = 1;
  while ((1ll << b) < (long long)n_tiles) ++b;
  return b;
}

inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

struct Carve {
  char* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t n) {
    T* r = reinterpret_cast<T*>(base + off);
    off += align_up(n * sizeof(T));
    return r;
  }
};

size_t cub_temp_bytes(int64_t P, int64_t n_vis, int64_t R, int n_tiles) {
  size_t a = 0, b = 0, c = 0, d = 0;
  cub::CountingInputIterator<uint32_t> it(0);
  cub::TransformInputIterator<bool, Positive, const uint32_t*> flags(nullptr, Positive());
  cub::DeviceSelect::Flagged(nullptr, a, it, flags, (uint32_t*)nullptr, (int*)nullptr, (int)std::max<int64_t>(P, 1));
  cub::DeviceRadixSort::SortPairs(nullptr, b, (uint32_t*)nullptr, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (uint32_t*)nullptr, (int)std::max<int64_t>(n_vis, 1), 0, 32);
  cub::DeviceScan::ExclusiveSum(nullptr, c, (uint32_t*)nullptr, (uint32_t*)nullptr, (int)std::max<int64_t>(n_vis, 1));
  cub::DeviceRadixSort::SortPairs(nullptr, d, (uint32_t*)nullptr, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (uint32_t*)nullptr, (int)std::max<int64_t>(R, 1), 0, tile_bits(n_tiles));
  return std::max(std::max(a, b), std::max(c, d));
}

}  // namespace

int launch_bin_count(const BinParams& p, cudaStream_t st) {
  cudaMemsetAsync(p.totals, 0, 2 * sizeof(unsigned long long), st);
  if (p.P <= 0) return (int)cudaGetLastError();
  const int threads = 256;
  bin_count_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

size_t bin_scratch_bytes(int64_t P, int64_t n_vis, int64_t R, int n_tiles) {
  size_t s = 0;
  s += 5 * align_up(sizeof(uint32_t) * std::max<int64_t>(n_vis, 1));  // vis idx, keys, keys sorted, order, cnt
  s += align_up(sizeof(uint32_t) * std::max<int64_t>(n_vis, 1));      // offsets
  s += 3 * align_up(sizeof(uint32_t) * std::max<int64_t>(R, 1));      // tile keys, sorted keys, vals
  s += align_up(sizeof(int) * 4);                                     // num selected, error word
  s += align_up(cub_temp_bytes(P, n_vis, R, n_tiles));
  return s;
}

int launch_bin_sort(const BinSortParams& p, cudaStream_t st) {
  const int n_tiles = p.b.grid_x * p.b.grid_y;
  cudaMemsetAsync(p.ranges, 0, sizeof(uint2) * (size_t)n_tiles, st);
  if (p.R <= 0 || p.n_vis <= 0) return (int)cudaGetLastError();
  if (bin_scratch_bytes(p.b.P, p.n_vis, p.R, n_tiles) > p.scratch_bytes) return (int)cudaErrorInvalidValue;

  Carve cv{reinterpret_cast<char*>(p.scratch)};
  uint32_t* vis_idx = cv.take<uint32_t>(p.n_vis);
  uint32_t* dkeys = cv.take<uint32_t>(p.n_vis);
  uint32_t* dkeys_sorted = cv.take<uint32_t>(p.n_vis);
  uint32_t* order = cv.take<uint32_t>(p.n_vis);
  uint32_t* cnt_sorted = cv.take<uint32_t>(p.n_vis);
  uint32_t* offsets = cv.take<uint32_t>(p.n_vis);
  uint32_t* tkeys = cv.take<uint32_t>(p.R);
  uint32_t* tkeys_sorted = cv.take<uint32_t>(p.R);
  uint32_t* vals = cv.take<uint32_t>(p.R);
  int* misc = cv.take<int>(4);
  size_t temp_bytes = cub_temp_bytes(p.b.P, p.n_vis, p.R, n_tiles);
  void* temp = cv.take<char>(temp_bytes);

  const int nvis = (int)p.n_vis;
  const int R = (int)p.R;
  const int threads = 256;
  cudaError_t e;

  // 2. compact visible Gaussians (index order preserved)
  {
    cub::CountingInputIterator<uint32_t> it(0);
    cub::TransformInputIterator<bool, Positive, const uint32_t*> flags(p.b.counts, Positive());
    size_t tb = temp_bytes;
    e = cub::DeviceSelect::Flagged(temp, tb, it, flags, vis_idx, misc, (int)p.b.P, st);
    if (e != cudaSuccess) return (int)e;
  }
  gather_depth_keys<<<(nvis + threads - 1) / threads, threads, 0, st>>>(vis_idx, p.b.depths, dkeys, nvis);
  // 3. stable depth sort over visible Gaussians
  {
    size_t tb = temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(temp, tb, dkeys, dkeys_sorted, vis_idx, order, nvis, 0, 32, st);
    if (e != cudaSuccess) return (int)e;
  }
  // 4. offsets in depth order
  gather_counts<<<(nvis + threads - 1) / threads, threads, 0, st>>>(order, p.b.counts, cnt_sorted, nvis);
  {
    size_t tb = temp_bytes;
    e = cub::DeviceScan::ExclusiveSum(temp, tb, cnt_sorted, offsets, nvis, st);
    if (e != cudaSuccess) return (int)e;
  }
  // 5. emit tile ids
  emit_kernel<<<(nvis + threads - 1) / threads, threads, 0, st>>>(p.b, order, offsets, nvis, R, tkeys, vals,
                                                                  reinterpret_cast<unsigned*>(misc + 1));
  // 6. stable sort by tile id
  {
    size_t tb = temp_bytes;
    e = cub::DeviceRadixSort::SortPairs(temp, tb, tkeys, tkeys_sorted, vals, p.point_list, R, 0,
                                        tile_bits(n_tiles), st);
    if (e != cudaSuccess) return (int)e;
  }
  // 7. ranges
  tile_ranges_kernel<<<(R + threads - 1) / threads, threads, 0, st>>>(tkeys_sorted, R, p.ranges, (uint32_t)n_tiles);
  return (int)cudaGetLastError();
}

}  // namespace blitz
