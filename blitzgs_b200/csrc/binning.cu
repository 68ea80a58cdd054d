// Tile binning: per-tile lists of Gaussian indices in front-to-back order.
//
// The reference (submodule/diff-gaussian-rasterization_r/cuda_rasterizer/
// rasterizer_impl.cu:602-665) emits one 64-bit key (tile << 32 | depth bits)
// per (Gaussian, tile) instance and radix-sorts all R instances over
// 32 + ceil(log2 T) bits (6 onesweep passes at 1152x864).  Its result is the
// per-tile list ordered by (depth bits, Gaussian index), because the sort is
// stable and instances are emitted in index order.
//
// Here the same order comes from a bucket pass and per-tile sorts, five
// launches in all and no library sort:
//   1. bin_count (or the fused preprocess): per Gaussian, the number of
//      compute_locally tiles its square rect touches -> counts, totals;
//   2. tile_hist: instances per tile (a shared-memory histogram per
//      persistent block, one global atomic per touched bin);
//   3. tile_offsets: one block scans the T tile counts -> ranges (empty tiles
//      keep [0, 0), as the reference's zero-filled ranges do) and a write
//      cursor per tile;
//   4. tile_scatter: every instance takes a slot of its tile by an atomic on
//      the tile's cursor and writes the 64-bit key (depth bits << 32 | index);
//   5. tile_sort: one CTA per tile sorts the tile's keys in shared memory
//      (runs of 32 by warps on shuffles, then merge passes) for up to
//      kSortSmem keys; longer lists are sorted by one cooperative grid in
//      chunks of kSortSmem and merged pairwise (merge path, each output slice
//      staged in shared memory) -- and writes the indices.
// Keys are unique (the index is part of them), so the order within a tile is
// (depth bits, index) whatever order the scatter's atomics gave: identical
// to the reference's.
#include <algorithm>

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace cg = cooperative_groups;

namespace {

constexpr int kMaskSmem = 32 * 1024;  // tiles whose mask is staged in shared memory
constexpr int kHistSmem = 8192;       // tiles counted in a shared-memory histogram
constexpr int kSortSmem = 4096;       // keys a tile_sort CTA sorts in shared memory
constexpr int kSortThreads = 256;
// A merge round of the long lists is split into output slices of
// kMergeSlice keys, kMergeUnits per chunk: four times the CTAs of one slice
// per chunk, so a round over a few very long lists still fills the GPU.
constexpr int kMergeSlice = 1024;
constexpr int kMergeUnits = kSortSmem / kMergeSlice;

__device__ __forceinline__ bool tile_on(const bool* s_mask, const bool* g_mask, int t, bool use_smem) {
  if (!g_mask) return true;
  return use_smem ? s_mask[t] : g_mask[t];
}
// Full rasterizer: the tiles of Gaussian i's float rectangle that pass the
// exact tile test, in row-major order (rasterizer_impl.cu:135-170).
template <typename F>
__device__ __forceinline__ void for_each_reached_tile(const BinParams& p, int64_t i, F f) {
  const float2 m = reinterpret_cast<const float2*>(p.means2D)[i];
  const float2 e = reinterpret_cast<const float2*>(p.rects)[i];
  const float4 co = reinterpret_cast<const float4*>(p.conic_opacity)[i];
  const float thr = tile_reach_threshold(co.w);
  int2 lo, hi;
  tile_rect_f(m, e, p.grid_x, p.grid_y, lo, hi);
  for (int y = lo.y; y < hi.y; ++y)
    for (int x = lo.x; x < hi.x; ++x)
      if (tile_reached(co, m, thr, x, y)) f(y * p.grid_x + x);
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
    if (r > 0 && p.rects) {
      for_each_reached_tile(p, i, [&](int) { ++cnt; });
    } else if (r > 0) {
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

// Warp-cooperative instance expansion.  Each lane holds one Gaussian (g < 0:
// none); the candidate tiles of the warp's Gaussians (the w x h tiles of each
// rectangle) are dealt out 32 per step, one per lane, so the whole warp works
// while any lane has tiles left.  f(valid, i, t) is called by all 32 lanes
// together once per step: valid marks a lane holding a tile t of Gaussian i
// that passes the mask (square radius rectangles) or the exact tile test
// (RECTS).  Callers aggregate their atomics over the lanes of equal tiles.
template <bool RECTS, typename F>
__device__ __forceinline__ void warp_expand(const BinParams& p, int64_t g, const bool* s_mask, bool use_smem, F f) {
  const int lane = threadIdx.x & 31;
  int x0 = 0, y0 = 0, w = 0, n = 0;
  float2 m = make_float2(0.f, 0.f);
  float4 co = make_float4(0.f, 0.f, 0.f, 0.f);
  float thr = 0.f;
  if (g >= 0) {
    m = reinterpret_cast<const float2*>(p.means2D)[g];
    int2 lo, hi;
    if (RECTS) {
      tile_rect_f(m, reinterpret_cast<const float2*>(p.rects)[g], p.grid_x, p.grid_y, lo, hi);
      co = reinterpret_cast<const float4*>(p.conic_opacity)[g];
      thr = tile_reach_threshold(co.w);
    } else {
      tile_rect_int(m, p.radii[g], p.grid_x, p.grid_y, lo, hi);
    }
    x0 = lo.x;
    y0 = lo.y;
    w = hi.x - lo.x;
    n = w * (hi.y - lo.y);
  }
  int incl = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  const int excl = incl - n;
  for (int base = 0; base < total; base += 32) {
    const int k = base + lane;
    // owner: the last lane whose first tile is at or before k
    int j = 0;
#pragma unroll
    for (int sft = 16; sft > 0; sft >>= 1)
      if (__shfl_sync(0xffffffffu, excl, j + sft) <= k) j += sft;
    const int local = k - __shfl_sync(0xffffffffu, excl, j);
    const int ow = __shfl_sync(0xffffffffu, w, j);
    const int ox = __shfl_sync(0xffffffffu, x0, j), oy = __shfl_sync(0xffffffffu, y0, j);
    const int64_t oi = __shfl_sync(0xffffffffu, g, j);
    bool valid = k < total;
    int tx = 0, ty = 0;
    if (valid) {
      ty = oy + local / ow;
      tx = ox + local - (local / ow) * ow;
    }
    const int t = ty * p.grid_x + tx;
    if (RECTS) {
      const float2 om = make_float2(__shfl_sync(0xffffffffu, m.x, j), __shfl_sync(0xffffffffu, m.y, j));
      const float4 oc = make_float4(__shfl_sync(0xffffffffu, co.x, j), __shfl_sync(0xffffffffu, co.y, j),
                                    __shfl_sync(0xffffffffu, co.z, j), __shfl_sync(0xffffffffu, co.w, j));
      const float othr = __shfl_sync(0xffffffffu, thr, j);
      valid = valid && tile_reached(oc, om, othr, tx, ty);
    } else {
      valid = valid && tile_on(s_mask, p.compute_locally, t, use_smem);
    }
    f(valid, oi, t);
  }
}

// Lanes of one warp holding the same tile: returns the lane mask of this
// lane's group (every lane calls it; invalid lanes form a group of their own).
__device__ __forceinline__ unsigned tile_peers(bool valid, int t) {
  return __match_any_sync(0xffffffffu, valid ? t : -1);
}

// Instances per tile, and the visible list: persistent blocks walk all P
// Gaussians 32 per warp; the visible ones (counts > 0) are appended to
// vis_list (any order) and expanded into their tiles, counted in a
// shared-memory histogram with one atomic per (warp step, tile).
template <bool RECTS>
__global__ void __launch_bounds__(256) tile_hist_kernel(BinParams p, unsigned* __restrict__ tile_count,
                                                        uint32_t* __restrict__ vis_list, unsigned* __restrict__ n_vis,
                                                        int64_t vis_cap, unsigned* __restrict__ err) {
  constexpr int kHistMask = 16 * 1024;  // with the histogram, within 48 KB of static shared memory
  __shared__ bool s_mask[kHistMask];
  __shared__ unsigned s_hist[kHistSmem];
  const int n_tiles = p.grid_x * p.grid_y;
  const bool use_smem = p.compute_locally && n_tiles <= kHistMask;
  const bool hist_smem = n_tiles <= kHistSmem;
  if (use_smem)
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_mask[t] = p.compute_locally[t];
  if (hist_smem)
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_hist[t] = 0u;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // kHistUnroll chunks of 32 counts per warp and round, loaded together: most
  // of a view's Gaussians are off-screen, so the walk is bound by the latency
  // of these loads, not by the work behind them
  constexpr int kHistUnroll = 8;
  for (int64_t base0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base0 < p.P;
       base0 += stride * kHistUnroll) {
    unsigned bits = 0u;  // bit u: this lane's Gaussian of chunk u is visible
#pragma unroll
    for (int u = 0; u < kHistUnroll; ++u) {
      const int64_t i = base0 + u * stride + lane;
      bits |= (i < p.P && __ldcs(p.counts + i) != 0u ? 1u : 0u) << u;
    }
    if (!__any_sync(0xffffffffu, bits)) continue;
#pragma unroll 1
    for (int u = 0; u < kHistUnroll; ++u) {
      const int64_t i = base0 + u * stride + lane;
      const bool vis = (bits >> u) & 1u;
      const unsigned vm = __ballot_sync(0xffffffffu, vis);
      if (!vm) continue;  // (warp-uniform)
      unsigned wb = 0u;
      if (lane == 0) wb = atomicAdd(n_vis, (unsigned)__popc(vm));
      wb = __shfl_sync(0xffffffffu, wb, 0);
      bool listed = false;  // only Gaussians with a list slot are counted: the scatter walks the list
      if (vis) {
        const int64_t slot = (int64_t)wb + __popc(vm & ((1u << lane) - 1u));
        listed = slot < vis_cap;
        if (listed)
          vis_list[slot] = (uint32_t)i;
        else
          atomicOr(err, kErrBinOverflow);
      }
      warp_expand<RECTS>(p, listed ? i : -1, s_mask, use_smem, [&](bool valid, int64_t, int t) {
        const unsigned peers = tile_peers(valid, t);
        if (valid && lane == __ffs(peers) - 1)
          atomicAdd(hist_smem ? &s_hist[t] : &tile_count[t], (unsigned)__popc(peers));
      });
    }
  }
  if (!hist_smem) return;
  __syncthreads();
  for (int t = threadIdx.x; t < n_tiles; t += blockDim.x)
    if (s_hist[t]) atomicAdd(&tile_count[t], s_hist[t]);
}

// Exclusive scan of v over the 1024 threads of a block (all threads call).
__device__ __forceinline__ unsigned block_exclusive_scan(unsigned v, unsigned* s_part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();
  if (lane == 31) s_part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned x = lane < (int)(blockDim.x >> 5) ? s_part[lane] : 0u;
    unsigned w = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    s_part[lane] = w - x;
  }
  __syncthreads();
  return s_part[warp] + incl - v;
}

// Lists longer than kSortSmem ("big" tiles) are sorted by the cooperative
// big_tile_sort_kernel in chunks of kSortSmem keys.
__device__ __forceinline__ unsigned big_chunks(unsigned c) {
  return c > (unsigned)kSortSmem ? (c + kSortSmem - 1) / kSortSmem : 0u;
}

// One block: exclusive scan of the tile counts -> ranges and cursors; the
// same scan over the big tiles' chunk counts -> chunk_start, and
// big[0] = all chunks, big[1] = the longest big list.
__global__ void __launch_bounds__(1024) tile_offsets_kernel(const unsigned* __restrict__ tile_count, int n_tiles,
                                                            unsigned cap, uint2* __restrict__ ranges,
                                                            unsigned* __restrict__ cursor,
                                                            unsigned* __restrict__ chunk_start,
                                                            unsigned* __restrict__ big) {
  __shared__ unsigned s_part[32];
  const int per = (n_tiles + blockDim.x - 1) / blockDim.x;  // consecutive tiles of this thread
  const int t0 = threadIdx.x * per;
  unsigned sum = 0u;
  for (int k = 0; k < per; ++k)
    if (t0 + k < n_tiles) sum += tile_count[t0 + k];
  const unsigned start0 = block_exclusive_scan(sum, s_part);
  // Ranges are clipped to the `cap` instances the buffers hold: a caller that
  // sized them from an estimate gets truncated lists (and re-bins), never an
  // access beyond them.  The scatter drops the instances past the cap.
  auto clipped = [&](unsigned start, unsigned c) { return min(start + c, cap) - min(start, cap); };
  unsigned chunks = 0u, longest = 0u, start = start0;
  for (int k = 0; k < per; ++k)
    if (t0 + k < n_tiles) {
      const unsigned c = tile_count[t0 + k], ce = clipped(start, c);
      chunks += big_chunks(ce);
      if (big_chunks(ce)) longest = max(longest, ce);
      start += c;
    }
  const unsigned cstart0 = block_exclusive_scan(chunks, s_part);
  if (longest) atomicMax(&big[1], longest);
  start = start0;
  unsigned cstart = cstart0;
  for (int k = 0; k < per; ++k) {
    const int t = t0 + k;
    if (t >= n_tiles) break;
    const unsigned c = tile_count[t], ce = clipped(start, c);
    ranges[t] = ce ? make_uint2(start, start + ce) : make_uint2(0u, 0u);
    cursor[t] = start;
    chunk_start[t] = cstart;
    start += c;
    cstart += big_chunks(ce);
  }
  if (threadIdx.x == blockDim.x - 1) big[0] = cstart;
}

// Instances take their slots from the tile cursors.  Blocks walk the visible
// list 32 Gaussians per warp (the same Gaussians in both passes): pass 1
// counts the block's instances per tile in shared memory, one global atomic
// per touched tile reserves the block's run of slots, pass 2 hands the slots
// out from shared memory and writes the keys (depth bits << 32 | index).  In
// both passes the lanes of a warp holding the same tile share one atomic.
template <bool RECTS>
__global__ void __launch_bounds__(256) tile_scatter_kernel(BinParams p, const uint32_t* __restrict__ vis_list,
                                                           int64_t vis_cap, const unsigned* __restrict__ vis_count,
                                                           unsigned* __restrict__ cursor,
                                                           unsigned long long* __restrict__ keys, int64_t R,
                                                           unsigned* err) {
  // entries the histogram pass wrote (never more than the list holds)
  const int64_t n_vis = std::min<int64_t>(vis_cap, (int64_t)*vis_count);
  constexpr int kScatterMask = 16 * 1024;
  __shared__ bool s_mask[kScatterMask];
  __shared__ unsigned s_slot[kHistSmem];
  const int n_tiles = p.grid_x * p.grid_y;
  const bool use_smem = p.compute_locally && n_tiles <= kScatterMask;
  const bool agg = n_tiles <= kHistSmem;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  if (use_smem)
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_mask[t] = p.compute_locally[t];
  // hands out slots from *ctr (shared or global) and writes the keys
  auto emit = [&](unsigned* ctr_base) {
    for (int64_t base = first; base < n_vis; base += stride) {
      const int64_t g = base + lane < n_vis ? (int64_t)vis_list[base + lane] : -1;
      warp_expand<RECTS>(p, g, s_mask, use_smem, [&](bool valid, int64_t i, int t) {
        const unsigned peers = tile_peers(valid, t);
        const int leader = __ffs(peers) - 1;
        unsigned b = 0u;
        if (valid && lane == leader) b = atomicAdd(&ctr_base[t], (unsigned)__popc(peers));
        b = __shfl_sync(0xffffffffu, b, leader);
        if (valid) {
          const unsigned slot = b + __popc(peers & ((1u << lane) - 1u));
          if ((int64_t)slot < R)
            keys[slot] = ((unsigned long long)float_bits(p.depths[i]) << 32) | (unsigned long long)(uint32_t)i;
          else
            atomicOr(err, kErrBinOverflow);
        }
      });
    }
  };
  if (!agg) {
    __syncthreads();
    emit(cursor);
    return;
  }
  for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) s_slot[t] = 0u;
  __syncthreads();
  for (int64_t base = first; base < n_vis; base += stride) {
    const int64_t g = base + lane < n_vis ? (int64_t)vis_list[base + lane] : -1;
    warp_expand<RECTS>(p, g, s_mask, use_smem, [&](bool valid, int64_t, int t) {
      const unsigned peers = tile_peers(valid, t);
      if (valid && lane == __ffs(peers) - 1) atomicAdd(&s_slot[t], (unsigned)__popc(peers));
    });
  }
  __syncthreads();
  for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) {
    const unsigned c = s_slot[t];
    if (c) s_slot[t] = atomicAdd(&cursor[t], c);
  }
  __syncthreads();
  emit(s_slot);
}

// Shared-memory layout of a sort buffer: one pad word after every 16 keys, so
// that threads which each own 16 consecutive keys hit different banks.
__device__ __forceinline__ int pad(int x) { return x + (x >> 4); }
constexpr int kSortWords = kSortSmem + kSortSmem / 16;  // padded buffer length

// Sort of 32 keys held one per lane (bitonic network on shuffles).
__device__ __forceinline__ unsigned long long warp_sort32(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool up = (lane & k) == 0;   // this lane's 2k-block sorts ascending
      const bool low = (lane & j) == 0;  // this lane keeps the smaller key of its pair
      v = (low == up) ? (o < v ? o : v) : (o < v ? v : o);
    }
  return v;
}

// Co-rank of output position k when merging sorted a[0, na) and b[0, nb)
// (unique keys, read through the accessors): the number of a's keys among
// the first k outputs.
template <class A, class B>
__device__ __forceinline__ int co_rank(A a, int na, B b, int nb, int k) {
  int lo = max(0, k - nb), hi = min(k, na);
  while (lo < hi) {
    const int i = (lo + hi) >> 1;
    if (a(i) < b(k - i - 1))
      lo = i + 1;
    else
      hi = i;
  }
  return lo;
}

// The same, searched by a whole warp 32 candidates at a time (for operands in
// global memory, where each probe is a long-latency load).  All lanes get it.
__device__ __forceinline__ int64_t co_rank_warp(const unsigned long long* a, int64_t na, const unsigned long long* b,
                                                int64_t nb, int64_t k) {
  const int lane = threadIdx.x & 31;
  int64_t lo = k - nb > 0 ? k - nb : 0, hi = k < na ? k : na;
  // invariant: the answer i* (first i with a[i] > b[k-i-1]) lies in [lo, hi]
  while (lo < hi) {
    const int64_t step = (hi - lo + 31) / 32;
    const int64_t i = lo + lane * step;
    const bool below = i < hi && a[i] < b[k - i - 1];  // true on a prefix of the lanes
    const int c = __popc(__ballot_sync(0xffffffffu, below));
    if (c == 0) {
      hi = lo;
    } else {
      const int64_t last = lo + (int64_t)(c - 1) * step;  // largest probe below i*
      hi = min(hi, lo + (int64_t)c * step);
      lo = last + 1;
    }
  }
  return lo;
}

// Merge `cnt` (<= PER) outputs starting at output position k of the sorted
// runs a and b (accessors) into registers o[0, cnt).
template <int PER, class A, class B>
__device__ __forceinline__ void merge_regs(A a, int na, B b, int nb, int k, int cnt, unsigned long long (&o)[PER]) {
  int i = co_rank(a, na, b, nb, k), j = k - i;
#pragma unroll
  for (int q = 0; q < PER; ++q)
    if (q < cnt) {
      if (i < na && (j >= nb || a(i) < b(j)))
        o[q] = a(i++);
      else
        o[q] = b(j++);
    }
}

// Sort s[0, n) (padded layout, n <= kSortSmem) in place, by the block: runs
// of 32 sorted by warps on shuffles, then merge passes of widths 32, 64, ...
// Each pass every thread merges a slice of `per` consecutive outputs (per a
// power of two, per * blockDim >= n, so no slice straddles a pair of runs)
// into registers, and the block writes them back after a barrier.  The keys
// must already be in s; all threads of the block call this.
__device__ void block_sort(unsigned long long* s, int n) {
  constexpr int kPer = kSortSmem / kSortThreads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n_warps = blockDim.x >> 5;
  for (int r = warp; r < (n + 31) >> 5; r += n_warps) {
    const int i = r * 32 + lane;
    const unsigned long long v = warp_sort32(i < n ? s[pad(i)] : ~0ull);
    if (i < n) s[pad(i)] = v;  // the padding keys sort last and are dropped
  }
  __syncthreads();
  int per = 1;
  while (per * (int)blockDim.x < n) per <<= 1;
  const int k = (int)threadIdx.x * per;
  const int cnt = max(0, min(per, n - k));
  for (int w = 32; w < n; w <<= 1) {
    unsigned long long o[kPer];
    if (cnt > 0) {
      const int a0 = k & ~(2 * w - 1);
      const int na = min(w, n - a0), nb = max(0, min(w, n - a0 - w));
      merge_regs<kPer>([&](int i) { return s[pad(a0 + i)]; }, na, [&](int j) { return s[pad(a0 + na + j)]; }, nb,
                       k - a0, cnt, o);
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (q < cnt) s[pad(k + q)] = o[q];
    __syncthreads();
  }
}

// Lists of at most kSortSmem keys: one CTA per tile, sorted in shared memory.
__global__ void __launch_bounds__(kSortThreads) tile_sort_kernel(const uint2* __restrict__ ranges,
                                                                 const unsigned long long* __restrict__ keys,
                                                                 uint32_t* __restrict__ point_list) {
  __shared__ unsigned long long s[kSortWords];
  const uint2 r = ranges[blockIdx.x];
  const int n = (int)(r.y - r.x);
  if (n <= 0 || n > kSortSmem) return;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s[pad(i)] = keys[r.x + i];
  __syncthreads();
  block_sort(s, n);
  for (int i = threadIdx.x; i < n; i += blockDim.x) point_list[r.x + i] = (uint32_t)(s[pad(i)] & 0xffffffffull);
}

// Tile of big chunk b: the last tile whose chunk_start <= b (chunk_start is
// non-decreasing; tiles without big chunks repeat the next one's start).
__device__ __forceinline__ int tile_of_chunk(const unsigned* chunk_start, int n_tiles, unsigned b) {
  int lo = 0, hi = n_tiles - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_start[mid] <= b)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Lists longer than kSortSmem, all big tiles at once, by a cooperative grid:
// every chunk of kSortSmem keys is sorted in shared memory by some CTA, then
// runs of width w = kSortSmem, 2 kSortSmem, ... are merged pairwise until
// the longest list is one run, with a grid-wide barrier between steps.  In a
// merge step a CTA produces one kMergeSlice-key output slice: a warp-wide
// co-rank search finds the input ranges of both runs in global memory, the
// block stages them in shared memory with coalesced loads, merges there and
// stores the slice coalesced -- as indices, in the last step.
__global__ void __launch_bounds__(kSortThreads) big_tile_sort_kernel(const uint2* __restrict__ ranges,
                                                                     const unsigned* __restrict__ chunk_start,
                                                                     const unsigned* __restrict__ big, int n_tiles,
                                                                     unsigned long long* __restrict__ keys,
                                                                     unsigned long long* __restrict__ tmp,
                                                                     uint32_t* __restrict__ point_list) {
  constexpr int kPer = kSortSmem / kSortThreads;
  __shared__ unsigned long long s[kSortWords];
  __shared__ int64_t s_rank[2];
  cg::grid_group grid = cg::this_grid();
  const unsigned n_chunks = big[0], longest = big[1];
  if (n_chunks == 0u) return;  // uniform: every CTA leaves before any barrier
  for (unsigned b = blockIdx.x; b < n_chunks; b += gridDim.x) {
    const int t = tile_of_chunk(chunk_start, n_tiles, b);
    const uint2 r = ranges[t];
    const int c0 = (int)(b - chunk_start[t]) * kSortSmem;
    const int len = min(kSortSmem, (int)(r.y - r.x) - c0);
    unsigned long long* g = keys + r.x + c0;
    for (int i = threadIdx.x; i < len; i += blockDim.x) s[pad(i)] = g[i];
    __syncthreads();
    block_sort(s, len);
    for (int i = threadIdx.x; i < len; i += blockDim.x) g[i] = s[pad(i)];
    __syncthreads();
  }
  unsigned long long *src = keys, *dst = tmp;
  const int warp = threadIdx.x >> 5;
  // (64-bit widths: longest < 2^32, so the doubling ends before any overflow)
  for (int64_t w = kSortSmem; w < (int64_t)longest; w <<= 1) {
    const bool last = 2 * w >= (int64_t)longest;
    grid.sync();
    for (unsigned u = blockIdx.x; u < n_chunks * kMergeUnits; u += gridDim.x) {
      const unsigned b = u / kMergeUnits;
      const int t = tile_of_chunk(chunk_start, n_tiles, b);
      const uint2 r = ranges[t];
      const int64_t n = (int64_t)(r.y - r.x);
      // this output slice of the tile: kSortSmem / kMergeUnits outputs
      const int64_t k0 = (int64_t)(b - chunk_start[t]) * kSortSmem + (int64_t)(u % kMergeUnits) * kMergeSlice;
      if (k0 >= n) continue;  // (uniform over the CTA) the tail of the tile's last chunk
      const int64_t a0 = (k0 / (2 * w)) * (2 * w);  // its pair of runs
      const int64_t na = std::min<int64_t>(w, n - a0), nb = std::max<int64_t>(0, std::min<int64_t>(w, n - a0 - w));
      const int len = (int)std::min<int64_t>(kMergeSlice, n - k0);
      const unsigned long long* ga = src + r.x + a0;
      const unsigned long long* gb = ga + na;
      if (warp < 2) {
        const int64_t i = co_rank_warp(ga, na, gb, nb, k0 - a0 + (warp ? len : 0));
        if ((threadIdx.x & 31) == 0) s_rank[warp] = i;
      }
      __syncthreads();
      const int64_t i0 = s_rank[0], j0 = k0 - a0 - i0;
      const int la = (int)(s_rank[1] - i0), lb = len - la;
      for (int x = threadIdx.x; x < len; x += blockDim.x) s[pad(x)] = x < la ? ga[i0 + x] : gb[j0 + x - la];
      __syncthreads();
      int per = 1;
      while (per * (int)blockDim.x < len) per <<= 1;
      const int k = (int)threadIdx.x * per;
      const int cnt = max(0, min(per, len - k));
      unsigned long long o[kPer];
      if (cnt > 0)
        merge_regs<kPer>([&](int i) { return s[pad(i)]; }, la, [&](int j) { return s[pad(la + j)]; }, lb, k, cnt, o);
      __syncthreads();
#pragma unroll
      for (int q = 0; q < kPer; ++q)
        if (q < cnt) s[pad(k + q)] = o[q];
      __syncthreads();
      if (last) {
        for (int x = threadIdx.x; x < len; x += blockDim.x)
          point_list[r.x + k0 + x] = (uint32_t)(s[pad(x)] & 0xffffffffull);
      } else {
        for (int x = threadIdx.x; x < len; x += blockDim.x) dst[r.x + k0 + x] = s[pad(x)];
      }
      __syncthreads();
    }
    unsigned long long* x = src;
    src = dst;
    dst = x;
  }
}

inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

int launch_bin_count(const BinParams& p, cudaStream_t st) {
  cudaMemsetAsync(p.totals, 0, 2 * sizeof(unsigned long long), st);
  if (p.P <= 0) return (int)cudaGetLastError();
  const int threads = 256;
  bin_count_kernel<<<(unsigned)((p.P + threads - 1) / threads), threads, 0, st>>>(p);
  return (int)cudaGetLastError();
}

size_t bin_scratch_bytes(int64_t P, int64_t n_vis, int64_t R, int n_tiles) {
  (void)P;
  size_t s = 0;
  s += 2 * align_up(sizeof(unsigned long long) * (size_t)std::max<int64_t>(R, 1));  // keys, merge buffer
  s += 3 * align_up(sizeof(unsigned) * (size_t)std::max(n_tiles, 1));  // tile counts, cursors, chunk starts
  s += align_up(sizeof(uint32_t) * (size_t)std::max<int64_t>(n_vis, 1));  // visible list
  s += align_up(sizeof(unsigned) * 4);  // big-tile totals, error word, visible count
  return s;
}

int launch_bin_sort(const BinSortParams& p, cudaStream_t st) {
  const int n_tiles = p.b.grid_x * p.b.grid_y;
  cudaMemsetAsync(p.ranges, 0, sizeof(uint2) * (size_t)n_tiles, st);
  if (p.R <= 0 || p.n_vis <= 0) return (int)cudaGetLastError();
  if (bin_scratch_bytes(p.b.P, p.n_vis, p.R, n_tiles) > p.scratch_bytes) return (int)cudaErrorInvalidValue;
  char* b = reinterpret_cast<char*>(p.scratch);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* r = b + off;
    off += align_up(bytes);
    return r;
  };
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(take(8 * (size_t)p.R));
  unsigned long long* tmp = reinterpret_cast<unsigned long long*>(take(8 * (size_t)p.R));
  unsigned* tile_count = reinterpret_cast<unsigned*>(take(4 * (size_t)n_tiles));
  unsigned* cursor = reinterpret_cast<unsigned*>(take(4 * (size_t)n_tiles));
  unsigned* chunk_start = reinterpret_cast<unsigned*>(take(4 * (size_t)n_tiles));
  uint32_t* vis_list = reinterpret_cast<uint32_t*>(take(4 * (size_t)std::max<int64_t>(p.n_vis, 1)));
  unsigned* misc = reinterpret_cast<unsigned*>(take(16));  // big[2], error word, visible count
  cudaMemsetAsync(tile_count, 0, 4 * (size_t)n_tiles, st);
  cudaMemsetAsync(misc, 0, 16, st);
  static const int sms = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return std::max(n, 1);
  }();
  // persistent grids over all P Gaussians (a visible one is a few percent)
  const int64_t need = (p.b.P + 255) / 256;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(need, 4 * (int64_t)sms));
  const unsigned vblocks = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>((p.n_vis + 255) / 256, 4 * (int64_t)sms));
  if (p.b.rects) {
    tile_hist_kernel<true><<<blocks, 256, 0, st>>>(p.b, tile_count, vis_list, misc + 3, p.n_vis, misc + 2);
    tile_offsets_kernel<<<1, 1024, 0, st>>>(tile_count, n_tiles, (unsigned)p.R, p.ranges, cursor, chunk_start, misc);
    tile_scatter_kernel<true><<<vblocks, 256, 0, st>>>(p.b, vis_list, p.n_vis, misc + 3, cursor, keys, p.R,
                                                        misc + 2);
  } else {
    tile_hist_kernel<false><<<blocks, 256, 0, st>>>(p.b, tile_count, vis_list, misc + 3, p.n_vis, misc + 2);
    tile_offsets_kernel<<<1, 1024, 0, st>>>(tile_count, n_tiles, (unsigned)p.R, p.ranges, cursor, chunk_start, misc);
    tile_scatter_kernel<false><<<vblocks, 256, 0, st>>>(p.b, vis_list, p.n_vis, misc + 3, cursor, keys, p.R,
                                                         misc + 2);
  }
  tile_sort_kernel<<<(unsigned)n_tiles, kSortThreads, 0, st>>>(p.ranges, keys, p.point_list);
  // big lists: a cooperative grid of co-resident CTAs (it leaves at once when there are none)
  static const int coop_blocks = [] {
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, big_tile_sort_kernel, kSortThreads, 0);
    return std::max(per_sm, 1) * sms;
  }();
  const uint2* ranges = p.ranges;
  const unsigned* cs = chunk_start;
  const unsigned* big = misc;
  int nt = n_tiles;
  uint32_t* pl = p.point_list;
  void* args[] = {(void*)&ranges, (void*)&cs, (void*)&big, (void*)&nt, (void*)&keys, (void*)&tmp, (void*)&pl};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)big_tile_sort_kernel, dim3(coop_blocks), dim3(kSortThreads),
                                              args, 0, st);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaGetLastError();
}

}  // namespace blitz
