// Ordered prefix sums across the blocks of one launch, in a single pass
// (chained scan with decoupled look-back, Merrill & Garland 2016).
//
// A launch splits its input into tiles taken in ticket order (an atomic
// counter read by each block when it starts a tile).  For counter c, tile t
// publishes its own total ("aggregate") at once, then walks back over tiles
// t-1, t-2, ... adding their aggregates until it meets a tile that has
// published its inclusive prefix, and finally publishes its own inclusive
// prefix.  The result is tile t's exclusive prefix: the sum over the tiles
// before it, so outputs written at those offsets keep the input order no
// matter in which order the blocks ran.
//
// Progress: every tile a block waits on was ticketed earlier by a block that
// is already running, and a block publishes its aggregate before it waits on
// anything, so each wait ends.  The waits are bounded regardless: after
// kScanSpinLimit polls the block ORs kScanTimeout into *status and goes on
// with the partial sum, and the host reports the status.  Each tile's
// look-back is done by one warp, 32 predecessor tiles per step.
//
// State: one 64-bit word per (tile, counter), zero before the launch; bits
// 62-63 hold the flag, bits 0-61 the value, so a word is published and read
// in one access.
#pragma once
#include <cstdint>

namespace blitz {

constexpr unsigned kScanTimeout = 1u << 4;  // status bit: a look-back gave up waiting
constexpr unsigned long long kScanAgg = 1ull << 62;
constexpr unsigned long long kScanIncl = 2ull << 62;
constexpr unsigned long long kScanValue = (1ull << 62) - 1;
constexpr int kScanSpinLimit = 1 << 20;

__device__ __forceinline__ void scan_store(unsigned long long* w, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(w), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long scan_load(const unsigned long long* w) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
  return v;
}

// Exclusive prefix of counter c for tile `tile` whose own total is `agg`.
// state: [n_tiles][stride] words.  All 32 lanes of one warp call this
// together and all get the result.  The warp reads the 32 tiles before its
// window at once, so a tile whose predecessors have only published their
// aggregates walks back 32 tiles per step, not one.
__device__ __forceinline__ unsigned long long scan_exclusive(unsigned long long* state, int64_t tile, int stride,
                                                             int c, unsigned long long agg, unsigned* status) {
  const int lane = threadIdx.x & 31;
  unsigned long long* mine = state + tile * stride + c;
  if (tile == 0) {
    if (lane == 0) scan_store(mine, kScanIncl | agg);
    return 0ull;
  }
  if (lane == 0) scan_store(mine, kScanAgg | agg);
  unsigned long long excl = 0ull;
  int64_t top = tile - 1;  // nearest tile of the window (lane 0)
  int spins = 0;
  for (;;) {
    const int64_t t = top - lane;
    // before tile 0 the sum is an inclusive zero
    const unsigned long long w = t >= 0 ? scan_load(state + t * stride + c) : kScanIncl;
    const unsigned long long flag = w & ~kScanValue;
    if (__any_sync(0xffffffffu, flag == 0ull)) {
      if (++spins > kScanSpinLimit) {
        if (lane == 0) atomicOr(status, kScanTimeout);
        break;
      }
      __nanosleep(32);
      continue;
    }
    const unsigned incl = __ballot_sync(0xffffffffu, flag == kScanIncl);
    const int stop = incl ? __ffs(incl) - 1 : 31;  // the nearest inclusive tile covers all before it
    unsigned long long v = lane <= stop ? (w & kScanValue) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    excl += v;
    if (incl) break;
    top -= 32;
  }
  if (lane == 0) scan_store(mine, kScanIncl | (excl + agg));
  return excl;
}

}  // namespace blitz
