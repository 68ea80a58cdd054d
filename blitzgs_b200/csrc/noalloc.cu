// Binning without any caller-provided scratch: blitz_render_bin_noalloc.
//
// Who needs this: a caller that can hand over its input and output buffers
// but cannot allocate device memory at call time.  Examples: a host whose own
// memory pool owns the whole GPU, so an extra allocation fails or fragments
// the pool; a plain-C or FFI host that has no device allocator of its own;
// a latency-critical loop where an allocation's implicit device
// synchronisation is not acceptable.  blitz_render_bin needs a scratch buffer
// whose size is only known after blitz_render_count, which such a caller
// cannot provide.
//
// Here the scratch is one fixed array in device global memory, part of this
// library's module: every GPU that loads the library holds kNoAllocScratch
// bytes of it until the process exits.  Nothing is allocated per call: no
// cudaMalloc / cudaFree and no allocating library routine.
//
// Limits and rules:
//   * capacity: blitz_render_scratch_bytes(P, n_vis, R, H, W) must not exceed
//     BLITZ_NOALLOC_SCRATCH_BYTES (64 MiB); larger requests are rejected with
//     BLITZ_ESCRATCH and a message, before anything is launched;
//   * the array is shared by every call in the process on a given device and
//     keeps whatever the last call left in it; the parts that must start at
//     zero (the per-tile counters and the small block of totals and error
//     word) are cleared by the binning itself on the call's stream, with
//     cudaMemsetAsync, before its first kernel; every other buffer in it is
//     written before it is read;
//   * two calls whose work overlaps on the GPU (different streams, or host
//     threads without ordering) race on the array: order them;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress with that device current) and caches it; make
//     that first call before any stream capture on the device;
//   * the cached address belongs to the device's primary context (the one
//     the CUDA runtime, and PyTorch, use): a host that drives the device
//     through a context of its own, or resets the device within the
//     process, must not call this entry point.
#include <cstdio>
#include <mutex>

#include "blitzgs_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratch = BLITZ_NOALLOC_SCRATCH_BYTES;

// The scratch.  In host code this name is only a handle for the runtime, not
// a device address: it must go through cudaGetSymbolAddress before a kernel
// may use it.
static __device__ __align__(256) unsigned char g_bin_scratch[kNoAllocScratch];

constexpr int kMaxDevices = 64;
constexpr int kErrDeviceOrdinal = -1;  // internal: the current device's ordinal is >= kMaxDevices
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

thread_local char g_msg[320];

int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return kErrDeviceOrdinal;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bin_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int blitz_render_bin_noalloc(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width,
                                        const float* means2D, const float* depths, const int32_t* radii,
                                        const uint8_t* compute_locally, const uint32_t* counts,
                                        uint32_t* point_list, uint32_t* ranges, void* stream) {
  using namespace blitz;
  if (P < 0 || n_vis < 0 || R < 0 || R >= (int64_t)0x7fffffff || n_vis > P || image_height <= 0 || image_width <= 0) {
    set_last_error("blitz_render_bin_noalloc: bad sizes");
    return BLITZ_EINVAL;
  }
  const size_t need = blitz_render_scratch_bytes(P, n_vis, R, image_height, image_width);
  if (R > 0 && need > kNoAllocScratch) {
    snprintf(g_msg, sizeof(g_msg),
             "blitz_render_bin_noalloc: needs %zu bytes of scratch, more than its fixed %zu-byte array "
             "(P=%lld, n_vis=%lld, R=%lld); use blitz_render_bin with a caller buffer",
             need, kNoAllocScratch, (long long)P, (long long)n_vis, (long long)R);
    set_last_error(g_msg);
    return BLITZ_ESCRATCH;
  }
  void* scratch = nullptr;
  int e = noalloc_scratch(&scratch);
  if (e == kErrDeviceOrdinal) {
    snprintf(g_msg, sizeof(g_msg), "blitz_render_bin_noalloc: the current device's ordinal is beyond the %d devices "
             "this entry point supports", kMaxDevices);
    set_last_error(g_msg);
    return BLITZ_EINVAL;
  }
  if (e) {
    snprintf(g_msg, sizeof(g_msg), "blitz_render_bin_noalloc: cudaGetSymbolAddress of the static scratch failed (%d)", e);
    set_last_error(g_msg);
    return e;
  }
  return blitz_render_bin(P, n_vis, R, image_height, image_width, means2D, depths, radii, compute_locally, counts,
                          scratch, kNoAllocScratch, point_list, ranges, stream);
}
