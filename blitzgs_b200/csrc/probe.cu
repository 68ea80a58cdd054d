// FP32 throughput probe: the denominator of the blend kernels' roofline.
// Every thread runs 8 independent FMA chains, so the FMA pipe, not latency,
// bounds it; FLOPs = 2 * 8 * iters per thread.
#include "kernels.h"

namespace blitz {
namespace {

__global__ void __launch_bounds__(256) fma_probe_kernel(int64_t iters, float* sink) {
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = threadIdx.x * 1e-7f + k * 1e-6f;
  const float b = 0.9999999f, c = 1e-7f;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = fmaf(a[k], b, c);
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += a[k];
  if (s == 12345.678f) sink[0] = s;  // keeps the chains alive, never true
}

}  // namespace

int launch_fma_probe(int blocks, int64_t iters, float* sink, cudaStream_t st) {
  fma_probe_kernel<<<blocks, 256, 0, st>>>(iters, sink);
  return (int)cudaGetLastError();
}

}  // namespace blitz
