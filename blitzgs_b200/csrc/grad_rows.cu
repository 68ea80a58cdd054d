// Zeroing listed rows of dense gradient buffers (one launch for all of them).
//
// The fused step hands out dense parameter gradients whose only non-zero
// rows are the ones an earlier view wrote; before a buffer is reused, those
// rows -- a few percent of the model -- are zeroed instead of the whole
// buffer.  blockIdx.y picks the array; the 32-bit words of the listed rows
// are spread over a grid-stride loop (row-major: consecutive threads write
// consecutive words of a row, then the next listed row).
#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

__global__ void __launch_bounds__(256) zero_rows_kernel(ZeroRowsParams p) {
  const int a = blockIdx.y;
  uint32_t* base = reinterpret_cast<uint32_t*>(p.arrays[a]);
  const int64_t words = p.row_words[a];
  const int64_t total = words * p.n_rows;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = w / words;
    base[(int64_t)p.rows[r] * words + (w - r * words)] = 0u;
  }
}

}  // namespace

int launch_zero_rows(const ZeroRowsParams& p, cudaStream_t st) {
  if (p.n_arrays <= 0 || p.n_rows <= 0) return 0;
  int64_t most = 0;
  for (int a = 0; a < p.n_arrays; ++a) most = p.row_words[a] > most ? p.row_words[a] : most;
  const int64_t need = (most * p.n_rows + 255) / 256;
  const unsigned blocks = (unsigned)(need < 4096 ? (need > 0 ? need : 1) : 4096);
  zero_rows_kernel<<<dim3(blocks, (unsigned)p.n_arrays), 256, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
