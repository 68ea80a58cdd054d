// Zeroing listed rows of dense gradient buffers (one launch for all of them).
//
// The fused step hands out dense parameter gradients whose only non-zero
// rows are the ones an earlier view wrote; before a buffer is reused, those
// rows -- a few percent of the model -- are zeroed instead of the whole
// buffer.  blockIdx.y picks the array; the words of the listed rows are
// spread over the threads of a grid-stride loop.
#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

__global__ void __launch_bounds__(256) zero_rows_kernel(ZeroRowsParams p) {
  const int a = blockIdx.y;
  uint32_t* base = reinterpret_cast<uint32_t*>(p.arrays[a]);
  const uint32_t words = (uint32_t)p.row_words[a];
  // flat (listed row, word) index: consecutive threads write consecutive words
  // of a row and then of the next listed row, so narrow rows (3-4 words)
  // still keep every lane busy; 32-bit arithmetic (the launcher checks the range)
  const uint32_t total = words * (uint32_t)p.n_rows;
  for (uint32_t f = blockIdx.x * blockDim.x + threadIdx.x; f < total; f += gridDim.x * blockDim.x) {
    const uint32_t r = f / words;
    base[(int64_t)p.rows[r] * words + (f - r * words)] = 0u;
  }
}

}  // namespace

int launch_zero_rows(const ZeroRowsParams& p, cudaStream_t st) {
  if (p.n_arrays <= 0 || p.n_rows <= 0) return 0;
  int64_t most = 0;
  for (int a = 0; a < p.n_arrays; ++a) most = p.row_words[a] > most ? p.row_words[a] : most;
  if (most * p.n_rows >= (int64_t)1 << 31) return (int)cudaErrorInvalidValue;  // (2^31 words: 8 GB of rows)
  const int64_t need = (most * p.n_rows + 255) / 256;
  const unsigned blocks = (unsigned)(need < 2368 ? need : 2368);
  zero_rows_kernel<<<dim3(blocks, (unsigned)p.n_arrays), 256, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
