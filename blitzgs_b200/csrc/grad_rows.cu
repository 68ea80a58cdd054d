// Zeroing listed rows of dense gradient buffers (one launch for all of them).
//
// The fused step hands out dense parameter gradients whose only non-zero
// rows are the ones an earlier view wrote; before a buffer is reused, those
// rows -- a few percent of the model -- are zeroed instead of the whole
// buffer.  blockIdx.y picks the array; each warp clears one listed row at a
// time, its lanes on consecutive words of the row.
#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

__global__ void __launch_bounds__(256) zero_rows_kernel(ZeroRowsParams p) {
  const int a = blockIdx.y;
  uint32_t* base = reinterpret_cast<uint32_t*>(p.arrays[a]);
  const int64_t words = p.row_words[a];
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  // one warp per listed row: its lanes clear the row's words (no division)
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < p.n_rows; r += warps) {
    uint32_t* row = base + (int64_t)p.rows[r] * words;
    for (int64_t c = lane; c < words; c += 32) row[c] = 0u;
  }
}

}  // namespace

int launch_zero_rows(const ZeroRowsParams& p, cudaStream_t st) {
  if (p.n_arrays <= 0 || p.n_rows <= 0) return 0;
  const int64_t need = (p.n_rows + 7) / 8;  // 8 warps (rows) per block and round
  const unsigned blocks = (unsigned)(need < 1184 ? need : 1184);
  zero_rows_kernel<<<dim3(blocks, (unsigned)p.n_arrays), 256, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
