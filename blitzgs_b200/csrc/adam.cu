// Sparse Adam step of the Gaussian parameters (the reference's
// SparseGaussianAdam, f/diff_gaussian_rasterization_f/__init__.py:830-863,
// kernel f/cuda_rasterizer/adam.cu:10-38): Adam moments and parameter are
// updated only for the Gaussians marked visible; the others keep their
// moments unchanged (lazy Adam).  The bias corrections are folded into lr by
// the caller, as in the reference.
//
// Two forms:
//   * dense: a [N, M] parameter with a dense gradient and a bool [N]
//     visibility mask (the reference's adamUpdate, bit for bit: the same
//     per-element expressions, so the same FMA contractions);
//   * rows: only the listed rows, with the gradient given as compact rows
//     (the sparse gradient of view_loss(sparse_grad=True)): no pass over the
//     invisible Gaussians at all.  It also folds in the trainer's gradient
//     scaling by 1/bsz (train_internal.py:504-515), bit for bit.
// Both are HBM bound: per updated element, read param, grad, two moments
// (16 B) and write param and moments (12 B).
#include "kernels.h"

namespace blitz {

namespace {

// The reference build contracts the two moment updates as
// fma(1 - b1, g, b1 * m) and fma((1 - b2) * g, g, b2 * v); they are written
// out here so that no other contraction can be chosen.  Divide and square
// root are the IEEE-rounded ones (no fast-math), as in the reference.
__device__ __forceinline__ void adam_element(float& param, float grad, float& m, float& v, float lr, float b1,
                                             float b2, float eps) {
  m = __fmaf_rn(1.0f - b1, grad, __fmul_rn(b1, m));
  v = __fmaf_rn(__fmul_rn(1.0f - b2, grad), grad, __fmul_rn(b2, v));
  const float step = __fdiv_rn(__fmul_rn(-lr, m), __fadd_rn(__fsqrt_rn(v), eps));
  param = __fadd_rn(param, step);
}

__global__ void __launch_bounds__(256) adam_dense_kernel(AdamParams p) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= p.N * p.M) return;
  const int64_t g = e / p.M;
  if (!p.visible[g]) return;
  float param = p.param[e], m = p.exp_avg[e], v = p.exp_avg_sq[e];
  adam_element(param, p.grad[e], m, v, p.lr, p.b1, p.b2, p.eps);
  p.param[e] = param;
  p.exp_avg[e] = m;
  p.exp_avg_sq[e] = v;
}

// element e of the listed rows: row j = e / M of the compact gradient,
// Gaussian rows[j] of the parameter and its moments
__global__ void __launch_bounds__(256) adam_rows_kernel(AdamParams p) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= p.n_rows * p.M) return;
  const int64_t j = e / p.M, c = e - j * p.M;
  const int64_t g = p.rows[j];
  if (g < 0 || g >= p.N) return;
  const int64_t k = g * p.M + c;
  float param = p.param[k], m = p.exp_avg[k], v = p.exp_avg_sq[k];
  // the trainer's grad /= bsz, fused: PyTorch divides a float tensor by a host
  // scalar as a multiplication by the scalar's float reciprocal
  adam_element(param, __fmul_rn(p.grad[e], p.grad_scale), m, v, p.lr, p.b1, p.b2, p.eps);
  p.param[k] = param;
  p.exp_avg[k] = m;
  p.exp_avg_sq[k] = v;
}

}  // namespace

int launch_adam(const AdamParams& p, cudaStream_t st) {
  const int64_t n = p.rows ? p.n_rows * p.M : p.N * p.M;
  if (n <= 0) return 0;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (p.rows)
    adam_rows_kernel<<<blocks, 256, 0, st>>>(p);
  else
    adam_dense_kernel<<<blocks, 256, 0, st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace blitz
