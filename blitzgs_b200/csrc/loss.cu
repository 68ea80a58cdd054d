// Fused L1 + SSIM over one image band, forward and backward.
//
// Semantics follow the reference loss (utils/loss_utils.py:83-124, called
// from gaussian_renderer/loss_distribution.py:220-263): per channel, an 11x11
// Gaussian window (sigma 1.5) applied as a depthwise convolution with zero
// padding at the band edges to img, gt, img^2, gt^2 and img*gt, then
//   SSIM = (2 mu1 mu2 + C1)(2 s12 + C2) / ((mu1^2 + mu2^2 + C1)(s11 + s22 + C2)),
// C1 = 0.01^2, C2 = 0.03^2.  The forward returns sum |img - gt| and sum SSIM
// over the band (accumulated in double) and keeps, per pixel and channel, the
// three partial derivatives of the SSIM map with respect to mu1, E[x^2] and
// E[xy]; the backward applies the (symmetric) window to those partials:
//   dL/dx = s_l1 sign(x - y) + s_ssim (W*P1 + 2 x W*P2 + y W*P3).
// The window is separable (the reference's 2D window is the outer product of
// the 1D one), so each pass costs 2 x 11 taps instead of 121.
//
// One CTA computes a 32x32 output tile of one channel; input halos (42x42)
// and the horizontal pass live in shared memory.
#include "common.cuh"
#include "kernels.h"

namespace blitz {

namespace {

constexpr int kLT = 32;              // output tile edge
constexpr int kHalo = 5;             // window radius
constexpr int kIn = kLT + 2 * kHalo; // 42
constexpr int kLossThreads = 256;
constexpr float kC1 = 0.01f * 0.01f;
constexpr float kC2 = 0.03f * 0.03f;

struct Win {
  float w[11];
};

__device__ __forceinline__ float load_gt(const LossParams& p, int64_t idx) {
  if (p.gt_u8) return fminf(fmaxf((float)p.gt_u8[idx] / 255.0f, 0.0f), 1.0f);
  return p.gt_f32[idx];
}

__global__ void __launch_bounds__(kLossThreads) loss_fwd_kernel(LossParams p, Win win, double* sums) {
  __shared__ float s_x[kIn][kIn + 1];
  __shared__ float s_y[kIn][kIn + 1];
  __shared__ float h[5][kIn][kLT + 1];
  __shared__ double s_red[2][8];

  const int c = blockIdx.z;
  const int x0 = blockIdx.x * kLT, y0 = blockIdx.y * kLT;
  const int64_t plane = (int64_t)p.Hb * p.W;
  const float* img = p.img + c * plane;
  const int tid = threadIdx.x;

  for (int k = tid; k < kIn * kIn; k += kLossThreads) {
    const int r = k / kIn, q = k % kIn;
    const int gy = y0 - kHalo + r, gx = x0 - kHalo + q;
    float xv = 0.f, yv = 0.f;
    if (gy >= 0 && gy < p.Hb && gx >= 0 && gx < p.W) {
      const int64_t idx = (int64_t)gy * p.W + gx;
      xv = img[idx];
      yv = load_gt(p, c * plane + idx);
    }
    s_x[r][q] = xv;
    s_y[r][q] = yv;
  }
  __syncthreads();
  // horizontal pass over all 42 input rows, 32 output columns; a thread
  // computes 4 neighbouring outputs of a row from 14 inputs held in
  // registers (each output sums its 11 taps in the same order as a
  // one-output loop, so the result is unchanged)
  for (int k = tid; k < kIn * (kLT / 4); k += kLossThreads) {
    const int r = k / (kLT / 4), q0 = (k % (kLT / 4)) * 4;
    float xs[14], ys[14];
#pragma unroll
    for (int u = 0; u < 14; ++u) {
      xs[u] = s_x[r][q0 + u];
      ys[u] = s_y[r][q0 + u];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = 0.f, b = 0.f, aa = 0.f, bb = 0.f, ab = 0.f;
#pragma unroll
      for (int t = 0; t < 11; ++t) {
        const float xv = xs[j + t], yv = ys[j + t], w = win.w[t];
        a += w * xv;
        b += w * yv;
        aa += w * (xv * xv);
        bb += w * (yv * yv);
        ab += w * (xv * yv);
      }
      h[0][r][q0 + j] = a;
      h[1][r][q0 + j] = b;
      h[2][r][q0 + j] = aa;
      h[3][r][q0 + j] = bb;
      h[4][r][q0 + j] = ab;
    }
  }
  __syncthreads();
  double l1 = 0.0, ss = 0.0;
  // vertical pass and SSIM: a thread takes 4 vertically neighbouring outputs
  // of one column (consecutive threads: consecutive columns)
  for (int k = tid; k < (kLT / 4) * kLT; k += kLossThreads) {
    const int r0 = (k / kLT) * 4, q = k % kLT;
    float m[5][4];
#pragma unroll
    for (int c5 = 0; c5 < 5; ++c5) {
      float v[14];
#pragma unroll
      for (int u = 0; u < 14; ++u) v[u] = h[c5][r0 + u][q];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 11; ++t) acc += win.w[t] * v[j + t];
        m[c5][j] = acc;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = r0 + j;
      const int gy = y0 + r, gx = x0 + q;
      if (gy >= p.Hb || gx >= p.W) continue;
      const float mu1 = m[0][j], mu2 = m[1][j], e11 = m[2][j], e22 = m[3][j], e12 = m[4][j];
      const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2, mu12 = mu1 * mu2;
      const float s11 = e11 - mu1_sq, s22 = e22 - mu2_sq, s12 = e12 - mu12;
      const float A1 = 2.f * mu12 + kC1, A2 = 2.f * s12 + kC2;
      const float B1 = mu1_sq + mu2_sq + kC1, B2 = s11 + s22 + kC2;
      // one rounded reciprocal of D = B1 B2 serves the four quotients
      // (1 / B2 = B1 / D)
      const float inv_D = __frcp_rn(B1 * B2);
      const float S = (A1 * A2) * inv_D;
      const float dmu1 = (2.f * mu2 * (A2 - A1) - S * 2.f * mu1 * (B2 - B1)) * inv_D;
      const float de11 = -S * (B1 * inv_D);
      const float de12 = 2.f * A1 * inv_D;
      const float xv = s_x[r + kHalo][q + kHalo], yv = s_y[r + kHalo][q + kHalo];
      l1 += fabsf(xv - yv);
      ss += S;
      float* pp = p.partials + 3 * (c * plane + (int64_t)gy * p.W + gx);
      pp[0] = dmu1;
      pp[1] = de11;
      pp[2] = de12;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if ((tid & 31) == 0) {
    s_red[0][tid >> 5] = l1;
    s_red[1][tid >> 5] = ss;
  }
  __syncthreads();
  if (tid == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kLossThreads / 32; ++w) {
      a += s_red[0][w];
      b += s_red[1][w];
    }
    atomicAdd(sums + 0, a);
    atomicAdd(sums + 1, b);
  }
}

__global__ void __launch_bounds__(kLossThreads) loss_bwd_kernel(LossBwdParams bp, Win win) {
  const LossParams& p = bp.f;
  __shared__ float s_p[3][kIn][kIn + 1];
  __shared__ float h[3][kLT + 2 * kHalo][kLT + 1];
  const int c = blockIdx.z;
  const int x0 = blockIdx.x * kLT, y0 = blockIdx.y * kLT;
  const int64_t plane = (int64_t)p.Hb * p.W;
  const int tid = threadIdx.x;
  for (int k = tid; k < kIn * kIn; k += kLossThreads) {
    const int r = k / kIn, q = k % kIn;
    const int gy = y0 - kHalo + r, gx = x0 - kHalo + q;
    float a = 0.f, b = 0.f, d = 0.f;
    if (gy >= 0 && gy < p.Hb && gx >= 0 && gx < p.W) {
      const float* pp = p.partials + 3 * (c * plane + (int64_t)gy * p.W + gx);
      a = pp[0];
      b = pp[1];
      d = pp[2];
    }
    s_p[0][r][q] = a;
    s_p[1][r][q] = b;
    s_p[2][r][q] = d;
  }
  __syncthreads();
  // horizontal pass: 4 neighbouring outputs of a row per thread, from 14
  // inputs in registers (per output the same tap order as a one-output loop)
  for (int k = tid; k < kIn * (kLT / 4); k += kLossThreads) {
    const int r = k / (kLT / 4), q0 = (k % (kLT / 4)) * 4;
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      float v[14];
#pragma unroll
      for (int u = 0; u < 14; ++u) v[u] = s_p[m][r][q0 + u];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 11; ++t) acc += win.w[t] * v[j + t];
        h[m][r][q0 + j] = acc;
      }
    }
  }
  __syncthreads();
  const float s_l1 = bp.scale[0], s_ss = bp.scale[1];
  // vertical pass: 4 vertically neighbouring outputs of a column per thread
  for (int k = tid; k < (kLT / 4) * kLT; k += kLossThreads) {
    const int r0 = (k / kLT) * 4, q = k % kLT;
    float qs[3][4];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      float v[14];
#pragma unroll
      for (int u = 0; u < 14; ++u) v[u] = h[m][r0 + u][q];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 11; ++t) acc += win.w[t] * v[j + t];
        qs[m][j] = acc;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gy = y0 + r0 + j, gx = x0 + q;
      if (gy >= p.Hb || gx >= p.W) continue;
      const int64_t idx = c * plane + (int64_t)gy * p.W + gx;
      const float xv = p.img[idx];
      const float yv = load_gt(p, idx);
      const float diff = xv - yv;
      const float sg = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
      bp.dL_dimg[idx] = s_l1 * sg + s_ss * (qs[0][j] + 2.f * xv * qs[1][j] + yv * qs[2][j]);
    }
  }
}

// The per-camera loss of the training step
//   loss = (1 - l) * (L1 / N3) + l * (1 - SSIM / N3) + w * reg / max(cnt, 1)
// (gaussian_renderer/loss_distribution.py:307-322 with the min-scale term as
// a sum and a count), evaluated once on the device in float32, rounding step
// by step as PyTorch's CUDA kernels evaluate the same expression on 0-dim
// float32 tensors: a Python float enters as float32, and a division by a
// Python number is a multiplication by its float32 reciprocal (PyTorch's
// true-division kernel takes that shortcut for a host scalar divisor).
// out = {loss, L1, SSIM, reg, cnt}.
__global__ void loss_combine_kernel(LossCombineParams p) {
  const float inv_n3 = __fdiv_rn(1.0f, p.n3);
  const float l1 = (float)p.sums[0];
  const float ss = (float)p.sums[1];
  float loss = __fadd_rn(__fmul_rn(p.one_minus_lambda, __fmul_rn(l1, inv_n3)),
                         __fmul_rn(p.lambda, __fsub_rn(1.0f, __fmul_rn(ss, inv_n3))));
  float reg = 0.f, cnt = 0.f;
  if (p.reg) {
    reg = (float)p.reg[0];
    cnt = (float)p.reg[1];
    loss = __fadd_rn(loss, __fdiv_rn(__fmul_rn(p.reg_weight, reg), fmaxf(cnt, 1.0f)));
  }
  p.out[0] = loss;
  p.out[1] = l1;
  p.out[2] = ss;
  p.out[3] = reg;
  p.out[4] = cnt;
}

// Gradients of the sums from the upstream gradients of {loss, L1, SSIM}, as
// PyTorch's autograd forms them for the expression above:
//   dsum L1 = (g * (1 - l)) * (1/N3) + g_L1,
//   dsum SSIM = -(g * l) * (1/N3) + g_SSIM,  dreg = (g / max(cnt, 1)) * w.
// scales = {dsum L1, dsum SSIM, dreg}; a NULL upstream pointer counts as 0.
__global__ void loss_combine_bwd_kernel(LossCombineParams p, const float* g_loss, const float* g_l1,
                                        const float* g_ss, float* scales) {
  const float inv_n3 = __fdiv_rn(1.0f, p.n3);
  const float g = g_loss ? *g_loss : 0.f;
  float s0 = __fmul_rn(__fmul_rn(g, p.one_minus_lambda), inv_n3);
  float s1 = __fmul_rn(-__fmul_rn(g, p.lambda), inv_n3);
  if (g_l1) s0 = __fadd_rn(s0, *g_l1);
  if (g_ss) s1 = __fadd_rn(s1, *g_ss);
  scales[0] = s0;
  scales[1] = s1;
  scales[2] = __fmul_rn(__fdiv_rn(g, fmaxf(p.out[4], 1.0f)), p.reg_weight);
}

}  // namespace

int launch_loss_combine(const LossCombineParams& p, cudaStream_t st) {
  loss_combine_kernel<<<1, 1, 0, st>>>(p);
  return (int)cudaGetLastError();
}

int launch_loss_combine_bwd(const LossCombineParams& p, const float* g_loss, const float* g_l1, const float* g_ss,
                            float* scales, cudaStream_t st) {
  loss_combine_bwd_kernel<<<1, 1, 0, st>>>(p, g_loss, g_l1, g_ss, scales);
  return (int)cudaGetLastError();
}

int launch_loss_fwd(const LossParams& p, const float* window11, double* sums, cudaStream_t st) {
  if (p.C <= 0 || p.Hb <= 0 || p.W <= 0) return 0;
  Win w;
  for (int i = 0; i < 11; ++i) w.w[i] = window11[i];
  dim3 grid((p.W + kLT - 1) / kLT, (p.Hb + kLT - 1) / kLT, p.C);
  loss_fwd_kernel<<<grid, kLossThreads, 0, st>>>(p, w, sums);
  return (int)cudaGetLastError();
}

int launch_loss_bwd(const LossBwdParams& p, const float* window11, cudaStream_t st) {
  if (p.f.C <= 0 || p.f.Hb <= 0 || p.f.W <= 0) return 0;
  Win w;
  for (int i = 0; i < 11; ++i) w.w[i] = window11[i];
  dim3 grid((p.f.W + kLT - 1) / kLT, (p.f.Hb + kLT - 1) / kLT, p.f.C);
  loss_bwd_kernel<<<grid, kLossThreads, 0, st>>>(p, w);
  return (int)cudaGetLastError();
}

}  // namespace blitz
