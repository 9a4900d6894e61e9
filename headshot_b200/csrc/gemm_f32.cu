// gemm_f32.cu — hs_linear for f32 storage: out (M, N) = x (M, K) · w (N, K)ᵀ
// + bias, then the fused element-wise op (none, GELU, LayerScale residual),
// all in f32 on the CUDA cores.
//
// The reference's f32 linear (linear.wesl, used by DINO and the camera head,
// which always run f32) is f32 arithmetic, and its own test holds it to 1e-4
// against an f64 sum (kernels.rs:63-100, K = 53).  A tensor-core TF32 product
// rounds each operand to a 10-bit mantissa and misses that by orders of
// magnitude, so this path stays on f32 FMAs: any M, K, N, no alignment rule.
//
// Tiling: a 256-thread block owns a 128 x 128 output tile; K advances in
// slices of 8 staged in shared memory k-major (As[k][m], Bs[k][n]) and double
// buffered (the next slice's global loads are in registers while the current
// one is multiplied).  Thread (ty, tx) accumulates the 8 x 8 outputs of rows
// {4ty..4ty+3, 64+4ty..64+4ty+3} and columns {4tx.., 64+4tx..}, read as float4
// from shared memory.
#include <math.h>
#include <stdint.h>

#include "hs_internal.h"

namespace hs {
namespace {

constexpr int kTM = 128, kTN = 128, kTK = 8;
constexpr int kThreads = 256;

// Abramowitz & Stegun 7.1.26 erf inside GELU (the formula of gelu.wesl),
// with IEEE division and expf.
__device__ __forceinline__ float gelu_erf(float v) {
  const float x = v * 0.70710678118654752f;
  const float a = fabsf(x);
  const float t = 1.0f / fmaf(0.3275911f, a, 1.0f);
  float p = fmaf(1.061405429f, t, -1.453152027f);
  p = fmaf(p, t, 1.421413741f);
  p = fmaf(p, t, -0.284496736f);
  p = fmaf(p, t, 0.254829592f);
  const float e = 1.0f - p * t * expf(-a * a);
  return 0.5f * v * (1.0f + copysignf(e, x));
}

__global__ void __launch_bounds__(kThreads) gemm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ out,
                                                            uint64_t m, uint32_t k, uint32_t n, int epi,
                                                            const float* __restrict__ res,
                                                            const float* __restrict__ gamma) {
  __shared__ __align__(16) float As[2][kTK][kTM];
  __shared__ __align__(16) float Bs[2][kTK][kTN];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const uint64_t m0 = static_cast<uint64_t>(blockIdx.y) * kTM;
  const uint32_t n0 = blockIdx.x * kTN;
  // Global -> shared: each thread moves 4 consecutive k of one row of A and of B.
  const int lr = tid >> 1, lk = (tid & 1) * 4;
  const uint64_t a_row = m0 + lr;
  const uint64_t b_row = n0 + lr;
  float ra[4], rb[4];
  auto fetch = [&](uint32_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t kk = k0 + lk + i;
      ra[i] = (a_row < m && kk < k) ? __ldg(x + a_row * k + kk) : 0.f;
      rb[i] = (b_row < n && kk < k) ? __ldg(w + b_row * k + kk) : 0.f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[buf][lk + i][lr] = ra[i];
      Bs[buf][lk + i][lr] = rb[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const uint32_t slices = (k + kTK - 1) / kTK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (uint32_t s = 0; s < slices; ++s) {
    const int buf = s & 1;
    if (s + 1 < slices) fetch((s + 1) * kTK);
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + 4 * tx]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (s + 1 < slices) {
      stash(buf ^ 1);  // the other buffer was last read one slice ago, before the barrier below
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint64_t row = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + (i - 4));
    if (row >= m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t col = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + (j - 4));
      if (col >= n) continue;
      float v = acc[i][j] + (bias ? bias[col] : 0.f);
      if (epi == kEpiGelu) {
        v = gelu_erf(v);
      } else if (epi == kEpiResidual) {
        v = res[row * n + col] + gamma[col] * v;
      }
      out[row * n + col] = v;
    }
  }
}

}  // namespace

cudaError_t launch_linear_f32(cudaStream_t stream, const float* x, const float* w, const float* bias, float* out,
                              uint64_t m, uint32_t k, uint32_t n, int epi, const float* res, const float* gamma) {
  if (m == 0 || n == 0) return cudaSuccess;
  const uint64_t row_tiles = (m + kTM - 1) / kTM;
  if (row_tiles > 65535u) return cudaErrorInvalidValue;
  const dim3 grid((n + kTN - 1) / kTN, static_cast<unsigned>(row_tiles));
  gemm_f32_kernel<<<grid, kThreads, 0, stream>>>(x, w, bias, out, m, k, n, epi, res, gamma);
  return cudaGetLastError();
}

}  // namespace hs
