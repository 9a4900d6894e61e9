// attention_d128.cu — non-causal attention with head_dim 128, the camera
// head's variant (GpuContext::attention's "attention_d128" pipeline,
// src/engine/ops.rs:233-237, shaders/attention.wesl with DV = 32).
//
// The camera head runs it in f32 over one sequence of N*17 prefix tokens per
// head (src/model/camera_head.rs:68-72): a few thousand tokens, tens of GFLOP.
// It keeps the reference's f32 arithmetic on the CUDA cores instead of
// rounding to a 16-bit tensor-core type: at this size the op is latency-
// bound, and f32 keeps it within f32 rounding of the reference.
//
// Layout: a block owns 64 queries of one (s, h) sequence, two threads per
// query (dims [0, 64) and [64, 128)); the sequence's keys stream through
// shared memory in tiles of 32 keys (K and V, converted to f32 on the way
// in).  Scores of a tile are formed first (a 64-dim partial dot per thread,
// one shuffle to join the halves), then one online-softmax update per tile:
// running max, rescale of the accumulator and sum by 2^(m_old - m_new),
// P = 2^(s*scale*log2e - m_new).  Every thread keeps 64 q and 64 accumulator
// values in registers.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "hs_internal.h"

namespace hs {
namespace {

constexpr int kQ = 64;       // queries per block
constexpr int kKeys = 32;    // keys per shared-memory tile
constexpr int kDim = 128;
constexpr int kThreads = 2 * kQ;

template <typename T>
__device__ __forceinline__ void load8f(const T* p, float* v) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if constexpr (std::is_same<T, __half>::value)
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store8f(T* p, const float* v) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __half>::value) {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Row (s, h, t) of a tensor whose 128-element rows sit at the strides of `l`.
struct Rows128 {
  uint64_t t, h, s;
  __device__ uint64_t at(uint64_t s_, uint64_t h_, uint64_t t_) const { return s_ * s + h_ * h + t_ * t; }
};

template <typename T>
__global__ void __launch_bounds__(kThreads) attention_d128_kernel(const T* __restrict__ q, Rows128 lq,
                                                                  const T* __restrict__ k, Rows128 lk,
                                                                  const T* __restrict__ v, Rows128 lv,
                                                                  T* __restrict__ out, Rows128 lo, uint32_t heads,
                                                                  uint32_t t_len, float scale_log2) {
  __shared__ __align__(16) float ks[kKeys][kDim];
  __shared__ __align__(16) float vs[kKeys][kDim];
  const uint32_t seq = blockIdx.y;
  const uint32_t sidx = seq / heads, hidx = seq % heads;
  const int tid = threadIdx.x;
  const int half = tid & 1;
  const uint32_t query = blockIdx.x * kQ + (tid >> 1);
  const bool valid = query < t_len;

  float qv[64], acc[64];
  if (valid) {
    const T* qr = q + lq.at(sidx, hidx, query) + 64 * half;
#pragma unroll
    for (int i = 0; i < 64; i += 8) load8f(qr + i, qv + i);
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) qv[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    qv[i] *= scale_log2;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;

  for (uint32_t k0 = 0; k0 < t_len; k0 += kKeys) {
    __syncthreads();  // the previous tile's readers are done
    // 32 keys x 128 dims of K and of V: 512 8-element granules each, 4 per thread.
    for (int g = tid; g < kKeys * kDim / 8; g += kThreads) {
      const int key = g / (kDim / 8), col = (g % (kDim / 8)) * 8;
      float kb[8], vb[8];
      if (k0 + key < t_len) {
        load8f(k + lk.at(sidx, hidx, k0 + key) + col, kb);
        load8f(v + lv.at(sidx, hidx, k0 + key) + col, vb);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) kb[i] = vb[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ks[key][col + i] = kb[i];
        vs[key][col + i] = vb[i];
      }
    }
    __syncthreads();
    const int n_keys = static_cast<int>(min(static_cast<uint32_t>(kKeys), t_len - k0));
    float s[kKeys];
    float m_tile = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      const float4* kr = reinterpret_cast<const float4*>(&ks[j][64 * half]);
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 kk = kr[i];
        d0 = fmaf(qv[4 * i], kk.x, d0);
        d1 = fmaf(qv[4 * i + 1], kk.y, d1);
        d2 = fmaf(qv[4 * i + 2], kk.z, d2);
        d3 = fmaf(qv[4 * i + 3], kk.w, d3);
      }
      float d = (d0 + d1) + (d2 + d3);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      s[j] = j < n_keys ? d : -INFINITY;
      m_tile = fmaxf(m_tile, s[j]);
    }
    const float m_new = fmaxf(m, m_tile);
    const float corr = exp2f(m - m_new);  // 0 on the first tile (m = -inf)
    l *= corr;
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] *= corr;
#pragma unroll
    for (int j = 0; j < kKeys; ++j) {
      const float p = exp2f(s[j] - m_new);
      l += p;
      const float4* vr = reinterpret_cast<const float4*>(&vs[j][64 * half]);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 vv = vr[i];
        acc[4 * i] = fmaf(p, vv.x, acc[4 * i]);
        acc[4 * i + 1] = fmaf(p, vv.y, acc[4 * i + 1]);
        acc[4 * i + 2] = fmaf(p, vv.z, acc[4 * i + 2]);
        acc[4 * i + 3] = fmaf(p, vv.w, acc[4 * i + 3]);
      }
    }
    m = m_new;
  }
  if (!valid) return;
  const float inv_l = 1.0f / l;
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] *= inv_l;
  T* orow = out + lo.at(sidx, hidx, query) + 64 * half;
#pragma unroll
  for (int i = 0; i < 64; i += 8) store8f(orow + i, acc + i);
}

template <typename T>
cudaError_t run_d128(cudaStream_t st, const AttnIO& io, uint32_t S, uint32_t H, uint32_t T_len, float scale) {
  auto rows = [](const RowLayout& l) { return Rows128{l.t, l.h, l.s}; };
  const dim3 grid((T_len + kQ - 1) / kQ, S * H);
  attention_d128_kernel<T><<<grid, kThreads, 0, st>>>(
      static_cast<const T*>(io.q), rows(io.lq), static_cast<const T*>(io.k), rows(io.lk),
      static_cast<const T*>(io.v), rows(io.lv), static_cast<T*>(io.out), rows(io.lo), H, T_len,
      scale * 1.4426950408889634f);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_d128(cudaStream_t stream, int code, const AttnIO& io, uint32_t S, uint32_t H, uint32_t T,
                                  float scale) {
  if (static_cast<uint64_t>(S) * H * T == 0) return cudaSuccess;
  switch (code) {
    case kF16: return run_d128<__half>(stream, io, S, H, T, scale);
    case kBF16: return run_d128<__nv_bfloat16>(stream, io, S, H, T, scale);
    default: return run_d128<float>(stream, io, S, H, T, scale);
  }
}

}  // namespace hs
