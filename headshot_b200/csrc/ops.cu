// ops.cu — memory-bound companions of the attention op:
//   qk_prep      Q' and K' = RoPE(LN(x)) (and plain 16-bit casts), one pass over HBM
//   layernorm    GpuContext::layernorm  (src/engine/ops.rs:130-153, shaders/layernorm.wesl)
//   rope_apply   GpuContext::rope_apply (src/engine/ops.rs:202-223, shaders/rope_apply.wesl)
//   split_heads  GpuContext::split_heads (src/engine/ops.rs:185-200, shaders/split_heads.wesl)
//   attn_merge   GpuContext::attn_merge  (src/engine/ops.rs:255-267, shaders/attn_merge.wesl)
// Storage may be f32, f16 or bf16; all arithmetic is f32.
#include <algorithm>
#include <type_traits>

#include "hs_internal.h"
#include "hs_ptx.cuh"

namespace hs {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ T cvt_to(float f);
template <>
__device__ __forceinline__ float cvt_to<float>(float f) { return f; }
template <>
__device__ __forceinline__ __half cvt_to<__half>(float f) { return __float2half_rn(f); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_to<__nv_bfloat16>(float f) { return __float2bfloat16_rn(f); }

// Eight consecutive elements <-> f32.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
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
      const float2 f = Elem<T>::unpack2(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// Squared norm of 8 values as a T store would round them.
template <typename T>
__device__ __forceinline__ float stored_norm2(const float (&v)[8]) {
  float n2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    float2 r;
    if constexpr (sizeof(T) == 4) {
      r = make_float2(v[i], v[i + 1]);
    } else {
      r = Elem<T>::unpack2(Elem<T>::pack2(v[i], v[i + 1]));
    }
    n2 = fmaf(r.x, r.x, n2);
    n2 = fmaf(r.y, r.y, n2);
  }
  return n2;
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    u.x = Elem<T>::pack2(v[0], v[1]);
    u.y = Elem<T>::pack2(v[2], v[3]);
    u.z = Elem<T>::pack2(v[4], v[5]);
    u.w = Elem<T>::pack2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

constexpr int kPrepTokens = 32;     // tokens per block (8 threads per 64-wide row)
constexpr int kPrepSeqPerBlock = 16;  // sequences (s, h) a block sweeps with one staged table slice
constexpr int kGlueUnroll = 4;      // independent 16-byte loads in flight per thread in the glue kernels

// One thread's 8 elements of a 64-wide row: [4g, 4g+4) and their RoPE
// partners [32+4g, 36+4g), raw as stored (8 bytes each half for 16-bit, 16
// for f32).
template <typename In>
struct RawHalves {
  static constexpr bool kF32 = sizeof(In) == 4;
  using Half = typename std::conditional<kF32, uint4, uint2>::type;
  Half lo, hi;
  __device__ __forceinline__ void load(const In* row, int g) {
    lo = __ldg(reinterpret_cast<const Half*>(row + 4 * g));
    hi = __ldg(reinterpret_cast<const Half*>(row + 32 + 4 * g));
  }
  __device__ __forceinline__ void zero() {
    if constexpr (kF32) {
      lo = hi = make_uint4(0u, 0u, 0u, 0u);
    } else {
      lo = hi = make_uint2(0u, 0u);
    }
  }
  // v[0..3] = elements 4g..4g+3, v[4..7] = elements 32+4g..35+4g.
  __device__ __forceinline__ void to_float(float (&v)[8]) const {
    if constexpr (kF32) {
      v[0] = __uint_as_float(lo.x); v[1] = __uint_as_float(lo.y); v[2] = __uint_as_float(lo.z);
      v[3] = __uint_as_float(lo.w); v[4] = __uint_as_float(hi.x); v[5] = __uint_as_float(hi.y);
      v[6] = __uint_as_float(hi.z); v[7] = __uint_as_float(hi.w);
    } else {
      const uint32_t w[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = Elem<In>::unpack2(w[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  }
};

// Stores v (layout of RawHalves::to_float) at row + 4g and row + 32 + 4g and
// returns the squared norm of the values as stored (after rounding).
template <typename Out>
__device__ __forceinline__ float store_halves(Out* row, int g, const float (&v)[8]) {
  float n2 = 0.f;
  if constexpr (sizeof(Out) == 4) {
    *reinterpret_cast<float4*>(row + 4 * g) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(row + 32 + 4 * g) = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
    for (int i = 0; i < 8; ++i) n2 = fmaf(v[i], v[i], n2);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = Elem<Out>::pack2(v[2 * i], v[2 * i + 1]);
      const float2 r = Elem<Out>::unpack2(w[i]);
      n2 = fmaf(r.x, r.x, n2);
      n2 = fmaf(r.y, r.y, n2);
    }
    *reinterpret_cast<uint2*>(row + 4 * g) = make_uint2(w[0], w[1]);
    *reinterpret_cast<uint2*>(row + 32 + 4 * g) = make_uint2(w[2], w[3]);
  }
  return n2;
}

// Q' or K' = RoPE(LN(x)) over (SH, T, 64).  A block owns kPrepTokens
// consecutive tokens of up to kPrepSeqPerBlock sequences.  Eight threads per
// row; thread g holds elements [4g, 4g+4) and their rotate-half partners
// [32+4g, 36+4g), so RoPE needs no exchange between threads, and the table
// values of its 8 columns, which depend on the token only, are loaded once
// and reused for every sequence.  Each thread issues the loads of all its
// rows before any arithmetic, so enough bytes are in flight for HBM.
template <typename In, typename Out>
__global__ void __launch_bounds__(256) qk_prep_kernel(PrepJobs jobs, uint32_t sh, uint32_t heads, uint32_t t) {
  // blockIdx.z picks the tensor (q, k, v casts) of this launch.
  const PrepJob& job = jobs.job[blockIdx.z];
  const In* __restrict__ x = static_cast<const In*>(job.x);
  Out* __restrict__ out = static_cast<Out*>(job.out);
  const RowLayout lx = job.lx;
  const QkPrologue& p = job.p;
  constexpr int kRows = sizeof(In) == 4 ? kPrepSeqPerBlock / 2 : kPrepSeqPerBlock;  // rows per pass
  const int lt = threadIdx.x >> 3;  // token within the block
  const int g = threadIdx.x & 7;
  const uint32_t tok = blockIdx.x * kPrepTokens + lt;
  const bool tok_ok = tok < t;
  const uint32_t seq0 = blockIdx.y * kPrepSeqPerBlock;
  const uint32_t seq_end = min(sh, seq0 + kPrepSeqPerBlock);
  // Input row of sequence q = s*heads + h in its own layout; output rows are head-major.
  auto in_at = [&](uint32_t q) { return lx.at(q / heads, q % heads, tok); };
  auto row_at = [&](uint32_t q) { return (static_cast<uint64_t>(q) * t + tok) * 64; };

  RawHalves<In> raw[kRows];
#pragma unroll
  for (int u = 0; u < kRows; ++u) {
    if (tok_ok && seq0 + u < seq_end) raw[u].load(x + in_at(seq0 + u), g);
    else raw[u].zero();
  }
  // This thread's table columns (pass-through rows: sin 0, cos 1).  Scalar
  // loads: the tables come through the C ABI with only 4-byte alignment.
  float sn[8], cs[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sn[i] = 0.f;
    cs[i] = 1.f;
  }
  if (p.rope && tok_ok) {
    const uint32_t ft = (tok + p.pos_offset) % p.tokens_per_frame;
    if (ft >= p.prefix) {
      const uint64_t r = static_cast<uint64_t>(ft - p.prefix) * 64;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sn[i] = __ldg(p.sin_t + r + 4 * g + i);
        sn[4 + i] = __ldg(p.sin_t + r + 32 + 4 * g + i);
        cs[i] = __ldg(p.cos_t + r + 4 * g + i);
        cs[4 + i] = __ldg(p.cos_t + r + 32 + 4 * g + i);
      }
    }
  }
  float w[8], bb[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w[i] = p.ln ? __ldg(p.ln_w + 4 * g + i) : 1.f;
    w[4 + i] = p.ln ? __ldg(p.ln_w + 32 + 4 * g + i) : 1.f;
    bb[i] = p.ln ? __ldg(p.ln_b + 4 * g + i) : 0.f;
    bb[4 + i] = p.ln ? __ldg(p.ln_b + 32 + 4 * g + i) : 0.f;
  }
  float n2_max = 0.f;
  for (uint32_t q0 = seq0; q0 < seq_end; q0 += kRows) {
    if (q0 != seq0) {  // f32 storage: a second pass over the block's sequences
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        if (tok_ok && q0 + u < seq_end) raw[u].load(x + in_at(q0 + u), g);
        else raw[u].zero();
      }
    }
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      float v[8];
      raw[u].to_float(v);
      if (p.ln) {
        float sm = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) sm += v[i];
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        sm += __shfl_xor_sync(0xffffffffu, sm, 4);
        const float mu = sm * (1.0f / 64);
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = v[i] - mu;
          sq = fmaf(d, d, sq);
        }
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        const float inv = rsqrtf(sq * (1.0f / 64) + p.eps);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (v[i] - mu) * inv * w[i] + bb[i];
      }
      if (p.rope) {
        // lower half: x*cos - x[i+32]*sin ; upper half: x*cos + x[i-32]*sin
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = v[i], hi = v[4 + i];
          v[i] = lo * cs[i] - hi * sn[i];
          v[4 + i] = hi * cs[4 + i] + lo * sn[4 + i];
        }
      }
      const bool row_ok = tok_ok && q0 + u < seq_end;
      float n2 = 0.f;
      if (row_ok) n2 = store_halves(out + row_at(q0 + u), g, v);
      if (p.norm2_max) {  // uniform branch: the row's 8 lanes add their parts
        n2 += __shfl_xor_sync(0xffffffffu, n2, 1);
        n2 += __shfl_xor_sync(0xffffffffu, n2, 2);
        n2 += __shfl_xor_sync(0xffffffffu, n2, 4);
        n2_max = fmaxf(n2_max, n2);
      }
    }
  }
  if (p.norm2_max) {
    // Max across the warp's 4 rows, one atomic per warp (non-negative
    // floats order like their bit patterns).
    n2_max = fmaxf(n2_max, __shfl_xor_sync(0xffffffffu, n2_max, 8));
    n2_max = fmaxf(n2_max, __shfl_xor_sync(0xffffffffu, n2_max, 16));
    if ((threadIdx.x & 31) == 0) atomicMax(p.norm2_max, __float_as_uint(n2_max));
  }
}

// ---- qk_prep for 16-bit rows, staged through shared memory by TMA ----------
//
// Work unit = 32 consecutive tokens of 8 sequences of one tensor.  A block
// takes a contiguous range of units (sequences fastest, so a thread's folded
// table constants, which depend on the token only, are rebuilt only when the
// token block changes) and streams them through two shared-memory stages.
// A ninth warp is the producer: its lane 0 issues the 8 TMA box loads (32
// rows x 128 B each) of unit i+2 into the stage unit i used as soon as all
// eight compute warps have released it (one arrival per warp on the stage's
// `empty` barrier), so HBM reads stay in flight while the block computes and
// the compute warps never wait for one another.  Thread (token, g) computes elements [4g, 4g+4) and
// their rotate-half partners [32+4g, 36+4g) of its token's row in each
// sequence of the unit.  LayerNorm's affine and the RoPE rotation fold into
// three constants per output element (d = x - mean, inv = 1/sqrt(var + eps)):
//   x'[i]    = inv * (A_lo d[i] + B_lo d[i+32]) + C_lo,   A_lo = w[i] cos[i],
//              B_lo = -w[i+32] sin[i],  C_lo = b[i] cos[i] - b[i+32] sin[i]
//   x'[i+32] = inv * (A_hi d[i+32] + B_hi d[i]) + C_hi,   A_hi = w[i+32] cos[i+32],
//              B_hi = w[i] sin[i+32],   C_hi = b[i+32] cos[i+32] + b[i] sin[i+32]
// (pass-through tokens: sin 0, cos 1; no LayerNorm: d = x, inv = 1, w = 1, b = 0).
constexpr int kTpTokens = 32;
constexpr int kTpSeqs = 8;
constexpr int kTpStages = 2;
constexpr uint32_t kTpBoxBytes = kTpTokens * 128;            // 32 rows of 64 16-bit elements
constexpr uint32_t kTpStageBytes = kTpSeqs * kTpBoxBytes;    // 32 KiB
constexpr int kTpThreads = kTpTokens * 8;           // compute threads (8 per 64-wide row)
constexpr int kTpComputeWarps = kTpThreads / 32;
constexpr int kTpBlockThreads = kTpThreads + 32;     // + the producer warp
constexpr int kTpBlocksPerSm = 3;
constexpr size_t kTpSmemBytes = 1024 /*alignment slack*/ + kTpStages * kTpStageBytes + 64;
constexpr int kSitePrepFull = 0x201;

struct TmaPrepArgs {
  PrepJobs jobs;      // x is read through the tensor maps
  uint32_t sh;        // sequences (S * H)
  uint32_t heads;
  uint32_t t;
  uint32_t n_tb;      // token blocks: ceil(t / 32)
  uint32_t n_sc;      // sequence chunks: ceil(sh / 8)
  uint64_t units;     // jobs * n_tb * n_sc
  int* status;
  uint64_t timeout_ns;
};

template <typename E>
__global__ void __launch_bounds__(kTpBlockThreads, kTpBlocksPerSm)
    qk_prep_tma_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1,
                       const __grid_constant__ CUtensorMap tm2, const __grid_constant__ TmaPrepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kTpStages * kTpStageBytes);  // unit landed
  uint64_t* empty = full + kTpStages;  // every compute warp is done with the stage
  int* abort_flag = reinterpret_cast<int*>(empty + kTpStages);

  const uint64_t u_begin = blockIdx.x * a.units / gridDim.x;
  const uint64_t u_end = (blockIdx.x + 1ull) * a.units / gridDim.x;
  const uint32_t per_job = a.n_tb * a.n_sc;

  // Warp w, lane (j, g): token lt = (w & 3) + 4j + 16(w >> 2).  The four rows
  // a warp reads at once are then lt, lt+4, lt+8, lt+12, whose 128-byte
  // swizzle phases put two rows in each half of the banks (two wavefronts per
  // 8-byte read of the warp, the minimum).
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  const int lt = (warp & 3) + 4 * (lane >> 3) + 16 * (warp >> 2);
  const uint32_t sw = static_cast<uint32_t>(lt & 7);
  const uint32_t off_lo = static_cast<uint32_t>(lt) * 128 + ((static_cast<uint32_t>(g >> 1) ^ sw) << 4) + (g & 1) * 8;
  const uint32_t off_hi =
      static_cast<uint32_t>(lt) * 128 + ((static_cast<uint32_t>(4 + (g >> 1)) ^ sw) << 4) + (g & 1) * 8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTpComputeWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // Tensor of unit u (units are tensor-major, at most kMaxPrepJobs tensors):
  // two compares instead of a 64-bit division.
  auto job_of = [&](uint64_t u) {
    return static_cast<uint32_t>(u >= per_job) + static_cast<uint32_t>(u >= 2ull * per_job);
  };
  // The producer lane: the TMA loads of unit u into stage `st`.
  auto issue = [&](uint64_t u, int st) {
    const uint32_t job = job_of(u);
    const uint32_t rem = static_cast<uint32_t>(u - static_cast<uint64_t>(job) * per_job);
    const uint32_t tb = rem / a.n_sc;
    const uint32_t q0 = (rem - tb * a.n_sc) * kTpSeqs;
    const uint32_t nq = min(static_cast<uint32_t>(kTpSeqs), a.sh - q0);
    const CUtensorMap* tm = job == 0 ? &tm0 : (job == 1 ? &tm1 : &tm2);
    mbar_arrive_expect_tx(&full[st], nq * kTpBoxBytes);
    for (uint32_t j = 0; j < nq; ++j) {
      const uint32_t q = q0 + j;
      tma_load_4d(tm, &full[st], stages + st * kTpStageBytes + j * kTpBoxBytes, 0,
                  static_cast<int>(tb * kTpTokens), static_cast<int>(q % a.heads), static_cast<int>(q / a.heads));
    }
  };
  if (warp == kTpComputeWarps) {
    if (lane == 0) {
      uint64_t n = 0;  // units issued
      for (uint64_t u = u_begin; u < u_end; ++u, ++n) {
        const int st = static_cast<int>(n % kTpStages);
        if (n >= kTpStages && !mbar_wait(&empty[st], static_cast<uint32_t>(n / kTpStages - 1) & 1u, abort_flag,
                                         a.status, kSitePrepFull, a.timeout_ns))
          break;
        issue(u, st);
      }
      // Let the last loads land before the block can exit (on the normal path
      // the compute warps have consumed them already); fixed teardown bound.
      for (uint64_t k = n > kTpStages ? n - kTpStages : 0; k < n; ++k)
        mbar_wait_teardown(&full[k % kTpStages], static_cast<uint32_t>(k / kTpStages) & 1u, a.status,
                           kSitePrepFull);
    }
    return;
  }

  float cA[8], cB[8], cC[8];  // [0..3] lower-half outputs, [4..7] upper-half outputs
  uint32_t cur_key = 0xffffffffu;
  uint32_t cur_job = 0xffffffffu;
  const PrepJob* job_p = nullptr;
  uint32_t tok = 0;
  bool tok_ok = false;
  // Largest squared row norm this thread stored for the current tensor.  A
  // block's units are tensor-major, so the tensor changes at the same unit
  // for every thread; the block's maxima go out then (one atomic per warp,
  // non-negative floats order like their bit patterns).
  float n2_run = 0.f;
  auto flush_norm = [&](uint32_t jb) {
    unsigned int* dst = a.jobs.job[jb].p.norm2_max;
    if (!dst) return;
    float m = fmaxf(n2_run, __shfl_xor_sync(0xffffffffu, n2_run, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    if (lane == 0 && m > 0.f) atomicMax(dst, __float_as_uint(m));
  };

  uint64_t i = 0;
  for (uint64_t u = u_begin; u < u_end; ++u, ++i) {
    const int st = static_cast<int>(i % kTpStages);
    const uint32_t job = job_of(u);
    const uint32_t rem = static_cast<uint32_t>(u - static_cast<uint64_t>(job) * per_job);
    const uint32_t tb = rem / a.n_sc;
    const uint32_t q0 = (rem - tb * a.n_sc) * kTpSeqs;
    const uint32_t key = job * a.n_tb + tb;
    if (key != cur_key) {  // fold this thread's constants for (job, token)
      cur_key = key;
      if (job != cur_job) {
        if (cur_job != 0xffffffffu) flush_norm(cur_job);
        n2_run = 0.f;
        cur_job = job;
      }
      job_p = &a.jobs.job[job];
      const QkPrologue& p = job_p->p;
      tok = tb * kTpTokens + lt;
      tok_ok = tok < a.t;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = 4 * g + k;
        float sn_lo = 0.f, sn_hi = 0.f, cs_lo = 1.f, cs_hi = 1.f;
        if (p.rope && tok_ok) {
          const uint32_t ft = (tok + p.pos_offset) % p.tokens_per_frame;
          if (ft >= p.prefix) {
            const uint64_t r = static_cast<uint64_t>(ft - p.prefix) * 64;
            sn_lo = __ldg(p.sin_t + r + c);
            sn_hi = __ldg(p.sin_t + r + 32 + c);
            cs_lo = __ldg(p.cos_t + r + c);
            cs_hi = __ldg(p.cos_t + r + 32 + c);
          }
        }
        const float w_lo = p.ln ? __ldg(p.ln_w + c) : 1.f, w_hi = p.ln ? __ldg(p.ln_w + 32 + c) : 1.f;
        const float b_lo = p.ln ? __ldg(p.ln_b + c) : 0.f, b_hi = p.ln ? __ldg(p.ln_b + 32 + c) : 0.f;
        cA[k] = w_lo * cs_lo;
        cB[k] = -w_hi * sn_lo;
        cC[k] = b_lo * cs_lo - b_hi * sn_lo;
        cA[4 + k] = w_hi * cs_hi;
        cB[4 + k] = w_lo * sn_hi;
        cC[4 + k] = b_hi * cs_hi + b_lo * sn_hi;
      }
    }
    // The tensor's flags, read once per unit rather than per row.
    const bool do_ln = job_p->p.ln != 0;
    const bool do_norm = job_p->p.norm2_max != nullptr;
    const float eps = job_p->p.eps;
    E* __restrict__ out = static_cast<E*>(job_p->out);

    const bool ok = mbar_wait(&full[st], static_cast<uint32_t>(i / kTpStages) & 1u, abort_flag, a.status, kSitePrepFull,
                              a.timeout_ns);
    if (ok) {
      const uint8_t* box0 = stages + st * kTpStageBytes;
      const uint32_t nq = min(static_cast<uint32_t>(kTpSeqs), a.sh - q0);
      // Four of the unit's sequences in flight per thread: -3.7 % time at 200 x 16 x 1374
      // against two (71 registers, still three blocks per SM).
#pragma unroll 4
      for (uint32_t j = 0; j < nq; ++j) {
        const uint2 rl = *reinterpret_cast<const uint2*>(box0 + j * kTpBoxBytes + off_lo);
        const uint2 rh = *reinterpret_cast<const uint2*>(box0 + j * kTpBoxBytes + off_hi);
        float v[8];
        {
          const float2 f0 = Elem<E>::unpack2(rl.x), f1 = Elem<E>::unpack2(rl.y);
          const float2 f2 = Elem<E>::unpack2(rh.x), f3 = Elem<E>::unpack2(rh.y);
          v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
          v[4] = f2.x; v[5] = f2.y; v[6] = f3.x; v[7] = f3.y;
        }
        float inv = 1.f;
        if (do_ln) {
          float s0, s1;
          add2(s0, s1, v[0], v[1], v[2], v[3]);
          add2(s0, s1, s0, s1, v[4], v[5]);
          add2(s0, s1, s0, s1, v[6], v[7]);
          float sm = s0 + s1;
          sm += __shfl_xor_sync(0xffffffffu, sm, 1);
          sm += __shfl_xor_sync(0xffffffffu, sm, 2);
          sm += __shfl_xor_sync(0xffffffffu, sm, 4);
          const float nmu = sm * (-1.0f / 64);
#pragma unroll
          for (int k = 0; k < 8; k += 2) add2(v[k], v[k + 1], v[k], v[k + 1], nmu, nmu);
          float q0s, q1s;
          mul2(q0s, q1s, v[0], v[1], v[0], v[1]);
#pragma unroll
          for (int k = 2; k < 8; k += 2) fma2(q0s, q1s, v[k], v[k + 1], v[k], v[k + 1], q0s, q1s);
          float sq = q0s + q1s;
          sq += __shfl_xor_sync(0xffffffffu, sq, 1);
          sq += __shfl_xor_sync(0xffffffffu, sq, 2);
          sq += __shfl_xor_sync(0xffffffffu, sq, 4);
          inv = rsqrtf(sq * (1.0f / 64) + eps);
        }
        // y_lo = inv * (A_lo d_lo + B_lo d_hi) + C_lo ; y_hi = inv * (A_hi d_hi + B_hi d_lo) + C_hi
        float y[8];
#pragma unroll
        for (int k = 0; k < 4; k += 2) {
          float t0, t1;
          mul2(t0, t1, cB[k], cB[k + 1], v[4 + k], v[5 + k]);
          fma2(t0, t1, cA[k], cA[k + 1], v[k], v[k + 1], t0, t1);
          fma2(y[k], y[k + 1], t0, t1, inv, inv, cC[k], cC[k + 1]);
          mul2(t0, t1, cB[4 + k], cB[5 + k], v[k], v[k + 1]);
          fma2(t0, t1, cA[4 + k], cA[5 + k], v[4 + k], v[5 + k], t0, t1);
          fma2(y[4 + k], y[5 + k], t0, t1, inv, inv, cC[4 + k], cC[5 + k]);
        }
        const uint32_t w0 = Elem<E>::pack2(y[0], y[1]), w1 = Elem<E>::pack2(y[2], y[3]);
        const uint32_t w2 = Elem<E>::pack2(y[4], y[5]), w3 = Elem<E>::pack2(y[6], y[7]);
        float n2 = 0.f;
        if (tok_ok) {
          E* row = out + (static_cast<uint64_t>(q0 + j) * a.t + tok) * 64;
          *reinterpret_cast<uint2*>(row + 4 * g) = make_uint2(w0, w1);
          *reinterpret_cast<uint2*>(row + 32 + 4 * g) = make_uint2(w2, w3);
          if (do_norm) {  // squared norm of the values as stored
            const float2 r0 = Elem<E>::unpack2(w0), r1 = Elem<E>::unpack2(w1);
            const float2 r2 = Elem<E>::unpack2(w2), r3 = Elem<E>::unpack2(w3);
            float m0, m1;
            mul2(m0, m1, r0.x, r0.y, r0.x, r0.y);
            fma2(m0, m1, r1.x, r1.y, r1.x, r1.y, m0, m1);
            fma2(m0, m1, r2.x, r2.y, r2.x, r2.y, m0, m1);
            fma2(m0, m1, r3.x, r3.y, r3.x, r3.y, m0, m1);
            n2 = m0 + m1;
          }
        }
        if (do_norm) {  // uniform branch: the row's 8 lanes add their parts
          n2 += __shfl_xor_sync(0xffffffffu, n2, 1);
          n2 += __shfl_xor_sync(0xffffffffu, n2, 2);
          n2 += __shfl_xor_sync(0xffffffffu, n2, 4);
          n2_run = fmaxf(n2_run, n2);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with stage st
    if (__any_sync(0xffffffffu, !ok || *reinterpret_cast<volatile int*>(abort_flag) != 0)) break;
  }

  if (cur_job != 0xffffffffu) flush_norm(cur_job);
}

// One warp per row, any width; two-pass statistics like layernorm.wesl.
template <typename T>
__global__ void __launch_bounds__(256) layernorm_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                        const float* __restrict__ w, const float* __restrict__ b,
                                                        uint64_t rows, uint32_t dim, float eps) {
  const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * dim;
  float s = 0.f;
  for (uint32_t j = lane; j < dim; j += 32) s += ld_f(xr + j);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mu = s / static_cast<float>(dim);
  float q = 0.f;
  for (uint32_t j = lane; j < dim; j += 32) {
    const float d = ld_f(xr + j) - mu;
    q = fmaf(d, d, q);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float inv = rsqrtf(q / static_cast<float>(dim) + eps);
  T* orow = out + row * dim;
  for (uint32_t j = lane; j < dim; j += 32) orow[j] = cvt_to<T>((ld_f(xr + j) - mu) * inv * w[j] + b[j]);
}

// Model-width rows (dim = 256*C, the blocks' norm1/norm2 and the final
// norms): one warp per row held in registers, lane l owning the 8-element
// granules l, l+32, ...; 16-byte loads and stores, the same two-pass
// statistics (mean, then the centred variance) from the registers.
template <typename T, int C>
__global__ void __launch_bounds__(256) layernorm_wide_kernel(const T* __restrict__ x, T* __restrict__ out,
                                                             const float* __restrict__ w,
                                                             const float* __restrict__ b, uint64_t rows,
                                                             float eps) {
  constexpr uint32_t kDim = 256 * C;
  const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * kDim;
  float v[C][8];
#pragma unroll
  for (int c = 0; c < C; ++c) load8(xr + 8 * (lane + 32 * c), v[c]);
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[c][i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mu = s / static_cast<float>(kDim);
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[c][i] -= mu;
      q = fmaf(v[c][i], v[c][i], q);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float inv = rsqrtf(q / static_cast<float>(kDim) + eps);
  T* orow = out + row * kDim;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const uint32_t j = 8 * (lane + 32 * c);
    float wv[8], bv[8];
    load8(w + j, wv);
    load8(b + j, bv);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[c][i] = v[c][i] * inv * wv[i] + bv[i];
    store8(orow + j, v[c]);
  }
}

// One thread per rotation pair, in place (rope_apply.wesl:36-56).
template <typename T>
__global__ void __launch_bounds__(256) rope_apply_kernel(T* __restrict__ x, const float* __restrict__ sin_t,
                                                         const float* __restrict__ cos_t, uint32_t s, uint32_t h,
                                                         uint32_t t, uint32_t d, uint32_t prefix, uint32_t tpf) {
  const uint32_t half = d / 2;
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t total = static_cast<uint64_t>(s) * h * t * half;
  if (i >= total) return;
  const uint32_t dp = static_cast<uint32_t>(i % half);
  const uint64_t tok_flat = i / half;  // (s*h)*t + t
  const uint32_t tok = static_cast<uint32_t>(tok_flat % t);
  const uint32_t ft = tok % tpf;
  if (ft < prefix) return;
  const uint64_t row = static_cast<uint64_t>(ft - prefix) * d;
  const uint64_t base = tok_flat * d + dp;
  const float lo = ld_f(x + base), hi = ld_f(x + base + half);
  x[base] = cvt_to<T>(lo * cos_t[row + dp] - hi * sin_t[row + dp]);
  x[base + half] = cvt_to<T>(hi * cos_t[row + half + dp] + lo * sin_t[row + half + dp]);
}

// (S*T, H*D) <-> (S, H, T, D); `merge` selects the direction.  One thread
// per 16-byte chunk when D allows it, else per element.
template <typename T, int V>
__global__ void __launch_bounds__(256) permute_heads_kernel(const T* __restrict__ x, T* __restrict__ out, uint32_t s,
                                                            uint32_t h, uint32_t t, uint32_t d, int merge) {
  const uint64_t i = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * V;
  const uint64_t total = static_cast<uint64_t>(s) * h * t * d;
  if (i >= total) return;
  // head-major index decode (s, h, t, d)
  const uint32_t dd = static_cast<uint32_t>(i % d);
  const uint64_t r1 = i / d;
  const uint32_t tt = static_cast<uint32_t>(r1 % t);
  const uint64_t r2 = r1 / t;
  const uint32_t hh = static_cast<uint32_t>(r2 % h);
  const uint64_t ss = r2 / h;
  const uint64_t tok = ((ss * t + tt) * h + hh) * d + dd;  // token-major index
  const uint64_t src = merge ? i : tok;
  const uint64_t dst = merge ? tok : i;
  if constexpr (V * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(out + dst) = *reinterpret_cast<const uint4*>(x + src);
  } else {
#pragma unroll
    for (int k = 0; k < V; ++k) out[dst + k] = x[src + k];
  }
}

inline unsigned blocks_for(uint64_t threads, unsigned per_block) {
  return static_cast<unsigned>((threads + per_block - 1) / per_block);
}

template <typename In>
cudaError_t prep_dispatch_out(cudaStream_t stream, const PrepJobs& jobs, int n_jobs, int out_code, uint32_t sh,
                              uint32_t heads, uint32_t t) {
  const dim3 grid((t + kPrepTokens - 1) / kPrepTokens, (sh + kPrepSeqPerBlock - 1) / kPrepSeqPerBlock, n_jobs);
  switch (out_code) {
    case kBF16: qk_prep_kernel<In, __nv_bfloat16><<<grid, 256, 0, stream>>>(jobs, sh, heads, t); break;
    case kF16: qk_prep_kernel<In, __half><<<grid, 256, 0, stream>>>(jobs, sh, heads, t); break;
    default: qk_prep_kernel<In, float><<<grid, 256, 0, stream>>>(jobs, sh, heads, t); break;
  }
  return cudaGetLastError();
}

// The TMA-staged prep, when every tensor of the launch can be described by a
// tensor map (16-byte aligned, row strides multiples of 8 elements);
// *launched stays false otherwise and the caller takes the register kernel.
template <typename E>
cudaError_t prep_tma(cudaStream_t stream, const PrepJobs& jobs, int n_jobs, uint32_t S, uint32_t H, uint32_t t,
                     int* status, uint64_t timeout_ns, bool* launched) {
  CUtensorMap maps[kMaxPrepJobs];
  for (int i = 0; i < n_jobs; ++i) {
    const PrepJob& j = jobs.job[i];
    const RowLayout& l = j.lx;
    if ((reinterpret_cast<uintptr_t>(j.x) & 15u) || (reinterpret_cast<uintptr_t>(j.out) & 15u) || (l.t & 7u) ||
        (l.h & 7u) || (l.s & 7u))
      return cudaSuccess;
    if (!make_row_map(&maps[i], j.x, l, Elem<E>::kBf16, t, H, S, kTpTokens, nullptr)) return cudaSuccess;
  }
  for (int i = n_jobs; i < kMaxPrepJobs; ++i) maps[i] = maps[0];
  TmaPrepArgs a{};
  a.jobs = jobs;
  a.sh = S * H;
  a.heads = H;
  a.t = t;
  a.n_tb = (t + kTpTokens - 1) / kTpTokens;
  a.n_sc = (a.sh + kTpSeqs - 1) / kTpSeqs;
  a.units = static_cast<uint64_t>(n_jobs) * a.n_tb * a.n_sc;
  a.status = status;
  a.timeout_ns = timeout_ns;
  const cudaError_t e =
      ensure_dynamic_smem(reinterpret_cast<const void*>(qk_prep_tma_kernel<E>), static_cast<int>(kTpSmemBytes));
  if (e != cudaSuccess) return e;
  const uint64_t cap = static_cast<uint64_t>(kTpBlocksPerSm) * static_cast<uint64_t>(current_sm_count());
  const unsigned grid = static_cast<unsigned>(a.units < cap ? a.units : cap);
  qk_prep_tma_kernel<E><<<grid, kTpBlockThreads, kTpSmemBytes, stream>>>(maps[0], maps[1], maps[2], a);
  *launched = true;
  return cudaGetLastError();
}

// Row blocks: for g < groups, rows [g*src_stride, +rows) of src go to rows
// [g*dst_stride, +rows) of dst (the trunk's register gather and scatter,
// trunk.rs:109-122, and copy_rows).  16-byte granules; a block of threads
// per (group, granule range).
__global__ void __launch_bounds__(256) copy_row_blocks_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                              uint64_t groups, uint64_t src_stride_g,
                                                              uint64_t dst_stride_g, uint64_t granules_per_group) {
  // Grid-stride over 16-byte granules, kGlueUnroll independent loads in flight per thread
  // before their stores (one load per thread leaves HBM latency uncovered).
  const uint64_t total = groups * granules_per_group;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i0 = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i0 < total;
       i0 += kGlueUnroll * stride) {
    uint4 v[kGlueUnroll];
    uint64_t d[kGlueUnroll];
#pragma unroll
    for (int u = 0; u < kGlueUnroll; ++u) {
      const uint64_t i = i0 + u * stride;
      if (i < total) {
        const uint64_t g = i / granules_per_group, k = i - g * granules_per_group;
        v[u] = __ldg(src + g * src_stride_g + k);
        d[u] = g * dst_stride_g + k;
      }
    }
#pragma unroll
    for (int u = 0; u < kGlueUnroll; ++u)
      if (i0 + u * stride < total) dst[d[u]] = v[u];
  }
}

// Head-input cache row (Cache::build, cache.rs:25-52): out[r] = [f32(a[r]) | f32(b[r])],
// the concat_channels + cast_to_f32 of the frame- and global-block outputs.  The cache is
// written once and read much later, so its stores stream past L2 (st.global.cs).
template <typename T>
__global__ void __launch_bounds__(256) cache_build_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                          float* __restrict__ out, uint64_t rows, uint32_t ca,
                                                          uint32_t cb) {
  const uint32_t ga = ca / 8, gb = cb / 8;  // 8-element granules per row
  const uint64_t total = rows * (ga + gb);
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t i0 = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i0 < total;
       i0 += kGlueUnroll * stride) {
    float v[kGlueUnroll][8];
    float* dst[kGlueUnroll];
#pragma unroll
    for (int u = 0; u < kGlueUnroll; ++u) {
      const uint64_t i = i0 + u * stride;
      if (i < total) {
        const uint64_t r = i / (ga + gb);
        const uint32_t k = static_cast<uint32_t>(i - r * (ga + gb));
        const T* src = k < ga ? a + r * ca + 8ull * k : b + r * cb + 8ull * (k - ga);
        load8(src, v[u]);
        dst[u] = out + r * (ca + cb) + 8ull * k;
      }
    }
#pragma unroll
    for (int u = 0; u < kGlueUnroll; ++u) {
      if (i0 + u * stride < total) {
        float4* o = reinterpret_cast<float4*>(dst[u]);
        __stcs(o, make_float4(v[u][0], v[u][1], v[u][2], v[u][3]));
        __stcs(o + 1, make_float4(v[u][4], v[u][5], v[u][6], v[u][7]));
      }
    }
  }
}

// Patch embedding front half (im2col_patch.wesl): images (N, 3, H, W) f32 in
// [0, 1] -> rows (N*P, row_stride) of T, patch-major (n, py, px), column
// c*ps*ps + ky*ps + kx = (pixel(c, py*ps + ky, px*ps + kx) - mean[c]) *
// inv_std[c] (the conv weight's (C_out, 3, ps, ps) order); columns
// [3*ps*ps, row_stride) are zero so the patch GEMM can take a K padded to a
// 16-byte multiple (3*14*14 = 588 -> 592).
template <typename T>
__global__ void __launch_bounds__(256) im2col_patch_kernel(const float* __restrict__ img, T* __restrict__ out,
                                                           uint32_t n, uint32_t height, uint32_t width, uint32_t ps,
                                                           uint32_t row_stride, float3 mean, float3 inv_std) {
  const uint32_t hp = height / ps, wp = width / ps, kk = ps * ps;
  const uint64_t total = static_cast<uint64_t>(n) * hp * wp * row_stride;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t patch = i / row_stride;
    const uint32_t col = static_cast<uint32_t>(i - patch * row_stride);
    float v = 0.f;
    if (col < 3 * kk) {
      const uint32_t c = col / kk, ky = (col - c * kk) / ps, kx = col - c * kk - ky * ps;
      const uint64_t frame = patch / (static_cast<uint64_t>(hp) * wp);
      const uint32_t pi = static_cast<uint32_t>(patch - frame * hp * wp);
      const uint32_t py = pi / wp, px = pi - py * wp;
      const float m = c == 0 ? mean.x : c == 1 ? mean.y : mean.z;
      const float is = c == 0 ? inv_std.x : c == 1 ? inv_std.y : inv_std.z;
      const float pix = __ldg(img + ((frame * 3 + c) * height + py * ps + ky) * static_cast<uint64_t>(width) +
                              px * ps + kx);
      v = (pix - m) * is;
    }
    out[i] = cvt_to<T>(v);
  }
}

// Grid of the glue kernels: one thread per kGlueUnroll granules, at most 8 resident
// 256-thread blocks on each of the 148 SMs (the grid-stride loop covers the rest).
unsigned grid_for(uint64_t work) {
  const uint64_t blocks = (work + 256 * kGlueUnroll - 1) / (256 * kGlueUnroll);
  return static_cast<unsigned>(blocks < 148ull * 8 ? (blocks ? blocks : 1) : 148ull * 8);
}

template <template <typename> class F, typename... A>
cudaError_t by_code(int code, A... args) {
  switch (code) {
    case kBF16: return F<__nv_bfloat16>::run(args...);
    case kF16: return F<__half>::run(args...);
    default: return F<float>::run(args...);
  }
}

template <typename T>
struct LayerNormRun {
  template <int C>
  static void wide(cudaStream_t st, const void* x, void* out, const float* w, const float* b, uint64_t rows,
                   float eps) {
    layernorm_wide_kernel<T, C><<<blocks_for(rows * 32, 256), 256, 0, st>>>(
        static_cast<const T*>(x), static_cast<T*>(out), w, b, rows, eps);
  }
  static cudaError_t run(cudaStream_t st, const void* x, void* out, const float* w, const float* b, uint64_t rows,
                         uint32_t dim, float eps) {
    const bool vec = dim % 256 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                                         reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
    switch (vec ? dim / 256 : 0) {
      case 1: wide<1>(st, x, out, w, b, rows, eps); break;
      case 2: wide<2>(st, x, out, w, b, rows, eps); break;
      case 3: wide<3>(st, x, out, w, b, rows, eps); break;
      case 4: wide<4>(st, x, out, w, b, rows, eps); break;
      case 6: wide<6>(st, x, out, w, b, rows, eps); break;
      case 8: wide<8>(st, x, out, w, b, rows, eps); break;
      default:
        layernorm_kernel<T><<<blocks_for(rows * 32, 256), 256, 0, st>>>(static_cast<const T*>(x),
                                                                         static_cast<T*>(out), w, b, rows, dim, eps);
    }
    return cudaGetLastError();
  }
};

template <typename T>
struct RopeRun {
  static cudaError_t run(cudaStream_t st, void* x, const float* sn, const float* cs, uint32_t s, uint32_t h,
                         uint32_t t, uint32_t d, uint32_t prefix, uint32_t tpf) {
    const uint64_t total = static_cast<uint64_t>(s) * h * t * (d / 2);
    rope_apply_kernel<T><<<blocks_for(total, 256), 256, 0, st>>>(static_cast<T*>(x), sn, cs, s, h, t, d, prefix, tpf);
    return cudaGetLastError();
  }
};

template <typename T>
struct PermuteRun {
  static cudaError_t run(cudaStream_t st, const void* x, void* out, uint32_t s, uint32_t h, uint32_t t, uint32_t d,
                         int merge) {
    const uint64_t total = static_cast<uint64_t>(s) * h * t * d;
    constexpr int kVec = 16 / sizeof(T);
    const bool vec = (d % kVec) == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) % 16) == 0;
    if (vec)
      permute_heads_kernel<T, kVec><<<blocks_for(total / kVec, 256), 256, 0, st>>>(
          static_cast<const T*>(x), static_cast<T*>(out), s, h, t, d, merge);
    else
      permute_heads_kernel<T, 1><<<blocks_for(total, 256), 256, 0, st>>>(static_cast<const T*>(x),
                                                                          static_cast<T*>(out), s, h, t, d, merge);
    return cudaGetLastError();
  }
};

}  // namespace

cudaError_t launch_qk_prep(cudaStream_t stream, int in_code, int out_code, uint32_t S, uint32_t H, uint32_t t,
                           const PrepJob* jobs, int n_jobs, int* status, uint64_t timeout_ns) {
  const uint32_t sh = S * H;
  if (sh == 0 || t == 0 || n_jobs == 0) return cudaSuccess;
  if (n_jobs < 0 || n_jobs > kMaxPrepJobs) return cudaErrorInvalidValue;
  PrepJobs all{};
  for (int i = 0; i < n_jobs; ++i) all.job[i] = jobs[i];
  if (in_code == out_code && in_code != kF32 && status) {
    bool launched = false;
    const cudaError_t e = in_code == kBF16
                              ? prep_tma<__nv_bfloat16>(stream, all, n_jobs, S, H, t, status, timeout_ns, &launched)
                              : prep_tma<__half>(stream, all, n_jobs, S, H, t, status, timeout_ns, &launched);
    if (launched || e != cudaSuccess) return e;
  }
  switch (in_code) {
    case kBF16: return prep_dispatch_out<__nv_bfloat16>(stream, all, n_jobs, out_code, sh, H, t);
    case kF16: return prep_dispatch_out<__half>(stream, all, n_jobs, out_code, sh, H, t);
    default: return prep_dispatch_out<float>(stream, all, n_jobs, out_code, sh, H, t);
  }
}

cudaError_t launch_qk_prep(cudaStream_t stream, const void* x, int in_code, const RowLayout& lx, void* out,
                           int out_code, uint32_t S, uint32_t H, uint32_t t, const QkPrologue& p, int* status,
                           uint64_t timeout_ns) {
  PrepJob job{x, lx, out, p};
  return launch_qk_prep(stream, in_code, out_code, S, H, t, &job, 1, status, timeout_ns);
}

cudaError_t launch_layernorm(cudaStream_t stream, const void* x, void* out, int code, const float* w, const float* b,
                             uint64_t rows, uint32_t dim, float eps) {
  if (rows == 0 || dim == 0) return cudaSuccess;
  return by_code<LayerNormRun>(code, stream, x, out, w, b, rows, dim, eps);
}

cudaError_t launch_rope_apply(cudaStream_t stream, void* x, int code, const float* sin_t, const float* cos_t,
                              uint32_t s, uint32_t h, uint32_t t, uint32_t d, uint32_t prefix,
                              uint32_t tokens_per_frame) {
  if (static_cast<uint64_t>(s) * h * t * d == 0) return cudaSuccess;
  return by_code<RopeRun>(code, stream, x, sin_t, cos_t, s, h, t, d, prefix, tokens_per_frame);
}

cudaError_t launch_split_heads(cudaStream_t stream, const void* x, void* out, int code, uint32_t s, uint32_t t,
                               uint32_t h, uint32_t d) {
  if (static_cast<uint64_t>(s) * h * t * d == 0) return cudaSuccess;
  return by_code<PermuteRun>(code, stream, x, out, s, h, t, d, 0);
}

cudaError_t launch_attn_merge(cudaStream_t stream, const void* x, void* out, int code, uint32_t s, uint32_t h,
                              uint32_t t, uint32_t d) {
  if (static_cast<uint64_t>(s) * h * t * d == 0) return cudaSuccess;
  return by_code<PermuteRun>(code, stream, x, out, s, h, t, d, 1);
}

cudaError_t launch_copy_row_blocks(cudaStream_t stream, const void* src, void* dst, uint64_t groups,
                                   uint64_t src_stride_rows, uint64_t dst_stride_rows, uint64_t rows,
                                   uint64_t row_bytes) {
  if (groups == 0 || rows == 0 || row_bytes == 0) return cudaSuccess;
  const uint64_t gran = row_bytes / 16;
  copy_row_blocks_kernel<<<grid_for(groups * rows * gran), 256, 0, stream>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), groups, src_stride_rows * gran,
      dst_stride_rows * gran, rows * gran);
  return cudaGetLastError();
}

cudaError_t launch_im2col_patch(cudaStream_t stream, const float* images, void* out, int code, uint32_t n,
                                uint32_t height, uint32_t width, uint32_t patch, uint32_t row_stride,
                                const float mean[3], const float inv_std[3]) {
  const uint64_t total = static_cast<uint64_t>(n) * (height / patch) * (width / patch) * row_stride;
  if (total == 0) return cudaSuccess;
  const float3 m = make_float3(mean[0], mean[1], mean[2]);
  const float3 is = make_float3(inv_std[0], inv_std[1], inv_std[2]);
  const unsigned grid = static_cast<unsigned>(std::min<uint64_t>((total + 255) / 256, 148ull * 16));
  switch (code) {
    case kBF16:
      im2col_patch_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(images, static_cast<__nv_bfloat16*>(out), n,
                                                                   height, width, patch, row_stride, m, is);
      break;
    case kF16:
      im2col_patch_kernel<__half><<<grid, 256, 0, stream>>>(images, static_cast<__half*>(out), n, height, width,
                                                            patch, row_stride, m, is);
      break;
    default:
      im2col_patch_kernel<float><<<grid, 256, 0, stream>>>(images, static_cast<float*>(out), n, height, width, patch,
                                                           row_stride, m, is);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch_cache_build(cudaStream_t stream, const void* a, const void* b, float* out, int code,
                               uint64_t rows, uint32_t ca, uint32_t cb) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = grid_for(rows * (ca + cb) / 8);
  switch (code) {
    case kBF16:
      cache_build_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(a),
                                                                  static_cast<const __nv_bfloat16*>(b), out, rows,
                                                                  ca, cb);
      break;
    case kF16:
      cache_build_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(a),
                                                           static_cast<const __half*>(b), out, rows, ca, cb);
      break;
    default:
      cache_build_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(a),
                                                          static_cast<const float*>(b), out, rows, ca, cb);
      break;
  }
  return cudaGetLastError();
}

}  // namespace hs
