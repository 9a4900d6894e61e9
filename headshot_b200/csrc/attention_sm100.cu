// attention_sm100.cu — non-causal flash attention, head_dim 64, on tcgen05.
//
// Replaces the reference's per-query WGSL kernel
// (crates/headshot-server/shaders/attention.wesl:36-82, dispatched by
// GpuContext::attention, src/engine/ops.rs:228-253) for the aggregator's
// frame and global attention.  Same contract: q, k, v, out head-major
// (S·H, T, 64); out = softmax(q·kᵀ·scale)·v with f32 softmax statistics.
//
// One CTA owns 256 query rows of one (s, h) sequence as two 128-row tiles
// and streams all key/value tiles of that sequence:
//
//   warps 0-3   softmax warpgroup for Q tile 0 (one thread per query row)
//   warps 4-7   softmax warpgroup for Q tile 1
//   warp  8     TMA producer: K/V 128x64 tiles, 128B-swizzled, kStages ring
//   warp  9     TMEM owner + single-thread UMMA issue
//
// TMEM (512 columns x 128 lanes, f32): S0 [0,128) S1 [128,256) O0 [256,320)
// O1 [320,384) P0 [384,448) P1 [448,512); P holds the probabilities as
// packed 16-bit pairs and feeds the PV product straight from TMEM.
//
// Per KV tile j the MMA warp issues S_i(j+1) = Q_i·K_{j+1}ᵀ as soon as the
// softmax of S_i(j) has been consumed, then O_i += P_i(j)·V_j, so the tensor
// core works on one Q tile while the other's softmax runs.  The softmax keeps
// a lazily-updated running max (rescale O only when the max grows by more
// than 2^8) and reads/writes TMEM with tcgen05.ld/st.
//
// The Q tile is loaded by the softmax threads themselves, one row per
// thread, and goes through the fused QK-norm + RoPE prologue in f32 before
// being written to shared memory in the UMMA 128B-swizzle layout.
#include <cuda.h>

#include "hs_internal.h"
#include "hs_ptx.cuh"

namespace hs {
namespace {

constexpr int kD = 64;
constexpr int kBM = 128;  // query rows per tile / softmax warpgroup
constexpr int kBN = 128;  // keys per KV tile
constexpr int kStages = 4;
constexpr int kTileBytes = kBM * kD * 2;  // 16 KiB for Q, K and V tiles alike
constexpr int kThreads = 384;  // 3 warpgroups: softmax 0, softmax 1, control (producer, MMA, 2 spare)
constexpr uint32_t kLaunchRegs = 168;  // 65536 / 384 rounded down to a multiple of 8
constexpr uint32_t kSoftmaxRegs = 224;
constexpr uint32_t kControlRegs = 56;
static_assert(2 * kSoftmaxRegs + kControlRegs <= 3 * kLaunchRegs, "setmaxnreg split exceeds the launch budget");
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int wg) { return wg ? 128u : 0u; }
__host__ __device__ constexpr uint32_t col_o(int wg) { return wg ? 320u : 256u; }
__host__ __device__ constexpr uint32_t col_p(int wg) { return wg ? 448u : 384u; }
constexpr float kRescaleThreshold = 8.0f;  // log2 units: p <= 2^8 between rescales

// Site codes written to the status word when a bounded wait gives up.
enum : int {
  kSiteQFull = 0x101,
  kSiteKFull = 0x102,
  kSiteVFull = 0x103,
  kSitePFull = 0x104,
  kSiteSFull = 0x105,
  kSiteODone = 0x106,
  kSiteKvEmpty = 0x107,
};

struct Ctrl {
  uint64_t k_full[kStages];
  uint64_t v_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t q_full[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  float ln_w[kD];
  float ln_b[kD];
};

constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + 2 * kTileBytes + 2 * kStages * kTileBytes + sizeof(Ctrl);

struct Args {
  const void* q;
  void* out;
  uint32_t t_q;   // query rows per sequence
  uint32_t t_kv;  // keys per sequence
  uint32_t n_kv;  // ceil(t_kv / 128)
  int q_f32;
  int out_f32;
  float scale_log2;
  QkPrologue qp;
  AttnState st;
  int* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// Bounded wait whose outcome is the same for all 32 lanes, so the
// .sync.aligned tcgen05 instructions that follow never see a split warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int site, uint64_t timeout_ns) {
  const bool r = mbar_wait(bar, parity, abort_flag, status, site, timeout_ns);
  return __all_sync(0xffffffffu, r);
}

// Loads one 64-wide query row (16-bit or f32 storage) into f32 registers.
template <typename E>
__device__ __forceinline__ void load_row(const Args& a, uint64_t row_index, float (&x)[kD]) {
  if (a.q_f32) {
    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(a.q) + row_index * kD);
#pragma unroll
    for (int c = 0; c < kD / 4; ++c) {
      float4 v = __ldg(src + c);
      x[4 * c + 0] = v.x;
      x[4 * c + 1] = v.y;
      x[4 * c + 2] = v.z;
      x[4 * c + 3] = v.w;
    }
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const E*>(a.q) + row_index * kD);
#pragma unroll
    for (int c = 0; c < kD / 8; ++c) {
      uint4 v = __ldg(src + c);
      float2 f0 = Elem<E>::unpack2(v.x), f1 = Elem<E>::unpack2(v.y);
      float2 f2 = Elem<E>::unpack2(v.z), f3 = Elem<E>::unpack2(v.w);
      x[8 * c + 0] = f0.x;
      x[8 * c + 1] = f0.y;
      x[8 * c + 2] = f1.x;
      x[8 * c + 3] = f1.y;
      x[8 * c + 4] = f2.x;
      x[8 * c + 5] = f2.y;
      x[8 * c + 6] = f3.x;
      x[8 * c + 7] = f3.y;
    }
  }
}

// QK-norm (two-pass mean/variance in f32) then rotate-half RoPE on one row.
__device__ __forceinline__ void prologue_row(const Args& a, const Ctrl* ctl, uint32_t token, float (&x)[kD]) {
  if (a.qp.ln) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kD; ++i) s += x[i];
    const float mu = s * (1.0f / kD);
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < kD; ++i) {
      const float d = x[i] - mu;
      v = fmaf(d, d, v);
    }
    const float inv = rsqrtf(v * (1.0f / kD) + a.qp.eps);
#pragma unroll
    for (int i = 0; i < kD; ++i) x[i] = (x[i] - mu) * inv * ctl->ln_w[i] + ctl->ln_b[i];
  }
  if (a.qp.rope) {
    const uint32_t ft = (token + a.qp.pos_offset) % a.qp.tokens_per_frame;
    if (ft >= a.qp.prefix) {
      const uint64_t r = static_cast<uint64_t>(ft - a.qp.prefix) * kD;
      const float4* sn = reinterpret_cast<const float4*>(a.qp.sin_t + r);
      const float4* cs = reinterpret_cast<const float4*>(a.qp.cos_t + r);
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // pairs (i, i+32), 4 at a time
        const float4 sl = __ldg(sn + c), sh = __ldg(sn + 8 + c);
        const float4 cl = __ldg(cs + c), ch = __ldg(cs + 8 + c);
        const float sl_[4] = {sl.x, sl.y, sl.z, sl.w}, sh_[4] = {sh.x, sh.y, sh.z, sh.w};
        const float cl_[4] = {cl.x, cl.y, cl.z, cl.w}, ch_[4] = {ch.x, ch.y, ch.z, ch.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = 4 * c + u;
          const float lo = x[i], hi = x[i + 32];
          x[i] = lo * cl_[u] - hi * sl_[u];
          x[i + 32] = hi * ch_[u] + lo * sh_[u];
        }
      }
    }
  }
}

template <typename E>
__device__ void softmax_role(const Args& a, uint8_t* sQ, Ctrl* ctl, uint32_t tmem, int warp, int lane) {
  const int wg = warp >> 2;
  const int wq = warp & 3;
  const uint32_t row = static_cast<uint32_t>(wq * 32 + lane);
  const uint32_t token = blockIdx.x * (2 * kBM) + wg * kBM + row;
  const bool valid = token < a.t_q;
  const uint64_t row_index = static_cast<uint64_t>(blockIdx.y) * a.t_q + token;
  volatile int* abort_flag = &ctl->abort_flag;

  // ---- Q prologue: global -> f32 -> QK-norm/RoPE -> swizzled smem --------
  {
    float x[kD];
    if (valid) {
      load_row<E>(a, row_index, x);
      prologue_row(a, ctl, token, x);
    } else {
#pragma unroll
      for (int i = 0; i < kD; ++i) x[i] = 0.f;
    }
    uint8_t* dst = sQ + wg * kTileBytes + row * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 v;
      v.x = Elem<E>::pack2(x[8 * c + 0], x[8 * c + 1]);
      v.y = Elem<E>::pack2(x[8 * c + 2], x[8 * c + 3]);
      v.z = Elem<E>::pack2(x[8 * c + 4], x[8 * c + 5]);
      v.w = Elem<E>::pack2(x[8 * c + 6], x[8 * c + 7]);
      *reinterpret_cast<uint4*>(dst + ((c ^ (row & 7)) << 4)) = v;
    }
    fence_proxy_async_smem();
    mbar_arrive(&ctl->q_full[wg]);
  }

  const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
  const uint32_t tS = tmem + lane_base + col_s(wg);
  const uint32_t tO = tmem + lane_base + col_o(wg);
  const uint32_t tP = tmem + lane_base + col_p(wg);
  const float c = a.scale_log2;
  const uint32_t tail = a.t_kv - (a.n_kv - 1) * kBN;  // valid keys in the last tile, 1..128

  float m_run = -INFINITY, l = 0.f;
  bool have_o = false;
  if (a.st.load && valid) {
    m_run = a.st.m[row_index];
    l = a.st.l[row_index];
  }
  if (a.st.load) {
    // Seed O in TMEM with the carried accumulator (zeros for padding rows).
    uint32_t o[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4* src = reinterpret_cast<const float4*>(a.st.o + row_index * kD + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 v = valid ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        o[4 * i + 0] = __float_as_uint(v.x);
        o[4 * i + 1] = __float_as_uint(v.y);
        o[4 * i + 2] = __float_as_uint(v.z);
        o[4 * i + 3] = __float_as_uint(v.w);
      }
      tmem_st32(tO + 32 * h, o);
    }
    tmem_wait_st();
    have_o = true;
    if (!valid) m_run = 0.f;
  }

  bool ok = true;
  for (uint32_t j = 0; j < a.n_kv; ++j) {
    if (!warp_wait(&ctl->s_full[wg], j & 1, abort_flag, a.status, kSiteSFull, a.timeout_ns)) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t s[128];
    tmem_ld32(tS + 0, s + 0);
    tmem_ld32(tS + 32, s + 32);
    tmem_ld32(tS + 64, s + 64);
    tmem_ld32(tS + 96, s + 96);
    tmem_wait_ld_regs<128>(s);
    if (j == a.n_kv - 1 && tail < kBN) {
#pragma unroll
      for (int i = 0; i < kBN; ++i)
        if (static_cast<uint32_t>(i) >= tail) s[i] = __float_as_uint(-INFINITY);
    }
    float mx8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) mx8[u] = u2f(s[u]);
#pragma unroll
    for (int i = 8; i < kBN; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], u2f(s[i]));
    const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                           fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
    const float m_tile = mx * c;

    float factor = 1.f;
    bool need = false;
    if (!have_o) {
      m_run = m_tile;
    } else if (m_tile > m_run + kRescaleThreshold) {
      factor = ex2_approx(m_run - m_tile);
      m_run = m_tile;
      l *= factor;
      need = true;
    }
    if (j > 0) {
      if (!warp_wait(&ctl->o_done[wg], (j - 1) & 1, abort_flag, a.status, kSiteODone, a.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
    }
    if (__any_sync(0xffffffffu, need)) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * h, o);
        tmem_wait_ld_regs<32>(o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(u2f(o[i]) * factor);
        tmem_st32(tO + 32 * h, o);
      }
    }
    const float neg_m = -m_run;
    float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = ex2_approx(fmaf(u2f(s[64 * h + 2 * i]), c, neg_m));
        const float p1 = ex2_approx(fmaf(u2f(s[64 * h + 2 * i + 1]), c, neg_m));
        ls4[i & 3] += p0 + p1;
        pk[i] = Elem<E>::pack2(p0, p1);
      }
      tmem_st32(tP + 32 * h, pk);
    }
    l += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
    have_o = true;
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&ctl->p_full[wg]);
  }

  if (!ok) return;
  if (!warp_wait(&ctl->o_done[wg], (a.n_kv - 1) & 1, abort_flag, a.status, kSiteODone, a.timeout_ns)) return;
  tc_fence_after();

  // ---- epilogue: O row from TMEM, normalise (or store the running state) --
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t o[32];
    tmem_ld32(tO + 32 * h, o);
    tmem_wait_ld_regs<32>(o);
    if (!valid) continue;
    if (a.st.store) {
      float4* dst = reinterpret_cast<float4*>(a.st.o + row_index * kD + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i] = make_float4(u2f(o[4 * i]), u2f(o[4 * i + 1]), u2f(o[4 * i + 2]), u2f(o[4 * i + 3]));
    } else {
      const float inv_l = 1.0f / l;
      if (a.out_f32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + row_index * kD + 32 * h);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = make_float4(u2f(o[4 * i]) * inv_l, u2f(o[4 * i + 1]) * inv_l, u2f(o[4 * i + 2]) * inv_l,
                               u2f(o[4 * i + 3]) * inv_l);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<E*>(a.out) + row_index * kD + 32 * h);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 v;
          v.x = Elem<E>::pack2(u2f(o[8 * i + 0]) * inv_l, u2f(o[8 * i + 1]) * inv_l);
          v.y = Elem<E>::pack2(u2f(o[8 * i + 2]) * inv_l, u2f(o[8 * i + 3]) * inv_l);
          v.z = Elem<E>::pack2(u2f(o[8 * i + 4]) * inv_l, u2f(o[8 * i + 5]) * inv_l);
          v.w = Elem<E>::pack2(u2f(o[8 * i + 6]) * inv_l, u2f(o[8 * i + 7]) * inv_l);
          dst[i] = v;
        }
      }
    }
  }
  if (valid && a.st.store) {
    a.st.m[row_index] = m_run;
    a.st.l[row_index] = l;
  }
}

__device__ void producer_role(const Args& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v, uint8_t* sK,
                              uint8_t* sV, Ctrl* ctl) {
  volatile int* abort_flag = &ctl->abort_flag;
  const int seq = static_cast<int>(blockIdx.y);
  uint32_t issued = 0;
  for (uint32_t j = 0; j < a.n_kv; ++j) {
    const uint32_t st = j % kStages;
    if (j >= kStages) {
      if (!mbar_wait(&ctl->kv_empty[st], ((j / kStages) - 1) & 1, abort_flag, a.status, kSiteKvEmpty,
                     a.timeout_ns))
        break;
    }
    mbar_arrive_expect_tx(&ctl->k_full[st], kTileBytes);
    tma_load_3d(tm_k, &ctl->k_full[st], sK + st * kTileBytes, 0, static_cast<int>(j * kBN), seq);
    mbar_arrive_expect_tx(&ctl->v_full[st], kTileBytes);
    tma_load_3d(tm_v, &ctl->v_full[st], sV + st * kTileBytes, 0, static_cast<int>(j * kBN), seq);
    issued = j + 1;
  }
  // Let every load this warp issued land before the CTA can exit.
  const uint32_t first = issued > kStages ? issued - kStages : 0;
  for (uint32_t j = first; j < issued; ++j) {
    const uint32_t st = j % kStages;
    const uint32_t ph = (j / kStages) & 1;
    int dummy_abort = 0;
    mbar_wait(&ctl->k_full[st], ph, &dummy_abort, a.status, kSiteKFull, a.timeout_ns);
    mbar_wait(&ctl->v_full[st], ph, &dummy_abort, a.status, kSiteVFull, a.timeout_ns);
  }
}

template <typename E>
__device__ void mma_role(const Args& a, uint8_t* sQ, uint8_t* sK, uint8_t* sV, Ctrl* ctl, uint32_t tmem) {
  volatile int* abort_flag = &ctl->abort_flag;
  constexpr bool kBf16 = Elem<E>::kBf16;
  constexpr uint32_t idesc_qk = idesc_f16(kBf16, kBM, kBN, false, false);
  constexpr uint32_t idesc_pv = idesc_f16(kBf16, kBM, kD, false, true);
  const uint32_t q_addr = smem_u32(sQ);
  const uint32_t k_addr = smem_u32(sK);
  const uint32_t v_addr = smem_u32(sV);

  auto issue_s = [&](int wg, uint32_t st) {
    const uint32_t qa = q_addr + wg * kTileBytes;
    const uint32_t ka = k_addr + st * kTileBytes;
#pragma unroll
    for (int k = 0; k < kD / 16; ++k)  // K = 16 per instruction: +32 bytes inside the swizzle atom
      umma_ss(tmem + col_s(wg), sdesc_sw128(qa + 32 * k, 16, 1024), sdesc_sw128(ka + 32 * k, 16, 1024), idesc_qk,
              k > 0 ? 1u : 0u);
  };
  auto issue_pv = [&](int wg, uint32_t st, bool acc) {
    const uint32_t va = v_addr + st * kTileBytes;
#pragma unroll
    for (int k = 0; k < kBN / 16; ++k)  // 16 keys per instruction: 2 swizzle atoms of V
      umma_ts(tmem + col_o(wg), tmem + col_p(wg) + 8 * k, sdesc_sw128(va + 2048 * k, 16, 1024), idesc_pv,
              (acc || k > 0) ? 1u : 0u);
  };

  bool ok = mbar_wait(&ctl->q_full[0], 0, abort_flag, a.status, kSiteQFull, a.timeout_ns) &&
            mbar_wait(&ctl->q_full[1], 0, abort_flag, a.status, kSiteQFull, a.timeout_ns);
  if (ok) tc_fence_after();
  const bool acc0 = a.st.load != 0;
  for (uint32_t j = 0; ok && j < a.n_kv; ++j) {
    const uint32_t st = j % kStages;
    const uint32_t ph = (j / kStages) & 1;
    if (j == 0) {
      if (!mbar_wait(&ctl->k_full[0], 0, abort_flag, a.status, kSiteKFull, a.timeout_ns)) break;
      tc_fence_after();
      issue_s(0, 0);
      umma_commit(&ctl->s_full[0]);
      issue_s(1, 0);
      umma_commit(&ctl->s_full[1]);
    }
    if (!mbar_wait(&ctl->v_full[st], ph, abort_flag, a.status, kSiteVFull, a.timeout_ns)) break;
    const bool more = j + 1 < a.n_kv;
    const uint32_t st2 = (j + 1) % kStages;
    const uint32_t ph2 = ((j + 1) / kStages) & 1;

    if (!mbar_wait(&ctl->p_full[0], j & 1, abort_flag, a.status, kSitePFull, a.timeout_ns)) break;
    tc_fence_after();
    if (more) {
      if (!mbar_wait(&ctl->k_full[st2], ph2, abort_flag, a.status, kSiteKFull, a.timeout_ns)) break;
      tc_fence_after();
      issue_s(0, st2);
      umma_commit(&ctl->s_full[0]);
    }
    issue_pv(0, st, j > 0 || acc0);
    umma_commit(&ctl->o_done[0]);

    if (!mbar_wait(&ctl->p_full[1], j & 1, abort_flag, a.status, kSitePFull, a.timeout_ns)) break;
    tc_fence_after();
    if (more) {
      issue_s(1, st2);
      umma_commit(&ctl->s_full[1]);
    }
    issue_pv(1, st, j > 0 || acc0);
    umma_commit(&ctl->o_done[1]);
    umma_commit(&ctl->kv_empty[st]);
  }
  // Drain: every MMA this thread issued has completed before TMEM is freed.
  umma_commit(&ctl->drain);
  int dummy_abort = 0;
  mbar_wait(&ctl->drain, 0, &dummy_abort, a.status, kSiteODone, a.timeout_ns);
}

template <typename E>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kTileBytes;
  uint8_t* sV = sK + kStages * kTileBytes;
  Ctrl* ctl = reinterpret_cast<Ctrl*>(sV + kStages * kTileBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->k_full[s], 1);
      mbar_init(&ctl->v_full[s], 1);
      mbar_init(&ctl->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->q_full[i], kBM);
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->p_full[i], kBM);
      mbar_init(&ctl->o_done[i], 1);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kD) {
    ctl->ln_w[threadIdx.x] = a.qp.ln ? a.qp.ln_w[threadIdx.x] : 1.f;
    ctl->ln_b[threadIdx.x] = a.qp.ln ? a.qp.ln_b[threadIdx.x] : 0.f;
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // Launch budget 384 x 168 registers; softmax warpgroups take 224 each and
  // the producer/MMA warpgroup keeps 56: 2*224 + 56 == 3*168.
  if (warp < 8) {
    regs_inc<kSoftmaxRegs>();
    softmax_role<E>(a, sQ, ctl, tmem, warp, lane);
  } else {
    regs_dec<kControlRegs>();
    if (warp == kProducerWarp) {
      if (lane == 0) producer_role(a, &tm_k, &tm_v, sK, sV, ctl);
    } else if (warp == kMmaWarp) {
      if (lane == 0) mma_role<E>(a, sQ, sK, sV, ctl, tmem);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// (SH, T, 64) 16-bit tensor as a 3-D map with 128x64 boxes, 128B swizzle.
// Rows past T inside a sequence read as zeros (out-of-bounds fill).
bool make_kv_map(CUtensorMap* map, const void* base, bool bf16, uint32_t t, uint32_t sh, std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(t), static_cast<cuuint64_t>(sh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(t) * kD * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kD), static_cast<cuuint32_t>(kBN), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

template <typename E>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& mk, const CUtensorMap& mv, const Args& a,
                         uint32_t sh) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_fwd_sm100<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((a.t_q + 2 * kBM - 1) / (2 * kBM), sh, 1);
  attn_fwd_sm100<E><<<grid, kThreads, kSmemBytes, stream>>>(mk, mv, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_sm100(cudaStream_t stream, int elem, const void* q, int q_code, const void* k,
                                   const void* v, void* out, int out_code, uint32_t sh, uint32_t t_q,
                                   uint32_t t_kv, float scale, const QkPrologue& qp, const AttnState& st,
                                   int* status, uint64_t timeout_ns, std::string* err) {
  if (t_q == 0 || sh == 0) return cudaSuccess;
  const bool bf16 = elem == kBF16;
  CUtensorMap mk, mv;
  if (!make_kv_map(&mk, k, bf16, t_kv, sh, err) || !make_kv_map(&mv, v, bf16, t_kv, sh, err))
    return cudaErrorInvalidValue;
  Args a{};
  a.q = q;
  a.out = out;
  a.t_q = t_q;
  a.t_kv = t_kv;
  a.n_kv = (t_kv + kBN - 1) / kBN;
  a.q_f32 = q_code == kF32;
  a.out_f32 = out_code == kF32;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.qp = qp;
  a.st = st;
  a.status = status;
  a.timeout_ns = timeout_ns;
  return bf16 ? launch_typed<__nv_bfloat16>(stream, mk, mv, a, sh) : launch_typed<__half>(stream, mk, mv, a, sh);
}

}  // namespace hs
