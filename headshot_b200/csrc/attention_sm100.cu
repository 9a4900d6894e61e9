// attention_sm100.cu — non-causal flash attention, head_dim 64, on tcgen05.
//
// Replaces the reference's per-query WGSL kernel
// (crates/headshot-server/shaders/attention.wesl:36-82, dispatched by
// GpuContext::attention, src/engine/ops.rs:228-253) for the aggregator's
// frame and global attention.  Same contract: q, k, v, out head-major
// (S·H, T, 64); out = softmax(q·kᵀ·scale)·v with f32 softmax statistics.
//
// One CTA owns 256 query rows of one (s, h) sequence as two 128-row tiles
// and streams all 96-key K/V tiles of that sequence:
//
//   warps 0-3   softmax warpgroup 0 (one thread per query row)
//   warps 4-7   softmax warpgroup 1
//   warp  8     TMA producer: K and V 96x64 tiles, 128B-swizzled, kStages ring
//   warp  9     UMMA issue for warpgroup 0 (whole warp; elect.sync issues)
//   warp  10    UMMA issue for warpgroup 1
//   warp  11    TMEM owner (alloc/free)
//
// TMEM (512 columns x 128 lanes): two score buffers per warpgroup,
// S[wg][b] = columns (2*wg + b) * 96 .. +96 (f32), and the accumulators
// O[wg] = columns 384 + 64*wg .. +64 (f32).  The softmax writes P (16-bit
// pairs) over the first 48 columns of the S buffer it has just read, and
// the PV product takes its A operand from there.
//
// Double-buffered S decouples the tensor core from the softmax: while a
// warpgroup turns S(j) into P(j), S(j+1) already sits in its other buffer,
// and the warpgroup's own MMA warp issues O += P(j)·V_j followed by S(j+2)
// into the freed buffer, then one commit for both (one thread's MMAs run in
// order, so S(j+2) cannot overwrite P(j) before the PV product has read
// it).  One MMA warp per warpgroup keeps the two issue chains independent;
// the MMA warps run converged so descriptors stay in uniform registers.
//
// The softmax keeps a lazily-updated running max (O is rescaled only when
// the max grows by more than 2^8), evaluates the exponentials partly on
// MUFU.EX2 and partly as a polynomial on the FMA pipe, works on packed
// f32x2 pairs, and reads/writes TMEM with tcgen05.ld/st.
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
constexpr int kBN = 96;   // keys per KV tile: 4 score buffers x 96 + 2 accumulators x 64 = 512 TMEM columns
constexpr int kPairs = kBN / 2;
constexpr int kStages = 6;
constexpr int kQTileBytes = kBM * kD * 2;   // 16 KiB
constexpr int kKvTileBytes = kBN * kD * 2;  // 12 KiB
constexpr int kThreads = 384;  // 3 warpgroups: softmax 0, softmax 1, control
constexpr uint32_t kLaunchRegs = 168;  // 65536 / 384 rounded down to a multiple of 8
constexpr uint32_t kSoftmaxRegs = 224;
constexpr uint32_t kControlRegs = 56;
static_assert(2 * kSoftmaxRegs + kControlRegs <= 3 * kLaunchRegs, "setmaxnreg split exceeds the launch budget");
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp0 = 9;  // + warpgroup index
constexpr int kTmemWarp = 11;
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int wg, int buf) { return static_cast<uint32_t>((2 * wg + buf) * kBN); }
__host__ __device__ constexpr uint32_t col_o(int wg) { return static_cast<uint32_t>(4 * kBN + 64 * wg); }
static_assert(4 * kBN + 2 * 64 <= 512, "TMEM budget");
constexpr float kRescaleThreshold = 8.0f;  // log2 units: p <= 2^8 between rescales
constexpr int kEmuPer8 = 1;                // of every 8 exponential pairs, this many run on the FMA pipe

// Site codes written to the status word when a bounded wait gives up.
enum : int {
  kSiteQFull = 0x101,
  kSiteKvFull = 0x102,
  kSitePFull = 0x104,
  kSiteSFull = 0x105,
  kSiteODone = 0x106,
  kSiteKvEmpty = 0x107,
};

// Every per-tile barrier is doubled by tile parity so no waiter can fall two
// phases behind (parity waits cannot tell phase n from phase n+2).
struct Ctrl {
  uint64_t kv_full[kStages];   // K and V tile of a stage landed (one transaction count)
  uint64_t kv_empty[kStages];  // both MMA warps are done with the stage
  uint64_t q_full[2];          // Q tile of a warpgroup is in shared memory
  uint64_t s_full[2][2];       // [wg][buf]: S(j) landed; next phase: PV(j) and S(j+2) landed
  uint64_t p_full[2][2];       // softmax wrote P (and rescaled O) for the tile in that buffer
  uint64_t drain[2];           // every MMA of that warpgroup's MMA warp completed
  uint32_t tmem_base;
  int abort_flag;
  float ln_w[kD];
  float ln_b[kD];
};

constexpr size_t kSmemBytes =
    1024 /*alignment slack*/ + 2 * kQTileBytes + 2 * kStages * kKvTileBytes + sizeof(Ctrl);
static_assert(kKvTileBytes % 1024 == 0, "swizzle atoms of each stage must stay 1024-byte aligned");

struct Args {
  const void* q;
  void* out;
  uint32_t t_q;   // query rows per sequence
  uint32_t t_kv;  // keys per sequence
  uint32_t n_kv;  // ceil(t_kv / kBN)
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

// ---- packed f32x2 arithmetic (sm_100) and the FMA-pipe exp2 -------------

__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe for a pair, x <= ~8 (inputs below -125 clamp there and
// return ~2^-125, which is zero for every later use).  Range reduction:
// adding 1.5*2^23 rounds x to the nearest integer j in the low mantissa bits,
// f = x - j lies in [-0.5, 0.5]; 2^f comes from a cubic fitted to minimise
// the maximum relative error on that interval (Lawson's iteratively
// reweighted least squares; max relative error 8.3e-5, below the 2^-12
// rounding of the 16-bit P that consumes it); j is then added directly to
// the exponent field.
constexpr float kExpMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kExpC0 = 0.99991959f;
constexpr float kExpC1 = 0.69326216f;
constexpr float kExpC2 = 0.24271429f;
constexpr float kExpC3 = 0.05521307f;

__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  x0 = fmaxf(x0, -125.f);
  x1 = fmaxf(x1, -125.f);
  float t0, t1, r0, r1, f0, f1, p0, p1;
  add2(t0, t1, x0, x1, kExpMagic, kExpMagic);
  add2(r0, r1, t0, t1, -kExpMagic, -kExpMagic);
  fma2(f0, f1, r0, r1, -1.f, -1.f, x0, x1);
  fma2(p0, p1, f0, f1, kExpC3, kExpC3, kExpC2, kExpC2);
  fma2(p0, p1, p0, p1, f0, f1, kExpC1, kExpC1);
  fma2(p0, p1, p0, p1, f0, f1, kExpC0, kExpC0);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
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
    uint8_t* dst = sQ + wg * kQTileBytes + row * 128;
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl->q_full[wg]);  // one arrival per warp
  }

  const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
  const uint32_t tO = tmem + lane_base + col_o(wg);
  const float c = a.scale_log2;
  const uint32_t tail = a.t_kv - (a.n_kv - 1) * kBN;  // valid keys in the last tile, 1..kBN

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
    const int b = static_cast<int>(j & 1);
    if (!warp_wait(&ctl->s_full[wg][b], (j >> 1) & 1, abort_flag, a.status, kSiteSFull, a.timeout_ns)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t tS = tmem + lane_base + col_s(wg, b);
    uint32_t s[kBN];
    tmem_ld32(tS + 0, s + 0);
    tmem_ld32(tS + 32, s + 32);
    tmem_ld32(tS + 64, s + 64);
    tmem_wait_ld_regs<kBN>(s);
    if (j == a.n_kv - 1 && tail < kBN) {
#pragma unroll
      for (int i = 0; i < kBN; ++i)
        if (static_cast<uint32_t>(i) >= tail) s[i] = __float_as_uint(-INFINITY);
    }
    // Row max: 3-input max in four independent chains.
    float m4[4] = {u2f(s[0]), u2f(s[1]), u2f(s[2]), u2f(s[3])};
#pragma unroll
    for (int i = 4; i < kBN; i += 2) m4[(i >> 1) & 3] = max3(m4[(i >> 1) & 3], u2f(s[i]), u2f(s[i + 1]));
    const float m_tile = max3(fmaxf(m4[0], m4[1]), m4[2], m4[3]) * c;

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
    // P = 2^(s*c - m) on packed f32x2 pairs; kEmuPer8 of every 8 pairs take
    // the FMA-pipe exp2, the rest MUFU.EX2.  P overwrites the first kPairs
    // columns of this S buffer (already read into registers).  The row sum
    // adds the rounded 16-bit P the tensor core multiplies (mixed-precision
    // add into f32), so the rounding of dominant weights cancels in O / l.
    const float neg_m = -m_run;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t pk[kPairs];
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
      float x0, x1, p0, p1;
      fma2(x0, x1, u2f(s[2 * i]), u2f(s[2 * i + 1]), c, c, neg_m, neg_m);
      if ((i & 7) < kEmuPer8) {
        exp2_poly2(x0, x1, p0, p1);
      } else {
        p0 = ex2_approx(x0);
        p1 = ex2_approx(x1);
      }
      pk[i] = Elem<E>::pack2(p0, p1);
      Elem<E>::acc2(acc[2 * (i & 1)], acc[2 * (i & 1) + 1], pk[i]);
      if (i == 31) tmem_st32(tS, pk);
    }
    tmem_st16(tS + 32, pk + 32);
    l += (acc[0] + acc[1]) + (acc[2] + acc[3]);
    // O rescale (rare), once the previous PV product has landed (the commit
    // after PV(j-1) completes the next phase of the other buffer's s_full).
    // PV(j) is issued only after p_full, so it accumulates onto the rescaled O.
    if (__any_sync(0xffffffffu, need)) {
      if (j > 0) {
        if (!warp_wait(&ctl->s_full[wg][(j - 1) & 1], ((j + 1) >> 1) & 1, abort_flag, a.status, kSiteODone,
                       a.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
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
    have_o = true;
    tmem_wait_st();
    tc_fence_before();
    // One arrival per warp: 128 single-thread arrivals on one barrier word
    // would serialise on the shared-memory atomic unit every tile.
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl->p_full[wg][b]);
  }

  if (!ok) return;
  // The commit after PV(n-1) is the next phase of the last tile's buffer.
  const uint32_t last = a.n_kv - 1;
  if (!warp_wait(&ctl->s_full[wg][last & 1], ((last + 2) >> 1) & 1, abort_flag, a.status, kSiteODone,
                 a.timeout_ns))
    return;
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
    mbar_arrive_expect_tx(&ctl->kv_full[st], 2 * kKvTileBytes);
    tma_load_3d(tm_k, &ctl->kv_full[st], sK + st * kKvTileBytes, 0, static_cast<int>(j * kBN), seq);
    tma_load_3d(tm_v, &ctl->kv_full[st], sV + st * kKvTileBytes, 0, static_cast<int>(j * kBN), seq);
    issued = j + 1;
  }
  // Let every load this warp issued land before the CTA can exit.
  const uint32_t first = issued > kStages ? issued - kStages : 0;
  for (uint32_t j = first; j < issued; ++j) {
    int no_abort = 0;
    mbar_wait(&ctl->kv_full[j % kStages], (j / kStages) & 1, &no_abort, a.status, kSiteKvFull, a.timeout_ns);
  }
}

// One MMA warp per softmax warpgroup, all 32 lanes: waits and descriptor
// math stay warp-uniform and elect.sync picks the lane that issues.
template <typename E>
__device__ void mma_role(const Args& a, int wg, uint8_t* sQ, uint8_t* sK, uint8_t* sV, Ctrl* ctl, uint32_t tmem) {
  volatile int* abort_flag = &ctl->abort_flag;
  constexpr bool kBf16 = Elem<E>::kBf16;
  constexpr uint32_t idesc_qk = idesc_f16(kBf16, kBM, kBN, false, false);
  constexpr uint32_t idesc_pv = idesc_f16(kBf16, kBM, kD, false, true);
  // Descriptor bases; a K=16 step of S advances the start field by
  // 32 B >> 4 = 2, a 16-key step of V by 2048 B >> 4 = 128.
  const uint64_t q_desc = sdesc_sw128(smem_u32(sQ + wg * kQTileBytes), 16, 1024);
  const uint64_t k_desc = sdesc_sw128(smem_u32(sK), 16, 1024);
  const uint64_t v_desc = sdesc_sw128(smem_u32(sV), 16, 1024);
  constexpr uint64_t kKvTileStep = kKvTileBytes >> 4;
  const uint32_t o_tmem = tmem + col_o(wg);

  // S[wg][buf] = Q_wg · K_stᵀ: K = 64 as four K=16 steps inside the swizzle atom.
  auto issue_s = [&](uint32_t st, int buf) {
    const uint64_t kd = k_desc + st * kKvTileStep;
    const uint32_t d = tmem + col_s(wg, buf);
#pragma unroll
    for (int k = 0; k < kD / 16; ++k) umma_ss_elect(d, q_desc + 2 * k, kd + 2 * k, idesc_qk, k > 0 ? 1u : 0u);
  };
  // O[wg] += P[wg][buf] · V_st: 16 keys per step = 8 TMEM columns of P, 2 swizzle atoms of V.
  auto issue_pv = [&](uint32_t st, int buf, bool acc) {
    const uint64_t vd = v_desc + st * kKvTileStep;
    const uint32_t p = tmem + col_s(wg, buf);
#pragma unroll
    for (int k = 0; k < kBN / 16; ++k)
      umma_ts_elect(o_tmem, p + 8 * k, vd + 128 * k, idesc_pv, (acc || k > 0) ? 1u : 0u);
  };

  bool ok = warp_wait(&ctl->q_full[wg], 0, abort_flag, a.status, kSiteQFull, a.timeout_ns);
  if (ok) tc_fence_after();
  // S(0) and S(1) up front.
  for (uint32_t t = 0; ok && t < 2 && t < a.n_kv; ++t) {
    if (!warp_wait(&ctl->kv_full[t % kStages], (t / kStages) & 1, abort_flag, a.status, kSiteKvFull,
                   a.timeout_ns)) {
      ok = false;
      break;
    }
    issue_s(t % kStages, static_cast<int>(t));
    umma_commit_elect(&ctl->s_full[wg][t]);
  }
  const bool acc0 = a.st.load != 0;
  for (uint32_t j = 0; ok && j < a.n_kv; ++j) {
    const int b = static_cast<int>(j & 1);
    const uint32_t st = j % kStages;  // V_j: this stage was waited on before S(j) was issued
    if (!warp_wait(&ctl->p_full[wg][b], (j >> 1) & 1, abort_flag, a.status, kSitePFull, a.timeout_ns)) break;
    tc_fence_after();
    issue_pv(st, b, j > 0 || acc0);
    if (j + 2 < a.n_kv) {
      const uint32_t st2 = (j + 2) % kStages;
      if (!warp_wait(&ctl->kv_full[st2], ((j + 2) / kStages) & 1, abort_flag, a.status, kSiteKvFull,
                     a.timeout_ns)) {
        ok = false;
        break;
      }
      issue_s(st2, b);  // after PV(j) in this warp's order, so it never overwrites P(j) early
    }
    umma_commit_elect(&ctl->s_full[wg][b]);
    if (j + kStages < a.n_kv) umma_commit_elect(&ctl->kv_empty[st]);  // the producer reuses this stage
  }
  // Drain: every MMA this warp issued has completed before TMEM is freed.
  umma_commit_elect(&ctl->drain[wg]);
  int no_abort = 0;
  warp_wait(&ctl->drain[wg], 0, &no_abort, a.status, kSiteODone, a.timeout_ns);
}

template <typename E>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kQTileBytes;
  uint8_t* sV = sK + kStages * kKvTileBytes;
  Ctrl* ctl = reinterpret_cast<Ctrl*>(sV + kStages * kKvTileBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->kv_full[s], 1);
      mbar_init(&ctl->kv_empty[s], 2);  // one commit per MMA warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->q_full[i], kBM / 32);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&ctl->s_full[i][b], 1);
        mbar_init(&ctl->p_full[i][b], kBM / 32);
      }
      mbar_init(&ctl->drain[i], 1);
    }
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
  if (warp == kTmemWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  // Launch budget 384 x 168 registers; softmax warpgroups take 224 each and
  // the control warpgroup keeps 56: 2*224 + 56 == 3*168.
  if (warp < 8) {
    regs_inc<kSoftmaxRegs>();
    softmax_role<E>(a, sQ, ctl, tmem, warp, lane);
  } else {
    regs_dec<kControlRegs>();
    if (warp == kProducerWarp) {
      if (lane == 0) producer_role(a, &tm_k, &tm_v, sK, sV, ctl);
    } else if (warp == kMmaWarp0 || warp == kMmaWarp0 + 1) {
      mma_role<E>(a, warp - kMmaWarp0, sQ, sK, sV, ctl, tmem);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kTmemWarp) {
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

// (SH, T, 64) 16-bit tensor as a 3-D map with kBN x 64 boxes, 128B swizzle.
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
