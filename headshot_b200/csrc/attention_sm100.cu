// attention_sm100.cu — non-causal flash attention, head_dim 64, on tcgen05.
//
// Replaces the reference's per-query WGSL kernel
// (crates/headshot-server/shaders/attention.wesl:36-82, dispatched by
// GpuContext::attention, src/engine/ops.rs:228-253) for the aggregator's
// frame and global attention.  Same contract: q, k, v, out head-major
// (S·H, T, 64); out = softmax(q·kᵀ·scale)·v with f32 softmax statistics.
// q, k and v reach this kernel as 16-bit rows; the QK-norm + RoPE prologue
// of the fused op has already been applied to q and k by qk_prep (ops.cu).
//
// The kernel is persistent: one CTA per SM takes work items from a global
// counter (the producer thread fetches the next index one item ahead, decodes
// it into (sequence, first row) and hands that to the other warps through a
// small ring in shared memory; the MMA warps take the next item as soon as
// they have issued an item's last score product, the softmax warps while the
// item's last PV product runs, so the hand-off stays off the item boundary).  An
// item is 256 query rows of one (s, h) sequence, split into two 128-row
// tiles, one per softmax warpgroup, against every 96-key K/V tile of that
// sequence.  Items go out in sequence-major order, so the CTAs working at
// one time share a few sequences' K/V in L2, and a CTA that runs ahead
// simply takes more items (no tail from a fixed assignment).  When one
// sequence's K and V outgrow a fraction of L2, consecutive waves of items
// (one item per CTA) walk the K/V tiles in alternating directions, so a wave
// starts on the tiles the one before it has just read (274,800 keys: DRAM
// reads 7.5 GB per launch instead of 15.7).
//
//   warps 0-3   softmax warpgroup 0 (one thread per query row)
//   warps 4-7   softmax warpgroup 1
//   warp  8     TMA producer: Q tiles (double-buffered per warpgroup) and
//               K and V 96x64 tiles (kStages ring), all 128B-swizzled
//   warp  9     UMMA issue for warpgroup 0 (whole warp; elect.sync issues)
//   warp  10    UMMA issue for warpgroup 1
//   warp  11    TMEM owner (alloc/free)
//
// The producer runs ahead across item boundaries, so the next item's Q and
// first K/V tiles are already in shared memory when the MMA warps finish an
// item; the MMA warps issue the next item's first score tiles while the
// softmax warpgroups are still storing the previous output.  When an item's
// second 128-row tile lies wholly past the sequence end, warpgroup 1 and its
// MMA warp skip the item (the MMA warp only releases the K/V stages).
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
#include <cuda.h>

#include <mutex>

#include "hs_internal.h"
#include "hs_ptx.cuh"

namespace hs {
namespace {

constexpr int kD = 64;
constexpr int kBM = 128;  // query rows per tile / softmax warpgroup
constexpr int kItemRows = 2 * kBM;
constexpr int kBN = 96;   // keys per KV tile: 4 score buffers x 96 + 2 accumulators x 64 = 512 TMEM columns
constexpr int kPairs = kBN / 2;
constexpr int kStages = 6;
constexpr int kQBufs = 2;                   // Q tiles per warpgroup: the current item's and the next one's
constexpr int kItemSlots = 4;               // item indices handed from the producer to the other warps
constexpr int kItemReaders = 8 + 2;         // one arrival per softmax warp and per MMA warp
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
constexpr int kEmuPer8 = 2;
constexpr uint64_t kSerpentineKvBytes = 24ull << 20;  // K+V bytes of one sequence above which waves alternate direction                // of every 8 exponential pairs, this many run on the FMA pipe

// Site codes written to the status word when a bounded wait gives up.
enum : int {
  kSiteQFull = 0x101,
  kSiteKvFull = 0x102,
  kSiteQEmpty = 0x103,
  kSitePFull = 0x104,
  kSiteSFull = 0x105,
  kSiteODone = 0x106,
  kSiteKvEmpty = 0x107,
  kSiteItemFull = 0x108,
  kSiteItemEmpty = 0x109,
};

// Barrier phases are counted per barrier across all items of a CTA; every
// waiter knows how many completions precede the one it wants.  A parity
// wait cannot tell phase n from phase n +- 2, so every barrier is arranged
// such that, when a waiter asks for completion k, completion k-1 has
// already happened and completion k+1 needs an action the waiter takes
// after this wait: S buffers are doubled by tile parity, Q buffers are
// doubled, and the two PV products at the end of an item (no S behind
// them) each complete a barrier of their own, once per item.
struct Ctrl {
  uint64_t kv_full[kStages];      // K and V tile of a stage landed (one transaction count)
  uint64_t kv_empty[kStages];     // both MMA warps are done with the stage
  uint64_t q_full[2][kQBufs];     // [wg][buf] Q tile landed
  uint64_t q_empty[2][kQBufs];    // the item's last QKᵀ product using that Q tile completed
  uint64_t s_full[2][2];          // [wg][buf]: S(j) landed (with PV(j-2) before it)
  uint64_t p_full[2][2];          // softmax wrote P (and rescaled O) for the tile in that buffer
  uint64_t pv_prev[2];            // PV(n-2) of the item completed (n >= 2)
  uint64_t pv_last[2];            // PV(n-1) of the item completed (with every MMA before it)
  uint64_t drain[2];              // every MMA of that warpgroup's MMA warp completed
  uint64_t item_full[kItemSlots];   // the producer wrote an item index into the slot
  uint64_t item_empty[kItemSlots];  // every reader took it
  uint32_t item_seq[kItemSlots];    // decoded item: sequence s*heads+h (kNoItem: no more work)
  uint32_t item_row0[kItemSlots];   // first query row of the item
  uint32_t item_rev[kItemSlots];    // K/V walk direction of the item
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t kSmemBytes =
    1024 /*alignment slack*/ + 2 * kQBufs * kQTileBytes + 2 * kStages * kKvTileBytes + sizeof(Ctrl);
static_assert(kKvTileBytes % 1024 == 0, "swizzle atoms of each stage must stay 1024-byte aligned");
static_assert(kSmemBytes <= 232448, "shared memory per CTA");

struct Args {
  void* out;
  RowLayout lo;     // output row layout (head-major, or merged token-major)
  uint32_t heads;   // sequence index = s * heads + h
  // Max squared norms of the q' and k' rows (f32 bit patterns, set by
  // qk_prep), or null.  Zeroed by the last CTA, ready for the next call,
  // unless shared: then they bound every launch that carries the same
  // softmax state (ring steps), which may then use the fixed offset too.
  unsigned int* qk_norm2;
  int norm2_shared;
  uint32_t t_q;      // query rows per sequence
  uint32_t t_kv;     // keys per sequence
  uint32_t n_kv;     // ceil(t_kv / kBN)
  uint32_t pairs;    // items per sequence: ceil(t_q / 256)
  uint32_t n_items;  // sequences x pairs
  int out_f32;
  float scale_log2;
  AttnState st;
  int* status;
  uint32_t* sched;  // [0] items handed out beyond the first gridDim.x, [1] CTAs finished
  uint64_t timeout_ns;
  uint32_t serp_wave;  // 0: every item walks K/V forward; else item i walks it backward when (i / serp_wave) is odd
};

struct Item {
  uint32_t seq;       // s * heads + h
  uint32_t row0;      // first query row of the item
  uint32_t rev = 0;   // 1: the item takes its K/V tiles last to first
};

__device__ __forceinline__ Item decode_item(const Args& a, uint32_t item) {
  const uint32_t seq = item / a.pairs;
  const uint32_t rev = a.serp_wave ? (item / a.serp_wave) & 1u : 0u;
  return Item{seq, (item - seq * a.pairs) * kItemRows, rev};
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

constexpr uint32_t kNoItem = 0xffffffffu;

// Position in the K/V stage ring: stage index and the parity of its use count.
struct RingPos {
  uint32_t stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1;
    }
  }
};

// Bounded wait whose outcome is the same for all 32 lanes, so the
// .sync.aligned tcgen05 instructions that follow never see a split warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int site, uint64_t timeout_ns) {
  const bool r = mbar_wait(bar, parity, abort_flag, status, site, timeout_ns);
  return __all_sync(0xffffffffu, r);
}

// Next item index for a reader warp (all lanes): waits for slot k % kItemSlots,
// reads it, and releases the slot with one arrival per warp.  Returns false
// on timeout/abort.
__device__ __forceinline__ bool next_item(const Args& a, Ctrl* ctl, uint32_t k, Item* item) {
  const uint32_t slot = k % kItemSlots;
  if (!warp_wait(&ctl->item_full[slot], (k / kItemSlots) & 1, &ctl->abort_flag, a.status, kSiteItemFull,
                 a.timeout_ns))
    return false;
  item->seq = *reinterpret_cast<volatile uint32_t*>(&ctl->item_seq[slot]);
  item->row0 = *reinterpret_cast<volatile uint32_t*>(&ctl->item_row0[slot]);
  item->rev = *reinterpret_cast<volatile uint32_t*>(&ctl->item_rev[slot]);
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&ctl->item_empty[slot]);
  return true;
}

// One arrival from a converged warp (the elected lane).
__device__ __forceinline__ void mbar_arrive_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// ---- the FMA-pipe exp2 (packed f32x2 helpers: hs_ptx.cuh) ----------------

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

// kFixed: every score is known to be bounded (Cauchy-Schwarz on the stored
// q' and k' rows), so P = 2^(s*c - m_fixed) for a fixed offset m_fixed
// stays inside the 16-bit type's normal range: no row max, no rescale.
template <typename E, bool kFixed>
__device__ void softmax_role(const Args& a, Ctrl* ctl, uint32_t tmem, int warp, int lane, float m_fixed) {
  const int wg = warp >> 2;
  const int wq = warp & 3;
  const uint32_t row = static_cast<uint32_t>(wq * 32 + lane);
  volatile int* abort_flag = &ctl->abort_flag;
  const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
  const uint32_t tO = tmem + lane_base + col_o(wg);
  const float c = a.scale_log2;
  const uint32_t n = a.n_kv;
  const uint32_t tail = a.t_kv - (n - 1) * kBN;  // valid keys in the last tile, 1..kBN
  // Completions per item: s_full[b] once per S tile with j % 2 == b;
  // pv_prev and pv_last once each.  Only the parities of the completion
  // counts before an item matter; they are packed into one register: bit 0
  // s_full[0], bit 1 s_full[1], bit 2 pv_prev and pv_last.  Per item the
  // counts grow by ceil(n/2), floor(n/2) and 1.
  const uint32_t step_bits = (((n + 1) >> 1) & 1) | (((n >> 1) & 1) << 1) | 4u;
  uint32_t base_bits = 0;
  auto s_parity = [&](uint32_t t) { return ((base_bits >> (t & 1)) + (t >> 1)) & 1; };

  Item nxt{};
  bool have_nxt = false;
  for (uint32_t k = 0;; ++k) {
    Item it;
    if (have_nxt) {
      it = nxt;
      have_nxt = false;
    } else if (!next_item(a, ctl, k, &it)) {
      return;
    }
    if (it.seq == kNoItem) break;
    const uint32_t tile0 = it.row0 + wg * kBM;
    if (tile0 >= a.t_q) continue;  // this warpgroup has no rows in the item
    const uint32_t token = tile0 + row;
    const bool valid = token < a.t_q;
    const uint64_t row_index = static_cast<uint64_t>(it.seq) * a.t_q + token;  // head-major (state arrays)
    const uint64_t out_index = a.lo.at(it.seq / a.heads, it.seq % a.heads, token);

    float m_run = kFixed ? m_fixed : -INFINITY, l = 0.f;
    bool have_o = false;
    if (a.st.load && valid) {
      m_run = a.st.m[row_index];
      l = a.st.l[row_index];
    }
    if (a.st.load) {
      // Seed O in TMEM with the carried accumulator (zeros for padding rows).
      // The previous item's epilogue finished reading O (tcgen05.wait::ld).
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

    for (uint32_t j = 0; j < n; ++j) {
      const int b = static_cast<int>(j & 1);
      if (!warp_wait(&ctl->s_full[wg][b], s_parity(j), abort_flag, a.status, kSiteSFull, a.timeout_ns)) return;
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + col_s(wg, b);
      uint32_t s[kBN];
      tmem_ld32(tS + 0, s + 0);
      tmem_ld32(tS + 32, s + 32);
      tmem_ld32(tS + 64, s + 64);
      tmem_wait_ld_regs<kBN>(s);
      if (j == (it.rev ? 0u : n - 1) && tail < kBN) {
#pragma unroll
        for (int i = 0; i < kBN; ++i)
          if (static_cast<uint32_t>(i) >= tail) s[i] = __float_as_uint(-INFINITY);
      }
      float factor = 1.f;
      bool need = false;
      if constexpr (!kFixed) {
        // Row max: 3-input max in four independent chains.
        float m4[4] = {u2f(s[0]), u2f(s[1]), u2f(s[2]), u2f(s[3])};
#pragma unroll
        for (int i = 4; i < kBN; i += 2) m4[(i >> 1) & 3] = max3(m4[(i >> 1) & 3], u2f(s[i]), u2f(s[i + 1]));
        const float m_tile = max3(fmaxf(m4[0], m4[1]), m4[2], m4[3]) * c;
        if (!have_o) {
          m_run = m_tile;
        } else if (m_tile > m_run + kRescaleThreshold) {
          factor = ex2_approx(m_run - m_tile);
          m_run = m_tile;
          l *= factor;
          need = true;
        }
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
      // O rescale (rare), once PV(j-1) has landed.  PV(j-1) was committed
      // together with S(j+1) when that tile exists, else (j = n-1) as the
      // item's first PV-only batch.  PV(j) is issued only after p_full, so it
      // accumulates onto the rescaled O.
      if (!kFixed && __any_sync(0xffffffffu, need)) {
        if (j > 0) {
          const bool ok = (j + 1 < n) ? warp_wait(&ctl->s_full[wg][(j + 1) & 1], s_parity(j + 1), abort_flag,
                                                  a.status, kSiteODone, a.timeout_ns)
                                      : warp_wait(&ctl->pv_prev[wg], (base_bits >> 2) & 1, abort_flag,
                                                  a.status, kSiteODone, a.timeout_ns);
          if (!ok) return;
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

    // The next item's hand-off while PV(n-1) runs.
    if (!next_item(a, ctl, k + 1, &nxt)) return;
    have_nxt = true;
    // PV(n-1) and every MMA before it have completed: the item's pv_last.
    if (!warp_wait(&ctl->pv_last[wg], (base_bits >> 2) & 1, abort_flag, a.status, kSiteODone, a.timeout_ns))
      return;
    tc_fence_after();
    base_bits ^= step_bits;

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
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + out_index + 32 * h);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(u2f(o[4 * i]) * inv_l, u2f(o[4 * i + 1]) * inv_l, u2f(o[4 * i + 2]) * inv_l,
                                 u2f(o[4 * i + 3]) * inv_l);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<E*>(a.out) + out_index + 32 * h);
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
}

// Fixed-offset softmax: with |s*c| <= B for every score, P = 2^(s*c - m)
// lies in [2^(-B-m), 2^(B-m)].  bf16 (8 exponent bits): m = B, so P <= 1,
// for B <= 48 (valid keys keep P >= 2^-96, ~30 binades above anything a
// masked key can round to).  f16 (5 exponent bits): m = B - 15.5, so P <=
// 2^15.5 < 65504 and P >= 2^(15.5 - 2B) >= 2^-12.5 (normal) for B <= 14.
template <typename E>
__host__ __device__ constexpr float fixed_offset_limit() { return Elem<E>::kBf16 ? 48.f : 14.f; }
template <typename E>
__host__ __device__ constexpr float fixed_offset_headroom() { return Elem<E>::kBf16 ? 0.f : 15.5f; }

template <typename E>
__device__ void softmax_dispatch(const Args& a, Ctrl* ctl, uint32_t tmem, int warp, int lane) {
  float bound = INFINITY;
  if (a.qk_norm2 && (a.norm2_shared || (!a.st.load && !a.st.store))) {
    const float qn = sqrtf(__uint_as_float(a.qk_norm2[0]));
    const float kn = sqrtf(__uint_as_float(a.qk_norm2[1]));
    // Margin for the f32 accumulation inside the tensor core.
    bound = qn * kn * a.scale_log2 * 1.0009765625f + 1e-3f;
  }
  if (bound <= fixed_offset_limit<E>())
    softmax_role<E, true>(a, ctl, tmem, warp, lane, bound - fixed_offset_headroom<E>());
  else
    softmax_role<E, false>(a, ctl, tmem, warp, lane, 0.f);
}

// One thread.  Per item: the Q tiles of the warpgroups with rows in it, then
// the item's K/V tiles through the stage ring.
__device__ void producer_role(const Args& a, const CUtensorMap* tm_q, const CUtensorMap* tm_k,
                              const CUtensorMap* tm_v, uint8_t* sQ, uint8_t* sK, uint8_t* sV, Ctrl* ctl) {
  volatile int* abort_flag = &ctl->abort_flag;
  uint32_t q_issued[2] = {0, 0};
  uint32_t g = 0;  // K/V tiles issued so far
  bool ok = true;
  uint32_t item = blockIdx.x;  // a CTA's first item is its index; later ones come from the counter
  for (uint32_t k = 0; ok; ++k) {
    const uint32_t slot = k % kItemSlots;
    if (k >= kItemSlots && !mbar_wait(&ctl->item_empty[slot], ((k / kItemSlots) - 1) & 1, abort_flag, a.status,
                                      kSiteItemEmpty, a.timeout_ns))
      break;
    const Item it = item < a.n_items ? decode_item(a, item) : Item{kNoItem, 0};
    ctl->item_seq[slot] = it.seq;
    ctl->item_row0[slot] = it.row0;
    ctl->item_rev[slot] = it.rev;
    mbar_arrive(&ctl->item_full[slot]);  // release: the item is visible to the readers' acquire
    if (it.seq == kNoItem) break;
    item = gridDim.x + atomicAdd(a.sched, 1u);  // used one item later: the latency hides behind the loads
#pragma unroll
    for (int wg = 0; wg < 2; ++wg) {
      const uint32_t tile0 = it.row0 + wg * kBM;
      if (!ok || tile0 >= a.t_q) continue;
      const uint32_t qi = q_issued[wg];
      const uint32_t qb = qi % kQBufs;
      if (qi >= kQBufs && !mbar_wait(&ctl->q_empty[wg][qb], ((qi / kQBufs) - 1) & 1, abort_flag, a.status,
                                     kSiteQEmpty, a.timeout_ns)) {
        ok = false;
        continue;
      }
      mbar_arrive_expect_tx(&ctl->q_full[wg][qb], kQTileBytes);
      tma_load_4d(tm_q, &ctl->q_full[wg][qb], sQ + (wg * kQBufs + qb) * kQTileBytes, 0, static_cast<int>(tile0),
                  static_cast<int>(it.seq % a.heads), static_cast<int>(it.seq / a.heads));
      q_issued[wg] = qi + 1;
    }
    const int hh = static_cast<int>(it.seq % a.heads), ss = static_cast<int>(it.seq / a.heads);
    for (uint32_t j = 0; ok && j < a.n_kv; ++j, ++g) {
      const uint32_t st = g % kStages;
      if (g >= kStages &&
          !mbar_wait(&ctl->kv_empty[st], ((g / kStages) - 1) & 1, abort_flag, a.status, kSiteKvEmpty,
                     a.timeout_ns)) {
        ok = false;
        break;
      }
      const int key0 = static_cast<int>((it.rev ? a.n_kv - 1 - j : j) * kBN);
      mbar_arrive_expect_tx(&ctl->kv_full[st], 2 * kKvTileBytes);
      tma_load_4d(tm_k, &ctl->kv_full[st], sK + st * kKvTileBytes, 0, key0, hh, ss);
      tma_load_4d(tm_v, &ctl->kv_full[st], sV + st * kKvTileBytes, 0, key0, hh, ss);
    }
  }
  // Let every load this thread issued land before the CTA can exit (on the
  // normal path they have all been consumed already); fixed teardown bound.
  const uint32_t first = g > kStages ? g - kStages : 0;
  for (uint32_t t = first; t < g; ++t)
    mbar_wait_teardown(&ctl->kv_full[t % kStages], (t / kStages) & 1, a.status, kSiteKvFull);
#pragma unroll
  for (int wg = 0; wg < 2; ++wg) {
    const uint32_t qi = q_issued[wg];
    for (uint32_t t = qi > kQBufs ? qi - kQBufs : 0; t < qi; ++t)
      mbar_wait_teardown(&ctl->q_full[wg][t % kQBufs], (t / kQBufs) & 1, a.status, kSiteQFull);
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
  const uint64_t q_desc0 = sdesc_sw128(smem_u32(sQ + wg * kQBufs * kQTileBytes), 16, 1024);
  const uint64_t k_desc = sdesc_sw128(smem_u32(sK), 16, 1024);
  const uint64_t v_desc = sdesc_sw128(smem_u32(sV), 16, 1024);
  constexpr uint64_t kKvTileStep = kKvTileBytes >> 4;
  constexpr uint64_t kQTileStep = kQTileBytes >> 4;
  const uint32_t o_tmem = tmem + col_o(wg);
  const uint32_t n = a.n_kv;
  uint32_t p_base0 = 0, p_base1 = 0;  // p_full completions before this item, per buffer
  uint32_t q_used = 0;
  RingPos s_pos;   // next K/V tile to wait for (S products, or release when idle)
  RingPos pv_pos;  // next K/V tile whose V feeds a PV product
  const bool acc0 = a.st.load != 0;
  bool ok = true;

  // S[wg][buf] = Q_wg · K_stᵀ: K = 64 as four K=16 steps inside the swizzle atom.
  auto issue_s = [&](uint64_t q_desc, uint32_t st, int buf) {
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
  auto kv_wait = [&](const RingPos& r) {
    return warp_wait(&ctl->kv_full[r.stage], r.phase, abort_flag, a.status, kSiteKvFull, a.timeout_ns);
  };

  // The next item is fetched as soon as the current one's last S product is
  // issued, so the hand-off is off the path from PV(n-1) to the next S(0).
  Item nxt{};
  bool have_nxt = false;
  auto fetch_next = [&](uint32_t k_next) {
    if (!have_nxt) {
      if (!next_item(a, ctl, k_next, &nxt)) return false;
      have_nxt = true;
    }
    return true;
  };
  for (uint32_t k = 0; ok; ++k) {
    Item it;
    if (have_nxt) {
      it = nxt;
      have_nxt = false;
    } else if (!next_item(a, ctl, k, &it)) {
      break;
    }
    if (it.seq == kNoItem) break;
    if (it.row0 + wg * kBM >= a.t_q) {
      // No rows for this warpgroup: release each stage once it has landed
      // (waiting keeps this warp's view of the ring phases exact).
      for (uint32_t j = 0; j < n; ++j, s_pos.next()) {
        if (!kv_wait(s_pos)) {
          ok = false;
          break;
        }
        mbar_arrive_elect(&ctl->kv_empty[s_pos.stage]);
      }
      pv_pos = s_pos;
      continue;
    }
    const uint32_t qb = q_used % kQBufs;
    if (!warp_wait(&ctl->q_full[wg][qb], (q_used / kQBufs) & 1, abort_flag, a.status, kSiteQFull, a.timeout_ns))
      break;
    tc_fence_after();
    const uint64_t q_desc = q_desc0 + qb * kQTileStep;
    // S(0) and S(1) up front.  The commit after the item's last S also frees its Q buffer.
    for (uint32_t t = 0; t < 2 && t < n; ++t) {
      if (!kv_wait(s_pos)) {
        ok = false;
        break;
      }
      issue_s(q_desc, s_pos.stage, static_cast<int>(t));
      s_pos.next();
      umma_commit_elect(&ctl->s_full[wg][t]);
      if (t == n - 1) {
        umma_commit_elect(&ctl->q_empty[wg][qb]);
        if (!fetch_next(k + 1)) ok = false;
      }
    }
    for (uint32_t j = 0; ok && j < n; ++j) {
      const int b = static_cast<int>(j & 1);
      const uint32_t st = pv_pos.stage;  // V_j: this stage was waited on before S(j) was issued
      pv_pos.next();
      if (!warp_wait(&ctl->p_full[wg][b], ((b ? p_base1 : p_base0) + (j >> 1)) & 1, abort_flag, a.status,
                     kSitePFull, a.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      issue_pv(st, b, j > 0 || acc0);
      if (j + 2 < n) {
        if (!kv_wait(s_pos)) {
          ok = false;
          break;
        }
        issue_s(q_desc, s_pos.stage, b);  // after PV(j) in this warp's order: P(j) is read first
        s_pos.next();
        umma_commit_elect(&ctl->s_full[wg][b]);
        if (j + 2 == n - 1) {
          umma_commit_elect(&ctl->q_empty[wg][qb]);
          if (!fetch_next(k + 1)) {
            ok = false;
            break;
          }
        }
      } else {
        umma_commit_elect(j + 1 == n ? &ctl->pv_last[wg] : &ctl->pv_prev[wg]);
      }
      umma_commit_elect(&ctl->kv_empty[st]);  // the producer may refill this stage
    }
    p_base0 += (n + 1) >> 1;
    p_base1 += n >> 1;
    ++q_used;
  }
  // Drain: every MMA this warp issued has completed before TMEM is freed
  // (fixed teardown bound, whatever the caller's timeout).
  umma_commit_elect(&ctl->drain[wg]);
  const bool drained = mbar_wait_teardown(&ctl->drain[wg], 0, a.status, kSiteODone);
  __syncwarp();
  (void)drained;
}

template <typename E>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + 2 * kQBufs * kQTileBytes;
  uint8_t* sV = sK + kStages * kKvTileBytes;
  Ctrl* ctl = reinterpret_cast<Ctrl*>(sV + kStages * kKvTileBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->kv_full[s], 1);
      mbar_init(&ctl->kv_empty[s], 2);  // one arrival per MMA warp
    }
    for (int i = 0; i < 2; ++i) {
      for (int b = 0; b < kQBufs; ++b) {
        mbar_init(&ctl->q_full[i][b], 1);
        mbar_init(&ctl->q_empty[i][b], 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(&ctl->s_full[i][b], 1);
        mbar_init(&ctl->p_full[i][b], kBM / 32);
      }
      mbar_init(&ctl->pv_prev[i], 1);
      mbar_init(&ctl->pv_last[i], 1);
      mbar_init(&ctl->drain[i], 1);
    }
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&ctl->item_full[i], 1);
      mbar_init(&ctl->item_empty[i], kItemReaders);
    }
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
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
  // the control warpgroup keeps 56: 2*224 + 56 == 3*168.  (The same code
  // without the split, at 384 or 352 threads, measured 4-5 % slower.)
  if (warp < 8) {
    regs_inc<kSoftmaxRegs>();
    softmax_dispatch<E>(a, ctl, tmem, warp, lane);
  } else {
    regs_dec<kControlRegs>();
    if (warp == kProducerWarp) {
      if (lane == 0) producer_role(a, &tm_q, &tm_k, &tm_v, sQ, sK, sV, ctl);
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
  // The last CTA to finish returns the counter to zero for the next launch
  // on this stream (every fetch of every CTA happened before its arrival).
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.sched[1], 1u) == gridDim.x - 1) {
      atomicExch(&a.sched[0], 0u);
      atomicExch(&a.sched[1], 0u);
      if (a.qk_norm2 && !a.norm2_shared) {  // every CTA read the bounds at its start
        atomicExch(&a.qk_norm2[0], 0u);
        atomicExch(&a.qk_norm2[1], 0u);
      }
    }
  }
}

// (S, H, T, 64) 16-bit tensor in row layout `l` as a 4-D map (64, T, H, S)
// with box_rows x 64 boxes, 128B swizzle (launch_util.cu).  Rows past T
// inside a sequence read as zeros (out-of-bounds fill).
bool make_map(CUtensorMap* map, const void* base, const RowLayout& l, bool bf16, uint32_t t, uint32_t heads,
              uint32_t seqs, uint32_t box_rows, std::string* err) {
  return make_row_map(map, base, l, bf16, t, heads, seqs, box_rows, err);
}

int sm_count_of_current_device() { return current_sm_count(); }

template <typename E>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                         const Args& a, uint32_t ctas) {
  const cudaError_t e =
      ensure_dynamic_smem(reinterpret_cast<const void*>(attn_fwd_sm100<E>), static_cast<int>(kSmemBytes));
  if (e != cudaSuccess) return e;
  attn_fwd_sm100<E><<<ctas, kThreads, kSmemBytes, stream>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_sm100(cudaStream_t stream, int elem, const AttnIO& io, uint32_t S, uint32_t H,
                                   uint32_t t_q, uint32_t t_kv, float scale, const AttnState& st, uint32_t max_ctas,
                                   int* status, uint32_t* sched, unsigned int* qk_norm2, bool norm2_shared,
                                   uint64_t timeout_ns, std::string* err) {
  const uint32_t sh = S * H;
  if (t_q == 0 || sh == 0) return cudaSuccess;
  const bool bf16 = elem == kBF16;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, io.q, io.lq, bf16, t_q, H, S, kBM, err) || !make_map(&mk, io.k, io.lk, bf16, t_kv, H, S, kBN, err) ||
      !make_map(&mv, io.v, io.lv, bf16, t_kv, H, S, kBN, err))
    return cudaErrorInvalidValue;
  Args a{};
  a.out = io.out;
  a.lo = io.lo;
  a.heads = H;
  a.t_q = t_q;
  a.t_kv = t_kv;
  a.n_kv = (t_kv + kBN - 1) / kBN;
  a.pairs = (t_q + kItemRows - 1) / kItemRows;
  const uint64_t items = static_cast<uint64_t>(sh) * a.pairs;
  if (items > 0x7fffffffull) {
    if (err) *err = "too many work items";
    return cudaErrorInvalidValue;
  }
  a.n_items = static_cast<uint32_t>(items);
  a.out_f32 = io.out_code == kF32;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.st = st;
  a.status = status;
  a.sched = sched;
  a.qk_norm2 = qk_norm2;
  a.norm2_shared = norm2_shared ? 1 : 0;
  a.timeout_ns = timeout_ns;
  uint32_t ctas = max_ctas ? max_ctas : static_cast<uint32_t>(sm_count_of_current_device());
  if (ctas > a.n_items) ctas = a.n_items;
  // A sequence whose K and V outgrow a fraction of L2: the CTAs that start
  // items at about the same time (one wave of `ctas` items) stream its K/V
  // together, and alternate waves walk it in opposite directions, so a wave
  // starts on the tiles the previous one has just brought into L2.
  if (static_cast<uint64_t>(a.n_kv) * 2 * kKvTileBytes > kSerpentineKvBytes) a.serp_wave = ctas;
  return bf16 ? launch_typed<__nv_bfloat16>(stream, mq, mk, mv, a, ctas)
              : launch_typed<__half>(stream, mq, mk, mv, a, ctas);
}

}  // namespace hs
