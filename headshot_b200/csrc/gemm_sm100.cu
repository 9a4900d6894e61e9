// gemm_sm100.cu — the block's linears on tcgen05, with the element-wise op
// that follows each of them in Block::forward fused into the epilogue.
//
// Replaces GpuContext::linear (src/engine/ops.rs:87-128, shaders/linear.wesl
// and linear_wmma.wgsl): out (M, N) = x (M, K) · w (N, K)ᵀ [+ bias (N, f32)],
// 16-bit storage, f32 accumulation.  Epilogues:
//   kEpiNone      out = x·wᵀ + b
//   kEpiGelu      out = gelu(x·wᵀ + b)              (MLP fc1 + GELU, block.rs:173-174;
//                 erf-based GELU, shaders/gelu.wesl)
//   kEpiResidual  out = res + gamma ⊙ (x·wᵀ + b)    (proj / fc2 + LayerScale residual,
//                 block.rs:150-155, shaders/residual_ls.wesl)
// The reference rounds the linear's output to the storage type before the
// element-wise kernel reads it; here it stays f32 into the epilogue.
//
// Persistent: one CTA per SM walks 128x256 output tiles (static stride).
//   warp 0      TMA producer: A (128x64) and B (256x64) K-blocks, 128B swizzle, kStages ring
//   warp 1      UMMA issue (whole warp, elect.sync): M=128, N=256, K=16, f32 in TMEM
//   warp 2      TMEM owner (512 columns = two 256-column accumulators)
//   warps 4-11  two epilogue warpgroups: one thread per output row of the
//               tile, each warpgroup taking half of the tile's 256 columns;
//               each warp stages its 32x32 output blocks in shared memory
//               and writes them with TMA stores (coalesced, asynchronous)
// The accumulator is double-buffered, so the epilogue of tile i overlaps the
// MMAs of tile i+1.  Every wait is bounded (hs_ptx.cuh) and every waiter
// waits completions in order.
#include <cuda.h>

#include <mutex>

#include "hs_internal.h"
#include "hs_ptx.cuh"

namespace hs {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // one 128-byte swizzle atom of 16-bit elements
constexpr int kStages = 4;
constexpr int kATileBytes = kBM * kBK * 2;  // 16 KiB
constexpr int kBTileBytes = kBN * kBK * 2;  // 32 KiB
constexpr int kThreads = 384;
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kTmemWarp = 2;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kEpiCols = kBN / (kEpiWarps / 4);  // columns per epilogue warpgroup
constexpr uint32_t kTmemCols = 512;

enum : int {
  kSiteFull = 0x201,
  kSiteEmpty = 0x202,
  kSiteAccFull = 0x203,
  kSiteAccEmpty = 0x204,
  kSiteDrain = 0x205,
};

struct Ctrl {
  uint64_t full[kStages];    // A and B K-block landed
  uint64_t empty[kStages];   // the MMAs reading the stage completed
  uint64_t acc_full[2];      // the tile's MMAs completed in accumulator b
  uint64_t acc_empty[2];     // the epilogue finished reading accumulator b (one arrival per warp)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr int kStageOutBytes = 32 * 32 * 2;  // one warp's 32x32 16-bit output block
constexpr size_t kSmemBytes =
    1024 + kStages * (kATileBytes + kBTileBytes) + kEpiWarps * 2 * kStageOutBytes + sizeof(Ctrl);
static_assert(kSmemBytes <= 232448, "shared memory per CTA");

struct Args {
  void* out;
  const void* res;     // kEpiResidual: (M, N) residual rows
  const float* bias;   // (N) or null
  const float* gamma;  // kEpiResidual: (N) LayerScale
  uint64_t m;
  uint32_t n, k;
  uint32_t m_tiles, n_tiles, k_blocks;
  uint32_t n_tiles_total;  // m_tiles * n_tiles
  int epi;
  int* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int site, uint64_t timeout_ns) {
  const bool r = mbar_wait(bar, parity, abort_flag, status, site, timeout_ns);
  return __all_sync(0xffffffffu, r);
}

// Packed f32x2 arithmetic (sm_100).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }

// GELU(v) = 0.5 v (1 + erf(v / sqrt 2)) on a pair, erf by Abramowitz &
// Stegun 7.1.26 (|error| <= 1.5e-7), the formula the reference's GELU kernel
// uses (shaders/gelu.wesl:16-26).  The fast reciprocal and exponential
// intrinsics keep the epilogue short; their relative error (~1e-6) is far
// below the 16-bit output rounding.
__device__ __forceinline__ float2 gelu_erf2(float2 v) {
  const float2 x = mul2(v, splat(0.70710678118654752f));
  const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 d = fma2(a, splat(0.3275911f), splat(1.0f));
  const float2 t = make_float2(__fdividef(1.0f, d.x), __fdividef(1.0f, d.y));
  float2 p = fma2(t, splat(1.061405429f), splat(-1.453152027f));
  p = fma2(p, t, splat(1.421413741f));
  p = fma2(p, t, splat(-0.284496736f));
  p = fma2(p, t, splat(0.254829592f));
  p = mul2(p, t);
  const float2 q = mul2(a, make_float2(-a.x, -a.y));
  const float2 ex = make_float2(__expf(q.x), __expf(q.y));
  const float2 e = fma2(make_float2(-p.x, -p.y), ex, splat(1.0f));
  const float2 h = mul2(v, splat(0.5f));
  return fma2(h, make_float2(copysignf(e.x, x.x), copysignf(e.y, x.y)), h);
}

// 32 consecutive f32 values of a per-column vector (bias, gamma), or zeros.
__device__ __forceinline__ void load_cols32(const float* p, uint32_t col0, uint32_t n, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p && col0 + 4 * q < n) f = __ldg(reinterpret_cast<const float4*>(p + col0) + q);
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

__device__ void producer_role(const Args& a, const CUtensorMap* tm_a, const CUtensorMap* tm_b, uint8_t* sA,
                              uint8_t* sB, Ctrl* ctl) {
  volatile int* abort_flag = &ctl->abort_flag;
  uint32_t g = 0;  // K-blocks issued
  bool ok = true;
  for (uint32_t tile = blockIdx.x; ok && tile < a.n_tiles_total; tile += gridDim.x) {
    const int m0 = static_cast<int>((tile / a.n_tiles) * kBM);
    const int n0 = static_cast<int>((tile % a.n_tiles) * kBN);
    for (uint32_t kb = 0; kb < a.k_blocks; ++kb, ++g) {
      const uint32_t st = g % kStages;
      if (g >= kStages &&
          !mbar_wait(&ctl->empty[st], ((g / kStages) - 1) & 1, abort_flag, a.status, kSiteEmpty, a.timeout_ns)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&ctl->full[st], kATileBytes + kBTileBytes);
      tma_load_3d(tm_a, &ctl->full[st], sA + st * kATileBytes, static_cast<int>(kb * kBK), m0, 0);
      tma_load_3d(tm_b, &ctl->full[st], sB + st * kBTileBytes, static_cast<int>(kb * kBK), n0, 0);
    }
  }
  const uint32_t first = g > kStages ? g - kStages : 0;
  for (uint32_t t = first; t < g; ++t)
    mbar_wait_teardown(&ctl->full[t % kStages], (t / kStages) & 1, a.status, kSiteFull);
}

template <bool kBf16>
__device__ void mma_role(const Args& a, uint8_t* sA, uint8_t* sB, Ctrl* ctl, uint32_t tmem) {
  volatile int* abort_flag = &ctl->abort_flag;
  constexpr uint32_t idesc = idesc_f16(kBf16, kBM, kBN, false, false);
  const uint64_t a_desc = sdesc_sw128(smem_u32(sA), 16, 1024);
  const uint64_t b_desc = sdesc_sw128(smem_u32(sB), 16, 1024);
  uint32_t g = 0;
  uint32_t i = 0;  // tiles of this CTA
  bool ok = true;
  for (uint32_t tile = blockIdx.x; ok && tile < a.n_tiles_total; tile += gridDim.x, ++i) {
    const uint32_t ab = i & 1;
    // Accumulator ab was last used by tile i-2: wait until its epilogue has read it.
    if (i >= 2 && !warp_wait(&ctl->acc_empty[ab], ((i >> 1) - 1) & 1, abort_flag, a.status, kSiteAccEmpty,
                             a.timeout_ns))
      break;
    tc_fence_after();
    const uint32_t d = tmem + ab * kBN;
    for (uint32_t kb = 0; kb < a.k_blocks; ++kb, ++g) {
      const uint32_t st = g % kStages;
      if (!warp_wait(&ctl->full[st], (g / kStages) & 1, abort_flag, a.status, kSiteFull, a.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t ad = a_desc + st * (kATileBytes >> 4);
      const uint64_t bd = b_desc + st * (kBTileBytes >> 4);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        umma_ss_elect(d, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
      umma_commit_elect(&ctl->empty[st]);
    }
    if (ok) umma_commit_elect(&ctl->acc_full[ab]);
  }
  umma_commit_elect(&ctl->drain);
  mbar_wait_teardown(&ctl->drain, 0, a.status, kSiteDrain);
  __syncwarp();
}

template <typename E>
__device__ void epilogue_role(const Args& a, const CUtensorMap* tm_out, uint8_t* sOut, Ctrl* ctl, uint32_t tmem,
                              int warp, int lane) {
  volatile int* abort_flag = &ctl->abort_flag;
  const int wq = (warp - kEpiWarp0) & 3;                  // TMEM lane quadrant of this warp
  const uint32_t col_base = ((warp - kEpiWarp0) >> 2) * kEpiCols;  // this warpgroup's columns
  const uint32_t row_in_tile = static_cast<uint32_t>(wq * 32 + lane);
  const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
  uint8_t* stage_base = sOut + (warp - kEpiWarp0) * 2 * kStageOutBytes;
  uint32_t blocks = 0;  // output blocks this warp has stored (alternating staging buffers)
  uint32_t i = 0;
  for (uint32_t tile = blockIdx.x; tile < a.n_tiles_total; tile += gridDim.x, ++i) {
    const uint32_t ab = i & 1;
    // On a timeout, leave the loop but still wait for this warp's stores below.
    if (!warp_wait(&ctl->acc_full[ab], (i >> 1) & 1, abort_flag, a.status, kSiteAccFull, a.timeout_ns)) break;
    tc_fence_after();
    const uint64_t row = static_cast<uint64_t>(tile / a.n_tiles) * kBM + row_in_tile;
    const uint32_t n0 = (tile % a.n_tiles) * kBN;
    const bool row_ok = row < a.m;
#pragma unroll 1
    for (int c = 0; c < kEpiCols / 32; ++c) {
      const uint32_t col0 = n0 + col_base + 32 * c;
      uint32_t acc[32];
      tmem_ld32(tmem + lane_base + ab * kBN + col_base + 32 * c, acc);
      tmem_wait_ld_regs<32>(acc);
      if (col0 >= a.n || row - lane >= a.m) continue;  // warp-uniform: nothing of this block is stored
      float v[32];
      load_cols32(a.bias, col0, a.n, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(acc[j]);
      if (a.epi == kEpiGelu) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 r = gelu_erf2(make_float2(v[j], v[j + 1]));
          v[j] = r.x;
          v[j + 1] = r.y;
        }
      } else if (a.epi == kEpiResidual && row_ok) {
        const E* res = static_cast<const E*>(a.res) + row * a.n + col0;
        float g[32];
        load_cols32(a.gamma, col0, a.n, g);
#pragma unroll
        for (int j8 = 0; j8 < 4; ++j8) {
          if (col0 + 8 * j8 >= a.n) break;
          const uint4 r = __ldg(reinterpret_cast<const uint4*>(res + 8 * j8));
          const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 f = Elem<E>::unpack2(w[u]);
            const int j = 8 * j8 + 2 * u;
            v[j] = f.x + g[j] * v[j];
            v[j + 1] = f.y + g[j + 1] * v[j + 1];
          }
        }
      }
      // Stage this warp's 32 rows x 32 columns (row = lane) and store the
      // block with one TMA store; rows past M and columns past N are clipped.
      uint8_t* stage = stage_base + (blocks & 1) * kStageOutBytes;
      if (blocks >= 2) {
        if (lane == 0) bulk_wait_group_read<1>();  // the store that used this buffer has read it
        __syncwarp();
      }
      uint4* srow = reinterpret_cast<uint4*>(stage + lane * 64);
#pragma unroll
      for (int j8 = 0; j8 < 4; ++j8) {
        uint4 o;
        o.x = Elem<E>::pack2(v[8 * j8 + 0], v[8 * j8 + 1]);
        o.y = Elem<E>::pack2(v[8 * j8 + 2], v[8 * j8 + 3]);
        o.z = Elem<E>::pack2(v[8 * j8 + 4], v[8 * j8 + 5]);
        o.w = Elem<E>::pack2(v[8 * j8 + 6], v[8 * j8 + 7]);
        srow[j8] = o;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tm_out, stage, static_cast<int>(col0), static_cast<int>(row - lane));
        bulk_commit_group();
      }
      ++blocks;
    }
    // The accumulator may be overwritten once every warp has read it.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ctl->acc_empty[ab]);
  }
  if (lane == 0) bulk_wait_group<0>();  // every store of this warp has landed before the CTA exits
  __syncwarp();
}

template <typename E>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sm100(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
               const __grid_constant__ CUtensorMap tm_out, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kStages * kATileBytes;
  uint8_t* sOut = sB + kStages * kBTileBytes;
  Ctrl* ctl = reinterpret_cast<Ctrl*>(sOut + kEpiWarps * 2 * kStageOutBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == kTmemWarp) {
    tmem_alloc(&ctl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == kProducerWarp) {
    if (lane == 0) producer_role(a, &tm_a, &tm_b, sA, sB, ctl);
  } else if (warp == kMmaWarp) {
    mma_role<Elem<E>::kBf16>(a, sA, sB, ctl, tmem);
  } else if (warp >= kEpiWarp0) {
    epilogue_role<E>(a, &tm_out, sOut, ctl, tmem, warp, lane);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kTmemWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

EncodeTiledFn encode_fn() { return encode_tiled_fn(); }

// Row-major (rows, cols) 16-bit output as a 2-D map with 32x32 boxes, no
// swizzle (the epilogue's staging layout).
bool make_out_map(CUtensorMap* map, void* base, bool bf16, uint64_t rows, uint32_t cols, std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled (output) failed with code " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

// Row-major (rows, cols) 16-bit matrix as a 3-D map (cols, rows, 1) with
// box_rows x 64 boxes, 128B swizzle; out-of-range rows and columns read 0.
bool make_map(CUtensorMap* map, const void* base, bool bf16, uint64_t rows, uint32_t cols, uint32_t box_rows,
              std::string* err) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    if (err) *err = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), 1};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols) * 2, static_cast<cuuint64_t>(cols) * 2 * rows};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), box_rows, 1};
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

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

template <typename E>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                         const Args& a, uint32_t ctas) {
  const cudaError_t e =
      ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_sm100<E>), static_cast<int>(kSmemBytes));
  if (e != cudaSuccess) return e;
  gemm_sm100<E><<<ctas, kThreads, kSmemBytes, stream>>>(ma, mb, mo, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_linear_sm100(cudaStream_t stream, int elem, const void* x, const void* w, const float* bias,
                                void* out, uint64_t m, uint32_t k, uint32_t n, int epi, const void* res,
                                const float* gamma, int* status, uint64_t timeout_ns, std::string* err) {
  if (m == 0 || n == 0) return cudaSuccess;
  const bool bf16 = elem == kBF16;
  CUtensorMap ma, mb, mo;
  if (!make_map(&ma, x, bf16, m, k, kBM, err) || !make_map(&mb, w, bf16, n, k, kBN, err) ||
      !make_out_map(&mo, out, bf16, m, n, err))
    return cudaErrorInvalidValue;
  Args a{};
  a.out = out;
  a.res = res;
  a.bias = bias;
  a.gamma = gamma;
  a.m = m;
  a.n = n;
  a.k = k;
  a.m_tiles = static_cast<uint32_t>((m + kBM - 1) / kBM);
  a.n_tiles = (n + kBN - 1) / kBN;
  a.k_blocks = (k + kBK - 1) / kBK;
  const uint64_t tiles = static_cast<uint64_t>(a.m_tiles) * a.n_tiles;
  if (tiles > 0x7fffffffull) {
    if (err) *err = "too many output tiles";
    return cudaErrorInvalidValue;
  }
  a.n_tiles_total = static_cast<uint32_t>(tiles);
  a.epi = epi;
  a.status = status;
  a.timeout_ns = timeout_ns;
  uint32_t ctas = static_cast<uint32_t>(sm_count());
  if (ctas > a.n_tiles_total) ctas = a.n_tiles_total;
  return bf16 ? launch_typed<__nv_bfloat16>(stream, ma, mb, mo, a, ctas)
              : launch_typed<__half>(stream, ma, mb, mo, a, ctas);
}

}  // namespace hs
