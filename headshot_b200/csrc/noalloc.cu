// noalloc.cu — hs_attention_fused_noalloc: the fused QK-norm + RoPE +
// attention op for callers that must not have the library allocate device
// memory.
//
// Who needs it: a host whose device memory is owned by its own allocator or
// fixed, pre-reserved pool (an embedding engine, a Rust host that budgets
// every buffer up front), and session loops that must not stall or fail on
// an allocation once they are running.  hs_attention_fused grows a scratch
// buffer with cudaMallocAsync for the normalised/rotated Q and K; this
// variant uses a fixed array compiled into the library instead and calls no
// cudaMalloc, cudaFree or other allocating routine.
//
// The array is a file-scope __device__ object, so every GPU that loads the
// library holds its kNoAllocScratchBytes until the process exits.  All calls
// on a device share it: two calls whose work overlaps on the GPU (different
// streams, no ordering between them) race on it.  Each call rewrites every
// row of the scratch it reads, so stale contents of an earlier call are
// never used; the status word is cleared at the start of each call.
#include <math.h>

#include <mutex>
#include <string>

#include "../../include/headshot_cuda.h"
#include "hs_abi_ctx.h"
#include "hs_internal.h"

namespace {

constexpr size_t kNoAllocRegionBytes = static_cast<size_t>(HS_NOALLOC_MAX_ROWS) * 64 * 2;
constexpr size_t kNoAllocScratchBytes = 2 * kNoAllocRegionBytes;  // Q rows, then K rows
constexpr int kMaxDevices = 64;
constexpr uint64_t kNoAllocTimeoutNs = 2000ull * 1000000ull;

// Normalised/rotated Q rows, then K rows (16-bit, 128 bytes per row of D = 64).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Bounded-wait status word used when the caller passes no status pointer.
static __device__ __align__(256) int g_noalloc_status[4];
// Work counter pair of the persistent attention kernel, then the q'/k'
// max squared row norms (all zero between calls).
static __device__ __align__(256) uint32_t g_noalloc_sched[4];

struct DevicePtrs {
  void* scratch = nullptr;
  int* status = nullptr;
  uint32_t* sched = nullptr;
};

std::mutex g_mu;
DevicePtrs g_ptrs[kMaxDevices];

// Device addresses of the three arrays on the current device, looked up once
// per device.  In host code the arrays' names only stand for the symbols;
// cudaGetSymbolAddress turns them into device addresses.
hs_status device_ptrs(int dev, DevicePtrs* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  DevicePtrs& p = g_ptrs[dev];
  if (!p.scratch) {
    void* s = nullptr;
    void* st = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&s, g_noalloc_scratch);
    if (e != cudaSuccess)
      return hs::abi_fail(HS_ERR_CUDA, std::string("hs_attention_fused_noalloc: scratch address: ") +
                                           cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess)
      return hs::abi_fail(HS_ERR_CUDA, std::string("hs_attention_fused_noalloc: status address: ") +
                                           cudaGetErrorString(e));
    void* sc = nullptr;
    e = cudaGetSymbolAddress(&sc, g_noalloc_sched);
    if (e != cudaSuccess)
      return hs::abi_fail(HS_ERR_CUDA, std::string("hs_attention_fused_noalloc: counter address: ") +
                                           cudaGetErrorString(e));
    p.scratch = s;
    p.status = static_cast<int*>(st);
    p.sched = static_cast<uint32_t*>(sc);
  }
  *out = p;
  return HS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" hs_status hs_attention_fused_noalloc(void* stream, int* status, const void* q, const void* k,
                                                const void* v, void* out, uint32_t S, uint32_t H, uint32_t T,
                                                uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                                                const float* q_norm_b, const float* k_norm_w,
                                                const float* k_norm_b, float eps, const float* rope_sin,
                                                const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                                uint32_t tokens_per_frame) {
  const char* name = "hs_attention_fused_noalloc";
  if (dtype != HS_F16 && dtype != HS_BF16)
    return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": only f16/bf16 storage (f32 needs more scratch)");
  const uint64_t rows = static_cast<uint64_t>(S) * H * T;
  if (rows * D == 0) return HS_OK;
  if (D != 64) return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": head_dim must be 64");
  if (static_cast<uint64_t>(S) * H > 65535u)
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": S*H > 65535");
  if (!q || !k || !v || !out) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": tensor pointers must be 16-byte aligned");
  const bool ln = q_norm_w != nullptr;
  if (ln != (k_norm_w != nullptr) || (ln && (!q_norm_b || !k_norm_b)))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": QK-norm needs all of q/k weight and bias, or none");
  const bool rope = rope_sin != nullptr;
  if (rope && !rope_cos) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": rope_cos missing");
  // Only the normalised/rotated Q and K rows live in the fixed scratch; with
  // neither QK-norm nor RoPE the kernel reads q and k directly and any size
  // the attention kernel takes is accepted.
  if ((ln || rope) && rows > HS_NOALLOC_MAX_ROWS)
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": S*H*T = " + std::to_string(rows) +
                                            " rows exceeds the fixed scratch of " +
                                            std::to_string(HS_NOALLOC_MAX_ROWS) + " rows");
  const uint32_t tpf = tokens_per_frame ? tokens_per_frame : T;
  if (rope) {
    if (prefix > tpf) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": prefix > tokens_per_frame");
    if (rope_rows < tpf - prefix)
      return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": rope tables too short");
    if (!aligned16(rope_sin) || !aligned16(rope_cos))
      return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": rope tables must be 16-byte aligned");
  }
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));

  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hs::abi_cuda_fail(e, name);
  if (dev < 0 || dev >= kMaxDevices) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": device id");
  DevicePtrs p;
  hs_status s = device_ptrs(dev, &p);
  if (s != HS_OK) return s;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status_word = status ? status : p.status;
  e = cudaMemsetAsync(status_word, 0, sizeof(int), st);
  if (e != cudaSuccess) return hs::abi_cuda_fail(e, name);

  hs::QkPrologue qp{};
  qp.ln = ln;
  qp.ln_w = q_norm_w;
  qp.ln_b = q_norm_b;
  qp.eps = eps;
  qp.rope = rope;
  qp.sin_t = rope_sin;
  qp.cos_t = rope_cos;
  qp.prefix = prefix;
  qp.tokens_per_frame = tpf;
  hs::QkPrologue kp = qp;
  kp.ln_w = k_norm_w;
  kp.ln_b = k_norm_b;
  const int code = static_cast<int>(dtype);
  const void* q_use = q;
  const void* k_use = k;
  if (ln || rope) {
    uint8_t* q_rows = static_cast<uint8_t*>(p.scratch);
    uint8_t* k_rows = q_rows + kNoAllocRegionBytes;
    qp.norm2_max = p.sched + 2;
    kp.norm2_max = p.sched + 3;
    const hs::RowLayout hm = hs::RowLayout::head_major(H, T);
    const hs::PrepJob jobs[2] = {{q, hm, q_rows, qp}, {k, hm, k_rows, kp}};
    e = hs::launch_qk_prep(st, code, code, S, H, T, jobs, 2, status_word, kNoAllocTimeoutNs);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, name);
    q_use = q_rows;
    k_use = k_rows;
  }
  std::string err;
  hs::AttnState state{};
  hs::AttnIO io;
  io.q = q_use;
  io.lq = hs::RowLayout::head_major(H, T);
  io.k = k_use;
  io.lk = io.lq;
  io.v = v;
  io.lv = io.lq;
  io.out = out;
  io.lo = io.lq;
  io.out_code = code;
  e = hs::launch_attention_sm100(st, code, io, S, H, T, T, scale, state, 0, status_word, p.sched,
                                 (ln || rope) ? p.sched + 2 : nullptr, false, kNoAllocTimeoutNs, &err);
  if (e != cudaSuccess)
    return hs::abi_fail(HS_ERR_CUDA, std::string(name) + ": " + (err.empty() ? cudaGetErrorString(e) : err));
  return HS_OK;
}
