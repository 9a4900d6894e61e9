// abi.cu — the extern "C" boundary declared in include/headshot_cuda.h.
//
// Validates every argument the way the reference's ops assert them
// (src/engine/ops.rs), turns violations into HS_ERR_INVALID + message,
// and dispatches to the kernels on the context's stream.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <string>

#include "../../include/headshot_cuda.h"
#include "hs_abi_ctx.h"
#include "hs_internal.h"

namespace {

thread_local std::string g_last_error;

hs_status fail(hs_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}

hs_status cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation) return fail(HS_ERR_OOM, std::string(what) + ": " + cudaGetErrorString(e));
  return fail(HS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_dtype(hs_dtype d) { return d == HS_F32 || d == HS_F16 || d == HS_BF16; }

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

namespace hs {

hs_status abi_fail(hs_status s, const std::string& msg) { return fail(s, msg); }
hs_status abi_cuda_fail(cudaError_t e, const char* what) { return cuda_fail(e, what); }

cudaStream_t ctx_stream(hs_ctx* ctx) { return ctx->has_user_stream ? ctx->user_stream : ctx->stream; }

// Grows the context scratch (stream-ordered) to at least `bytes`.
hs_status ctx_scratch(hs_ctx* ctx, size_t bytes, void** out) {
  if (bytes > ctx->scratch_bytes) {
    cudaStream_t st = ctx_stream(ctx);
    if (ctx->scratch) {
      cudaError_t e = cudaFreeAsync(ctx->scratch, st);
      if (e != cudaSuccess) return cuda_fail(e, "scratch free");
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
    }
    const size_t want = (bytes + (1u << 20) - 1) & ~static_cast<size_t>((1u << 20) - 1);
    cudaError_t e = cudaMallocAsync(&ctx->scratch, want, st);
    if (e != cudaSuccess) return cuda_fail(e, "scratch alloc");
    ctx->scratch_bytes = want;
  }
  *out = ctx->scratch;
  return HS_OK;
}

uint64_t ctx_timeout_ns(hs_ctx* ctx) { return static_cast<uint64_t>(ctx->wait_timeout_ms) * 1000000ull; }

ProfScope::ProfScope(hs_ctx* c, cudaStream_t s, const char* n) : ctx(c), st(s), name(n) {
  if (!ctx || !ctx->prof_on) return;
  for (cudaEvent_t* e : {&e0, &e1}) {
    if (!ctx->prof_free.empty()) {
      *e = ctx->prof_free.back();
      ctx->prof_free.pop_back();
    } else if (cudaEventCreate(e) != cudaSuccess) {
      *e = nullptr;
    }
  }
  if (e0) cudaEventRecord(e0, st);
}

ProfScope::~ProfScope() {
  if (!e0 || !e1) return;
  cudaEventRecord(e1, st);
  ctx->prof.push_back(hs_prof_rec{name, e0, e1});
}

// Shared validation + dispatch of the attention family.
// `merged`: q, k, v are (S*T, H*D) projection outputs and out is the
// (S*T, H*D) merged attention output; otherwise all four are (S, H, T, D).
hs_status attention_impl(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S, uint32_t H,
                         uint32_t T, uint32_t D, hs_dtype dtype, float scale, const QkPrologue& qp,
                         const QkPrologue& kp, const char* name, bool merged = false) {
  if (!ctx) return fail(HS_ERR_INVALID, std::string(name) + ": null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, std::string(name) + ": unknown dtype");
  const uint64_t n = static_cast<uint64_t>(S) * H * T * D;
  if (n == 0) return HS_OK;
  if (!q || !k || !v || !out) return fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
  if (D != 64 && D != 128)
    return fail(HS_ERR_UNSUPPORTED,
                std::string(name) + ": head_dim " + std::to_string(D) + " unsupported (this build implements 64, 128)");
  if (static_cast<uint64_t>(S) * H > 65535u)
    return fail(HS_ERR_INVALID, std::string(name) + ": S*H > 65535 (attention grid y overflow)");
  if (T > (1u << 30)) return fail(HS_ERR_INVALID, std::string(name) + ": T too large");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(HS_ERR_INVALID, std::string(name) + ": tensor pointers must be 16-byte aligned");
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));
  if (D == 128) {
    // The camera head's variant (ops.rs:236): no QK-norm or RoPE in its blocks.
    if (qp.ln || qp.rope || kp.ln || kp.rope)
      return fail(HS_ERR_UNSUPPORTED, std::string(name) + ": QK-norm/RoPE prologue needs head_dim 64");
    DeviceGuard guard(ctx->device);
    cudaStream_t st = ctx_stream(ctx);
    const RowLayout l128 = merged ? RowLayout{static_cast<uint64_t>(H) * 128, 128, static_cast<uint64_t>(T) * H * 128}
                                  : RowLayout{128, static_cast<uint64_t>(T) * 128, static_cast<uint64_t>(H) * T * 128};
    AttnIO io;
    io.q = q;
    io.lq = l128;
    io.k = k;
    io.lk = l128;
    io.v = v;
    io.lv = l128;
    io.out = out;
    io.lo = l128;
    io.out_code = static_cast<int>(dtype);
    cudaError_t e;
    {
      ProfScope prof(ctx, st, "attention_d128");
      e = launch_attention_d128(st, static_cast<int>(dtype), io, S, H, T, scale);
    }
    return e == cudaSuccess ? HS_OK : cuda_fail(e, name);
  }

  DeviceGuard guard(ctx->device);
  cudaStream_t st = ctx_stream(ctx);
  const int code = static_cast<int>(dtype);
  const int elem = dtype == HS_F16 ? kF16 : kBF16;  // tensor-core operand type (f32 -> bf16)
  const uint64_t rows = static_cast<uint64_t>(S) * H * T;
  const size_t tile_bytes = rows * 64 * 2;
  // Rows the attention kernel cannot take as given (f32 storage, or q/k that
  // need the QK-norm/RoPE prologue) go through qk_prep into scratch first.
  const bool q_direct = code != kF32 && !qp.ln && !qp.rope;
  const bool k_direct = code != kF32 && !kp.ln && !kp.rope;
  const bool v_direct = code != kF32;
  const size_t need = (q_direct ? 0 : tile_bytes) + (k_direct ? 0 : tile_bytes) + (v_direct ? 0 : tile_bytes);
  void* scratch = nullptr;
  if (need) {
    hs_status s = ctx_scratch(ctx, need, &scratch);
    if (s != HS_OK) return s;
  }
  const RowLayout head_major = RowLayout::head_major(H, T);
  const RowLayout given = merged ? RowLayout::token_major(H, T, static_cast<uint64_t>(H) * 64) : head_major;
  const void* use[3] = {q, k, v};
  RowLayout lay[3] = {given, given, given};
  const bool direct[3] = {q_direct, k_direct, v_direct};
  // When both q and k pass through qk_prep it also records their largest
  // row norms, which let the attention kernel bound every score.
  unsigned int* norm2 = (!q_direct && !k_direct) ? ctx->d_norm2 : nullptr;
  QkPrologue qpn = qp, kpn = kp;
  qpn.norm2_max = norm2;
  kpn.norm2_max = norm2 ? norm2 + 1 : nullptr;
  const QkPrologue none{};
  const QkPrologue* pro[3] = {&qpn, &kpn, &none};
  // Every tensor that needs a pass goes through one qk_prep launch.
  PrepJob jobs[3];
  int n_jobs = 0;
  uint8_t* cursor = static_cast<uint8_t*>(scratch);
  for (int i = 0; i < 3; ++i) {
    if (direct[i]) continue;
    jobs[n_jobs++] = PrepJob{use[i], given, cursor, *pro[i]};
    use[i] = cursor;
    lay[i] = head_major;
    cursor += tile_bytes;
  }
  cudaError_t e = cudaSuccess;
  if (n_jobs) {
    {
      ProfScope prof(ctx, st, "qk_prep");
      e = launch_qk_prep(st, code, elem, S, H, T, jobs, n_jobs, ctx->d_status, ctx_timeout_ns(ctx));
    }
    if (e != cudaSuccess) return cuda_fail(e, "qk_prep");
  }
  std::string err;
  AttnState state{};
  {
    ProfScope prof(ctx, st, "attention");
    AttnIO io;
    io.q = use[0];
    io.lq = lay[0];
    io.k = use[1];
    io.lk = lay[1];
    io.v = use[2];
    io.lv = lay[2];
    io.out = out;
    io.lo = given;
    io.out_code = code == kF32 ? kF32 : elem;
    e = launch_attention_sm100(st, elem, io, S, H, T, T, scale, state, 0, ctx->d_status, ctx->d_sched, norm2, false,
                               ctx_timeout_ns(ctx), &err);
  }
  if (e != cudaSuccess) return fail(HS_ERR_CUDA, std::string(name) + ": " + (err.empty() ? cudaGetErrorString(e) : err));
  return HS_OK;
}

}  // namespace hs

namespace hs {
// QK-norm + RoPE arguments of the fused entry points, validated.
hs_status fused_prologues(const char* name, uint32_t T, const float* q_norm_w, const float* q_norm_b,
                          const float* k_norm_w, const float* k_norm_b, float eps, const float* rope_sin,
                          const float* rope_cos, uint32_t rope_rows, uint32_t prefix, uint32_t tokens_per_frame,
                          QkPrologue* qp, QkPrologue* kp) {
  const bool ln = q_norm_w != nullptr;
  if (ln != (k_norm_w != nullptr) || (ln && (!q_norm_b || !k_norm_b)))
    return fail(HS_ERR_INVALID, std::string(name) + ": QK-norm needs all of q/k weight and bias, or none");
  const bool rope = rope_sin != nullptr;
  if (rope && !rope_cos) return fail(HS_ERR_INVALID, std::string(name) + ": rope_cos missing");
  const uint32_t tpf = tokens_per_frame ? tokens_per_frame : T;
  if (rope) {
    if (prefix > tpf) return fail(HS_ERR_INVALID, std::string(name) + ": prefix > tokens_per_frame");
    if (static_cast<uint64_t>(rope_rows) < static_cast<uint64_t>(tpf - prefix))
      return fail(HS_ERR_INVALID, std::string(name) + ": rope tables have " + std::to_string(rope_rows) +
                                      " rows, need tokens_per_frame - prefix = " + std::to_string(tpf - prefix));
    if (!aligned16(rope_sin) || !aligned16(rope_cos))
      return fail(HS_ERR_INVALID, std::string(name) + ": rope tables must be 16-byte aligned");
  }
  *qp = QkPrologue{};
  qp->ln = ln;
  qp->ln_w = q_norm_w;
  qp->ln_b = q_norm_b;
  qp->eps = eps;
  qp->rope = rope;
  qp->sin_t = rope_sin;
  qp->cos_t = rope_cos;
  qp->prefix = prefix;
  qp->tokens_per_frame = tpf;
  *kp = *qp;
  kp->ln_w = k_norm_w;
  kp->ln_b = k_norm_b;
  return HS_OK;
}
}  // namespace hs

using namespace hs;

extern "C" {

uint32_t hs_abi_version(void) { return HS_ABI_VERSION; }

const char* hs_last_error(void) { return g_last_error.c_str(); }

hs_status hs_ctx_create(int device, hs_ctx** out) {
  if (!out) return fail(HS_ERR_INVALID, "hs_ctx_create: null out");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "hs_ctx_create: cudaGetDeviceCount");
  if (device < 0 || device >= count) return fail(HS_ERR_INVALID, "hs_ctx_create: no such device");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "hs_ctx_create: properties");
  if (prop.major != 10 || prop.minor != 0)
    return fail(HS_ERR_UNSUPPORTED, "hs_ctx_create: device is sm_" + std::to_string(prop.major) +
                                        std::to_string(prop.minor) + ", this library is built for sm_100a (B200)");
  DeviceGuard guard(device);
  hs_ctx* ctx = new hs_ctx();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "hs_ctx_create: stream");
  }
  // [0] status word, [2..3] attention work counter, [4..5] q'/k' norm bounds.
  e = cudaMalloc(&ctx->d_status, sizeof(int) * 8);
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(int) * 8);
  ctx->d_sched = reinterpret_cast<uint32_t*>(ctx->d_status + 2);
  ctx->d_norm2 = reinterpret_cast<unsigned int*>(ctx->d_status + 4);
  if (e != cudaSuccess) {
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return cuda_fail(e, "hs_ctx_create: status word");
  }
  *out = ctx;
  return HS_OK;
}

hs_status hs_ctx_destroy(hs_ctx* ctx) {
  if (!ctx) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaStream_t st = ctx_stream(ctx);
  if (ctx->scratch) cudaFreeAsync(ctx->scratch, st);
  cudaStreamSynchronize(st);
  for (auto& r : ctx->prof) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  for (cudaEvent_t e : ctx->prof_free) cudaEventDestroy(e);
  cudaFree(ctx->d_status);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return HS_OK;
}

hs_status hs_ctx_set_stream(hs_ctx* ctx, void* stream) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_ctx_set_stream: null context");
  ctx->user_stream = static_cast<cudaStream_t>(stream);
  ctx->has_user_stream = true;
  return HS_OK;
}

hs_status hs_ctx_use_own_stream(hs_ctx* ctx) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_ctx_use_own_stream: null context");
  ctx->has_user_stream = false;
  ctx->user_stream = nullptr;
  return HS_OK;
}

void* hs_ctx_stream(hs_ctx* ctx) { return ctx ? static_cast<void*>(ctx_stream(ctx)) : nullptr; }

hs_status hs_ctx_set_wait_timeout_ms(hs_ctx* ctx, uint32_t ms) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_ctx_set_wait_timeout_ms: null context");
  ctx->wait_timeout_ms = ms;  // 0: kernels do not wait (see the header)
  return HS_OK;
}

hs_status hs_ctx_request_cancel(hs_ctx* ctx) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_ctx_request_cancel: null context");
  ctx->cancel.store(1);
  return HS_OK;
}

hs_status hs_ctx_clear_cancel(hs_ctx* ctx) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_ctx_clear_cancel: null context");
  ctx->cancel.store(0);
  return HS_OK;
}

hs_status hs_prof_enable(hs_ctx* ctx, int on) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_prof_enable: null context");
  ctx->prof_on = on != 0;
  return HS_OK;
}

hs_status hs_prof_reset(hs_ctx* ctx) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_prof_reset: null context");
  DeviceGuard guard(ctx->device);
  cudaStreamSynchronize(ctx_stream(ctx));
  for (auto& r : ctx->prof) {
    ctx->prof_free.push_back(r.start);
    ctx->prof_free.push_back(r.stop);
  }
  ctx->prof.clear();
  return HS_OK;
}

hs_status hs_prof_read(hs_ctx* ctx, const char* kernel, double* total_ms, uint64_t* launches) {
  if (!ctx || !kernel || !total_ms || !launches) return fail(HS_ERR_INVALID, "hs_prof_read: null argument");
  DeviceGuard guard(ctx->device);
  double ms = 0.0;
  uint64_t n = 0;
  const bool all = strcmp(kernel, "*") == 0;
  for (auto& r : ctx->prof) {
    if (!all && r.kernel != kernel) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "hs_prof_read");
    float one = 0.f;
    e = cudaEventElapsedTime(&one, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "hs_prof_read");
    ms += one;
    ++n;
  }
  *total_ms = ms;
  *launches = n;
  return HS_OK;
}

hs_status hs_alloc(hs_ctx* ctx, size_t bytes, void** out) {
  if (!ctx || !out) return fail(HS_ERR_INVALID, "hs_alloc: null argument");
  *out = nullptr;
  if (bytes == 0) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMallocAsync(out, bytes, ctx_stream(ctx));
  if (e != cudaSuccess) return cuda_fail(e, "hs_alloc");
  return HS_OK;
}

hs_status hs_free(hs_ctx* ctx, void* ptr) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_free: null context");
  if (!ptr) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaFreeAsync(ptr, ctx_stream(ctx));
  if (e != cudaSuccess) return cuda_fail(e, "hs_free");
  return HS_OK;
}

hs_status hs_memset(hs_ctx* ctx, void* dst, int value, size_t bytes) {
  if (!ctx || (!dst && bytes)) return fail(HS_ERR_INVALID, "hs_memset: null argument");
  if (!bytes) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMemsetAsync(dst, value, bytes, ctx_stream(ctx));
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_memset");
}

hs_status hs_memcpy_h2d(hs_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || ((!dst || !src) && bytes)) return fail(HS_ERR_INVALID, "hs_memcpy_h2d: null argument");
  if (!bytes) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx_stream(ctx));
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_memcpy_h2d");
}

hs_status hs_memcpy_d2h(hs_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || ((!dst || !src) && bytes)) return fail(HS_ERR_INVALID, "hs_memcpy_d2h: null argument");
  if (!bytes) return HS_OK;
  DeviceGuard guard(ctx->device);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx_stream(ctx));
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_memcpy_d2h");
}

hs_status hs_sync(hs_ctx* ctx) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_sync: null context");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = ctx_stream(ctx);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "hs_sync");
  int status = 0;
  e = cudaMemcpy(&status, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "hs_sync: status word");
  if (status != 0) {
    cudaMemset(ctx->d_status, 0, sizeof(int));
    char buf[128];
    snprintf(buf, sizeof buf, "hs_sync: a kernel's bounded wait timed out (site 0x%x)", status);
    return fail(HS_ERR_TIMEOUT, buf);
  }
  return HS_OK;
}

hs_status hs_attention(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S, uint32_t H,
                       uint32_t T, uint32_t D, hs_dtype dtype, float scale) {
  QkPrologue none{};
  return attention_impl(ctx, q, k, v, out, S, H, T, D, dtype, scale, none, none, "hs_attention");
}

hs_status hs_attention_fused(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S,
                             uint32_t H, uint32_t T, uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                             const float* q_norm_b, const float* k_norm_w, const float* k_norm_b, float eps,
                             const float* rope_sin, const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                             uint32_t tokens_per_frame) {
  const char* name = "hs_attention_fused";
  QkPrologue qp, kp;
  hs_status r = fused_prologues(name, T, q_norm_w, q_norm_b, k_norm_w, k_norm_b, eps, rope_sin, rope_cos, rope_rows,
                                prefix, tokens_per_frame, &qp, &kp);
  if (r != HS_OK) return r;
  return attention_impl(ctx, q, k, v, out, S, H, T, D, dtype, scale, qp, kp, name);
}

hs_status hs_linear(hs_ctx* ctx, const void* x, const void* w, const float* bias, void* out, uint64_t M, uint32_t K,
                    uint32_t N, hs_dtype dtype, int epilogue, const void* residual, const float* gamma) {
  const char* name = "hs_linear";
  if (!ctx) return fail(HS_ERR_INVALID, std::string(name) + ": null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, std::string(name) + ": unknown dtype");
  if (M == 0 || N == 0) return HS_OK;
  if (dtype == HS_F32) {  // the reference's f32 linear: f32 arithmetic, any shape
    if (K == 0) return fail(HS_ERR_INVALID, std::string(name) + ": K must be non-zero");
    if (epilogue < HS_LINEAR_PLAIN || epilogue > HS_LINEAR_RESIDUAL_LS)
      return fail(HS_ERR_INVALID, std::string(name) + ": unknown epilogue");
    if (!x || !w || !out) return fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
    if (epilogue == HS_LINEAR_RESIDUAL_LS && (!residual || !gamma))
      return fail(HS_ERR_INVALID, std::string(name) + ": the residual epilogue needs residual and gamma");
    if ((M + 127) / 128 > 65535u) return fail(HS_ERR_INVALID, std::string(name) + ": M > 65535 * 128 for f32");
    DeviceGuard guard(ctx->device);
    cudaStream_t st = ctx_stream(ctx);
    cudaError_t e;
    {
      ProfScope prof(ctx, st, "linear");
      e = launch_linear_f32(st, static_cast<const float*>(x), static_cast<const float*>(w), bias,
                            static_cast<float*>(out), M, K, N, epilogue, static_cast<const float*>(residual), gamma);
    }
    return e == cudaSuccess ? HS_OK : cuda_fail(e, name);
  }
  if (K == 0 || K % 8 || N % 8)
    return fail(HS_ERR_UNSUPPORTED, std::string(name) + ": K and N must be non-zero multiples of 8 (16-byte rows)");
  if (epilogue < HS_LINEAR_PLAIN || epilogue > HS_LINEAR_RESIDUAL_LS)
    return fail(HS_ERR_INVALID, std::string(name) + ": unknown epilogue");
  if (!x || !w || !out) return fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
  if (epilogue == HS_LINEAR_RESIDUAL_LS && (!residual || !gamma))
    return fail(HS_ERR_INVALID, std::string(name) + ": the residual epilogue needs residual and gamma");
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || (residual && !aligned16(residual)) ||
      (bias && !aligned16(bias)) || (gamma && !aligned16(gamma)))
    return fail(HS_ERR_INVALID, std::string(name) + ": tensor and bias/gamma pointers must be 16-byte aligned");
  DeviceGuard guard(ctx->device);
  cudaStream_t st = ctx_stream(ctx);
  const int elem = dtype == HS_F16 ? kF16 : kBF16;
  std::string err;
  cudaError_t e;
  {
    ProfScope prof(ctx, st, "linear");
    e = launch_linear_sm100(st, elem, x, w, bias, out, M, K, N, epilogue, residual, gamma, ctx->d_status,
                            ctx_timeout_ns(ctx), &err);
  }
  if (e != cudaSuccess) return fail(HS_ERR_CUDA, std::string(name) + ": " + (err.empty() ? cudaGetErrorString(e) : err));
  return HS_OK;
}

hs_status hs_attention_block_fused(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S,
                                   uint32_t T, uint32_t H, uint32_t D, hs_dtype dtype, float scale,
                                   const float* q_norm_w, const float* q_norm_b, const float* k_norm_w,
                                   const float* k_norm_b, float eps, const float* rope_sin, const float* rope_cos,
                                   uint32_t rope_rows, uint32_t prefix, uint32_t tokens_per_frame) {
  const char* name = "hs_attention_block_fused";
  QkPrologue qp, kp;
  hs_status r = fused_prologues(name, T, q_norm_w, q_norm_b, k_norm_w, k_norm_b, eps, rope_sin, rope_cos, rope_rows,
                                prefix, tokens_per_frame, &qp, &kp);
  if (r != HS_OK) return r;
  return attention_impl(ctx, q, k, v, out, S, H, T, D, dtype, scale, qp, kp, name, true);
}

hs_status hs_layernorm(hs_ctx* ctx, const void* x, const float* w, const float* b, void* out, uint64_t rows,
                       uint32_t dim, float eps, hs_dtype dtype) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_layernorm: null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, "hs_layernorm: unknown dtype");
  if (rows == 0 || dim == 0) return HS_OK;
  if (!x || !w || !b || !out) return fail(HS_ERR_INVALID, "hs_layernorm: null pointer");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "layernorm");
  cudaError_t e = launch_layernorm(ctx_stream(ctx), x, out, static_cast<int>(dtype), w, b, rows, dim, eps);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_layernorm");
}

hs_status hs_rope_apply(hs_ctx* ctx, void* x, const float* rope_sin, const float* rope_cos, uint32_t rope_rows,
                        uint32_t S, uint32_t H, uint32_t T, uint32_t D, uint32_t prefix, hs_dtype dtype) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_rope_apply: null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, "hs_rope_apply: unknown dtype");
  if (D == 0 || (D & 1)) return fail(HS_ERR_INVALID, "hs_rope_apply: D must be even");
  if (prefix > T) return fail(HS_ERR_INVALID, "hs_rope_apply: prefix > T");
  if (rope_rows != T - prefix)
    return fail(HS_ERR_INVALID, "hs_rope_apply: table size: rows " + std::to_string(rope_rows) +
                                    " != T - prefix = " + std::to_string(T - prefix));
  if (static_cast<uint64_t>(S) * H * T == 0) return HS_OK;
  if (!x || !rope_sin || !rope_cos) return fail(HS_ERR_INVALID, "hs_rope_apply: null pointer");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "rope_apply");
  cudaError_t e = launch_rope_apply(ctx_stream(ctx), x, static_cast<int>(dtype), rope_sin, rope_cos, S, H, T, D, prefix, T);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_rope_apply");
}

hs_status hs_split_heads(hs_ctx* ctx, const void* x, void* out, uint32_t S, uint32_t T, uint32_t H, uint32_t D,
                         hs_dtype dtype) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_split_heads: null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, "hs_split_heads: unknown dtype");
  if (static_cast<uint64_t>(S) * H * T * D == 0) return HS_OK;
  if (!x || !out) return fail(HS_ERR_INVALID, "hs_split_heads: null pointer");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "permute");
  cudaError_t e = launch_split_heads(ctx_stream(ctx), x, out, static_cast<int>(dtype), S, T, H, D);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_split_heads");
}

hs_status hs_attn_merge(hs_ctx* ctx, const void* x, void* out, uint32_t S, uint32_t H, uint32_t T, uint32_t D,
                        hs_dtype dtype) {
  if (!ctx) return fail(HS_ERR_INVALID, "hs_attn_merge: null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, "hs_attn_merge: unknown dtype");
  if (static_cast<uint64_t>(S) * H * T * D == 0) return HS_OK;
  if (!x || !out) return fail(HS_ERR_INVALID, "hs_attn_merge: null pointer");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "permute");
  cudaError_t e = launch_attn_merge(ctx_stream(ctx), x, out, static_cast<int>(dtype), S, H, T, D);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, "hs_attn_merge");
}

hs_status hs_copy_row_blocks(hs_ctx* ctx, const void* src, void* dst, uint64_t groups, uint64_t src_stride_rows,
                             uint64_t dst_stride_rows, uint64_t rows, uint32_t cols, hs_dtype dtype) {
  const char* name = "hs_copy_row_blocks";
  if (!ctx) return fail(HS_ERR_INVALID, std::string(name) + ": null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, std::string(name) + ": unknown dtype");
  if (groups == 0 || rows == 0 || cols == 0) return HS_OK;
  if (!src || !dst) return fail(HS_ERR_INVALID, std::string(name) + ": null pointer");
  const uint64_t row_bytes = static_cast<uint64_t>(cols) * (dtype == HS_F32 ? 4 : 2);
  if (row_bytes % 16 || !aligned16(src) || !aligned16(dst))
    return fail(HS_ERR_INVALID, std::string(name) + ": rows must be 16-byte multiples, pointers 16-byte aligned");
  if (groups > 1 && ((src_stride_rows != 0 && src_stride_rows < rows) || dst_stride_rows < rows))
    return fail(HS_ERR_INVALID, std::string(name) + ": group strides shorter than the rows copied");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "copy_rows");
  cudaError_t e = launch_copy_row_blocks(ctx_stream(ctx), src, dst, groups, src_stride_rows, dst_stride_rows, rows,
                                         row_bytes);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, name);
}

hs_status hs_im2col_patch(hs_ctx* ctx, const float* images, void* out, uint32_t n, uint32_t height, uint32_t width,
                          uint32_t patch, uint32_t row_stride, const float* mean, const float* std_dev,
                          hs_dtype dtype) {
  const char* name = "hs_im2col_patch";
  if (!ctx) return fail(HS_ERR_INVALID, std::string(name) + ": null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, std::string(name) + ": unknown dtype");
  if (patch == 0 || height % patch || width % patch)
    return fail(HS_ERR_INVALID, std::string(name) + ": image sides must be multiples of the patch size");
  if (row_stride < 3 * patch * patch)
    return fail(HS_ERR_INVALID, std::string(name) + ": row_stride < 3 * patch * patch");
  if (static_cast<uint64_t>(n) * height * width == 0) return HS_OK;
  if (!images || !out) return fail(HS_ERR_INVALID, std::string(name) + ": null pointer");
  // ImageNet statistics (headshot-shared model.rs IMAGENET_MEAN / IMAGENET_STD) when not given.
  const float m[3] = {mean ? mean[0] : 0.485f, mean ? mean[1] : 0.456f, mean ? mean[2] : 0.406f};
  const float sd[3] = {std_dev ? std_dev[0] : 0.229f, std_dev ? std_dev[1] : 0.224f, std_dev ? std_dev[2] : 0.225f};
  if (!(sd[0] > 0.f) || !(sd[1] > 0.f) || !(sd[2] > 0.f))
    return fail(HS_ERR_INVALID, std::string(name) + ": std must be positive");
  const float inv[3] = {1.0f / sd[0], 1.0f / sd[1], 1.0f / sd[2]};
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "im2col_patch");
  cudaError_t e = launch_im2col_patch(ctx_stream(ctx), images, out, static_cast<int>(dtype), n, height, width, patch,
                                      row_stride, m, inv);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, name);
}

hs_status hs_cache_build(hs_ctx* ctx, const void* frame_out, const void* global_out, float* out, uint64_t rows,
                         uint32_t cols_frame, uint32_t cols_global, hs_dtype dtype) {
  const char* name = "hs_cache_build";
  if (!ctx) return fail(HS_ERR_INVALID, std::string(name) + ": null context");
  if (!valid_dtype(dtype)) return fail(HS_ERR_INVALID, std::string(name) + ": unknown dtype");
  if (rows == 0) return HS_OK;
  if (!frame_out || !global_out || !out) return fail(HS_ERR_INVALID, std::string(name) + ": null pointer");
  if (cols_frame % 8 || cols_global % 8 || !aligned16(frame_out) || !aligned16(global_out) || !aligned16(out))
    return fail(HS_ERR_INVALID, std::string(name) + ": widths must be multiples of 8, pointers 16-byte aligned");
  DeviceGuard guard(ctx->device);
  ProfScope prof(ctx, ctx_stream(ctx), "cache_build");
  cudaError_t e = launch_cache_build(ctx_stream(ctx), frame_out, global_out, out, static_cast<int>(dtype), rows,
                                     cols_frame, cols_global);
  return e == cudaSuccess ? HS_OK : cuda_fail(e, name);
}

hs_status hs_rope_periods(float* out16) {
  if (!out16) return fail(HS_ERR_INVALID, "hs_rope_periods: null out");
  for (int i = 0; i < 16; ++i) out16[i] = powf(100.0f, 2.0f * static_cast<float>(i) / 32.0f);
  return HS_OK;
}

hs_status hs_rope_tables(const float* periods, uint32_t h_p, uint32_t w_p, float* sin_out, float* cos_out) {
  if (!sin_out || !cos_out) return fail(HS_ERR_INVALID, "hs_rope_tables: null out");
  float local[16];
  if (!periods) {
    hs_rope_periods(local);
    periods = local;
  }
  const float side = static_cast<float>(h_p > w_p ? h_p : w_p);
  const float tau = 6.28318530717958647692f;
  for (uint32_t row = 0; row < h_p; ++row) {
    for (uint32_t col = 0; col < w_p; ++col) {
      const size_t idx = (static_cast<size_t>(row) * w_p + col) * 64;
      const float ch = 2.0f * ((static_cast<float>(row) + 0.5f) / side) - 1.0f;
      const float cw = 2.0f * ((static_cast<float>(col) + 0.5f) / side) - 1.0f;
      for (int i = 0; i < 16; ++i) {
        const float ah = tau * ch / periods[i];
        const float aw = tau * cw / periods[i];
        const float sh = sinf(ah), chh = cosf(ah), sw = sinf(aw), cww = cosf(aw);
        for (int half = 0; half <= 32; half += 32) {
          sin_out[idx + half + i] = sh;
          cos_out[idx + half + i] = chh;
          sin_out[idx + half + 16 + i] = sw;
          cos_out[idx + half + 16 + i] = cww;
        }
      }
    }
  }
  return HS_OK;
}

}  // extern "C"
