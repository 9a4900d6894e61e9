// ring.cu — sequence-parallel (ring) global attention across GPUs.
//
// The reference runs global attention as one streaming kernel over N·T
// tokens on one device (src/model/trunk.rs:124-125); this is the new
// multi-GPU session layer.  Each rank owns a contiguous shard of the
// sequence (all heads): q, k, v, out are (H, T_r, 64) with T_r from
// hs_ring_shard.  K' = RoPE(LN(K)) is computed once per shard by its owner,
// then [K' | V] blocks travel around the ring with NCCL send/recv on a
// communication stream while the tcgen05 kernel processes the block that
// arrived in the previous step.  The running softmax state (unnormalised O,
// max m, sum l — f32) stays on the rank and is carried from step to step by
// the kernel itself; the last step writes the normalised output.
//
// NCCL is resolved at run time (dlopen "libnccl.so.2"), so the library loads
// and the single-GPU ops work without it.
#include <dlfcn.h>
#include <math.h>
#include <nccl.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>

#include "../../include/headshot_cuda.h"
#include "hs_abi_ctx.h"
#include "hs_internal.h"

namespace {

struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    bool ok = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) ok = false;
    };
    sym(api.GetUniqueId, "ncclGetUniqueId");
    sym(api.CommInitRank, "ncclCommInitRank");
    sym(api.CommDestroy, "ncclCommDestroy");
    sym(api.CommAbort, "ncclCommAbort");
    sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(api.Send, "ncclSend");
    sym(api.Recv, "ncclRecv");
    sym(api.AllReduce, "ncclAllReduce");
    sym(api.GroupStart, "ncclGroupStart");
    sym(api.GroupEnd, "ncclGroupEnd");
    sym(api.GetErrorString, "ncclGetErrorString");
    if (!ok) {
      api.error = "libnccl.so.2 lacks a required symbol";
      return;
    }
    api.loaded = true;
  });
  return api;
}

hs_status nccl_fail(ncclResult_t r, const char* what) {
  NcclApi& n = nccl();
  return hs::abi_fail(HS_ERR_NCCL, std::string(what) + ": " + (n.GetErrorString ? n.GetErrorString(r) : "nccl error"));
}

void shard(uint32_t n, int world, int rank, uint32_t* start, uint32_t* len) {
  const uint32_t base = n / static_cast<uint32_t>(world);
  const uint32_t rem = n % static_cast<uint32_t>(world);
  const uint32_t r = static_cast<uint32_t>(rank);
  *start = r * base + (r < rem ? r : rem);
  *len = base + (r < rem ? 1u : 0u);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Default SMs left to the block transfers: none.  Measured on B200s at
// 274,800 tokens: 2 ranks 1697 TFLOP/s with 0 SMs left free against 1682 /
// 1668 / 1645 with 2 / 4 / 8; 8 ranks 6582 with 0 against 6376 with 4.
uint32_t default_reserved_sms(int) { return 0u; }

}  // namespace

struct hs_ring {
  hs_ctx* ctx = nullptr;
  int rank = 0;
  int world = 1;
  ncclComm_t comm = nullptr;
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ev_block0 = nullptr;
  cudaEvent_t ev_recv[2] = {nullptr, nullptr};
  cudaEvent_t ev_compute[2] = {nullptr, nullptr};
  cudaEvent_t ev_done = nullptr;
  cudaEvent_t ev_bound = nullptr;  // the all-ranks score bound is ready
  // Largest squared q' and k' row norms over all ranks (f32 bit patterns):
  // one bound on every score of every ring step.
  unsigned int* norm2 = nullptr;
  void* buf[2] = {nullptr, nullptr};
  size_t buf_bytes = 0;
  // Per query row of this rank's shard: the normalised/rotated q (64 x 16-bit),
  // then the carried softmax state o (64 f32) | m (f32) | l (f32).
  uint8_t* state = nullptr;
  size_t state_rows = 0;
  bool aborted = false;
  // SMs the attention kernel leaves free during ring steps.  The kernel is
  // persistent and takes a whole SM per CTA (shared memory and registers), so
  // without free SMs NCCL's send/recv kernel for the next block waits for the
  // attention launch to end and every transfer adds to the step.  Freeing SMs
  // costs attention throughput in proportion; it pays when the transfers are
  // large next to the launches (many ranks, short shards).
  uint32_t reserved_sms = 0;
  // Head-parallel path (hs_ring_ulysses_attention_fused): this rank's Q' and
  // K' shards, then Q', K', V and the output of its H / R heads over the whole
  // sequence; events ordering the two all-to-alls against the attention.
  uint8_t* uly = nullptr;
  size_t uly_bytes = 0;
  cudaEvent_t ev_in = nullptr;   // the inbound all-to-all landed
  cudaEvent_t ev_attn = nullptr; // the attention over the gathered heads is done
};

extern "C" {

hs_status hs_ring_shard(uint32_t n, int world, int rank, uint32_t* start, uint32_t* len) {
  if (world < 1 || rank < 0 || rank >= world || !start || !len)
    return hs::abi_fail(HS_ERR_INVALID, "hs_ring_shard: bad arguments");
  shard(n, world, rank, start, len);
  return HS_OK;
}

hs_status hs_ring_plan(int rank, int world, int step, int* src_block, int* send_to, int* recv_from,
                       int* load_state, int* store_state) {
  if (world < 1 || rank < 0 || rank >= world || step < 0 || step >= world)
    return hs::abi_fail(HS_ERR_INVALID, "hs_ring_plan: bad arguments");
  if (src_block) *src_block = (rank - step + world) % world;
  const bool last = step == world - 1;
  if (send_to) *send_to = last ? -1 : (rank + 1) % world;
  if (recv_from) *recv_from = last ? -1 : (rank - 1 + world) % world;
  if (load_state) *load_state = step > 0 ? 1 : 0;
  if (store_state) *store_state = last ? 0 : 1;
  return HS_OK;
}

size_t hs_ring_id_bytes(void) { return NCCL_UNIQUE_ID_BYTES; }

hs_status hs_ring_unique_id(void* id_out) {
  if (!id_out) return hs::abi_fail(HS_ERR_INVALID, "hs_ring_unique_id: null out");
  NcclApi& n = nccl();
  if (!n.loaded) return hs::abi_fail(HS_ERR_NCCL, n.error);
  ncclUniqueId id;
  ncclResult_t r = n.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof id);
  return HS_OK;
}

hs_status hs_ring_create(hs_ctx* ctx, int rank, int world, const void* id, hs_ring** out) {
  if (!ctx || !id || !out || world < 1 || rank < 0 || rank >= world)
    return hs::abi_fail(HS_ERR_INVALID, "hs_ring_create: bad arguments");
  *out = nullptr;
  NcclApi& n = nccl();
  if (!n.loaded) return hs::abi_fail(HS_ERR_NCCL, n.error);
  cudaSetDevice(ctx->device);
  hs_ring* ring = new hs_ring();
  ring->ctx = ctx;
  ring->rank = rank;
  ring->world = world;
  ring->reserved_sms = default_reserved_sms(world);
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclResult_t r = n.CommInitRank(&ring->comm, world, uid, rank);
  if (r != ncclSuccess) {
    delete ring;
    return nccl_fail(r, "ncclCommInitRank");
  }
  cudaError_t e = cudaStreamCreateWithFlags(&ring->comm_stream, cudaStreamNonBlocking);
  for (cudaEvent_t* ev : {&ring->ev_block0, &ring->ev_recv[0], &ring->ev_recv[1], &ring->ev_compute[0],
                          &ring->ev_compute[1], &ring->ev_done, &ring->ev_bound, &ring->ev_in, &ring->ev_attn})
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMalloc(&ring->norm2, 2 * sizeof(unsigned int));
  if (e != cudaSuccess) {
    n.CommDestroy(ring->comm);
    delete ring;
    return hs::abi_cuda_fail(e, "hs_ring_create");
  }
  *out = ring;
  return HS_OK;
}

hs_status hs_ring_set_reserved_sms(hs_ring* ring, uint32_t sms) {
  if (!ring) return hs::abi_fail(HS_ERR_INVALID, "hs_ring_set_reserved_sms: null ring");
  if (sms + 1 > static_cast<uint32_t>(ring->ctx->sm_count))
    return hs::abi_fail(HS_ERR_INVALID, "hs_ring_set_reserved_sms: must leave at least one SM for attention");
  ring->reserved_sms = sms;
  return HS_OK;
}

hs_status hs_ring_destroy(hs_ring* ring) {
  if (!ring) return HS_OK;
  NcclApi& n = nccl();
  cudaSetDevice(ring->ctx->device);
  if (!ring->aborted) {
    cudaStreamSynchronize(ring->comm_stream);
    cudaStreamSynchronize(hs::ctx_stream(ring->ctx));
  }
  if (ring->comm) {
    if (ring->aborted)
      n.CommAbort(ring->comm);
    else
      n.CommDestroy(ring->comm);
  }
  for (void* b : ring->buf)
    if (b) cudaFree(b);
  if (ring->state) cudaFree(ring->state);
  if (ring->uly) cudaFree(ring->uly);
  if (ring->norm2) cudaFree(ring->norm2);
  for (cudaEvent_t ev : {ring->ev_block0, ring->ev_recv[0], ring->ev_recv[1], ring->ev_compute[0],
                         ring->ev_compute[1], ring->ev_done, ring->ev_bound, ring->ev_in, ring->ev_attn})
    if (ev) cudaEventDestroy(ev);
  if (ring->comm_stream) cudaStreamDestroy(ring->comm_stream);
  delete ring;
  return HS_OK;
}

}  // extern "C"

namespace {

// The ring attention of one rank.  `block`: q, k, v and out are this rank's
// (T_r, H*64) projection rows (Block::forward's layout) instead of (H, T_r,
// 64).  Shards are whole `unit`s of tokens (frames, for a frame-sharded
// trunk): rank r owns units shard(T_total / unit, R, r).
hs_status ring_attention(hs_ring* ring, const void* q, const void* k, const void* v, void* out, uint32_t H,
                         uint32_t T_total, uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                         const float* q_norm_b, const float* k_norm_w, const float* k_norm_b, float eps,
                         const float* rope_sin, const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                         uint32_t tokens_per_frame, bool block, uint32_t unit, const char* name) {
  if (!ring) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": null ring");
  if (ring->aborted) return hs::abi_fail(HS_ERR_NCCL, std::string(name) + ": ring was aborted");
  hs_ctx* ctx = ring->ctx;
  const int R = ring->world, r = ring->rank;
  if (ctx->cancel.load()) return hs::abi_fail(HS_ERR_CANCELLED, std::string(name) + ": cancelled");
  if (dtype != HS_F16 && dtype != HS_BF16)
    return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": ring path takes f16/bf16 storage");
  if (D != 64) return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": head_dim must be 64");
  if (unit == 0 || T_total % unit != 0)
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": T_total must be a multiple of shard_unit");
  if (H == 0 || H > 65535 || T_total / unit < static_cast<uint32_t>(R))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": need 1 <= H <= 65535 and one shard unit per rank");
  // Token range [t0, t0 + len) of rank i's shard.
  auto shard_of = [&](int i, uint32_t* t0_, uint32_t* len_) {
    shard(T_total / unit, R, i, t0_, len_);
    *t0_ *= unit;
    *len_ *= unit;
  };
  uint32_t t0, tr;
  shard_of(r, &t0, &tr);
  if (!q || !k || !v || !out) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": tensor pointers must be 16-byte aligned");
  const bool ln = q_norm_w != nullptr;
  if (ln != (k_norm_w != nullptr) || (ln && (!q_norm_b || !k_norm_b)))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": QK-norm needs all of q/k weight and bias, or none");
  const bool rope = rope_sin != nullptr;
  const uint32_t tpf = tokens_per_frame ? tokens_per_frame : T_total;
  if (rope && (!rope_cos || prefix > tpf || rope_rows < tpf - prefix || !aligned16(rope_sin) || !aligned16(rope_cos)))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": bad RoPE tables / prefix");
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));

  cudaSetDevice(ctx->device);
  NcclApi& n = nccl();
  cudaStream_t st = hs::ctx_stream(ctx);
  cudaStream_t cs = ring->comm_stream;
  const int code = static_cast<int>(dtype);
  const size_t row_bytes = 64 * 2;
  const uint32_t tmax = (T_total / unit + R - 1) / R * unit;
  const size_t need_buf = 2ull * H * tmax * row_bytes;
  cudaError_t e;
  if (ring->buf_bytes < need_buf && R > 1) {
    cudaStreamSynchronize(st);
    cudaStreamSynchronize(cs);
    for (void*& b : ring->buf) {
      if (b) cudaFree(b);
      b = nullptr;
      e = cudaMalloc(&b, need_buf);
      if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring buffers");
    }
    ring->buf_bytes = need_buf;
  }
  const size_t rows = static_cast<size_t>(H) * tr;
  if (ring->state_rows < rows && R > 1) {
    cudaStreamSynchronize(st);
    if (ring->state) cudaFree(ring->state);
    ring->state = nullptr;
    e = cudaMalloc(&ring->state, rows * (row_bytes + 66 * sizeof(float)));
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring state");
    ring->state_rows = rows;
  }

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
  qp.pos_offset = t0;
  hs::QkPrologue kp = qp;
  kp.ln_w = k_norm_w;
  kp.ln_b = k_norm_b;

  if (R == 1) {  // nothing to exchange: the single-device fused op
    if (block)
      return hs_attention_block_fused(ctx, q, k, v, out, 1, T_total, H, D, dtype, scale, q_norm_w, q_norm_b,
                                      k_norm_w, k_norm_b, eps, rope_sin, rope_cos, rope_rows, prefix,
                                      tokens_per_frame);
    return hs_attention_fused(ctx, q, k, v, out, 1, H, T_total, D, dtype, scale, q_norm_w, q_norm_b, k_norm_w,
                              k_norm_b, eps, rope_sin, rope_cos, rope_rows, prefix, tokens_per_frame);
  }
  // Where this rank's q, k, v and out rows live, and the layout of the K and V
  // halves of a ring block: K' head-major when the prologue writes it, else K
  // as given; V as given.  Every rank uses the same call, so every block
  // arriving over the ring has the sender's layout, which is this one.
  auto given = [&](uint32_t t) {
    return block ? hs::RowLayout::token_major(H, t, static_cast<uint64_t>(H) * 64) : hs::RowLayout::head_major(H, t);
  };

  // Block 0 = this rank's [K' | V] in buf[0], and this rank's Q'.  The
  // preps also record the largest q' and k' row norms; an all-ranks max of
  // those bounds every score of every step (fixed-offset softmax).
  const bool bounded = ln || rope;
  uint8_t* b0 = static_cast<uint8_t*>(ring->buf[0]);
  const void* q_use = q;
  if (bounded) {
    e = cudaMemsetAsync(ring->norm2, 0, 2 * sizeof(unsigned int), st);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring bound reset");
    kp.norm2_max = ring->norm2 + 1;
    qp.norm2_max = ring->norm2;
  }
  const hs::RowLayout in_rows = given(tr);
  if (bounded) {  // K' into block 0 and Q' into the state buffer, one launch
    const hs::PrepJob jobs[2] = {{k, in_rows, b0, kp}, {q, in_rows, ring->state, qp}};
    {
      hs::ProfScope prof(ctx, st, "qk_prep");
      e = hs::launch_qk_prep(st, code, code, 1, H, tr, jobs, 2, ctx->d_status, hs::ctx_timeout_ns(ctx));
    }
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring Q'/K' prep");
    q_use = ring->state;
  } else {
    e = cudaMemcpyAsync(b0, k, rows * row_bytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring K copy");
  }
  e = cudaMemcpyAsync(b0 + rows * row_bytes, v, rows * row_bytes, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return hs::abi_cuda_fail(e, "ring V copy");
  cudaEventRecord(ring->ev_block0, st);
  if (bounded) {
    cudaStreamWaitEvent(cs, ring->ev_block0, 0);
    ncclResult_t nr = n.AllReduce(ring->norm2, ring->norm2, 2, ncclUint32, ncclMax, ring->comm, cs);
    if (nr != ncclSuccess) return nccl_fail(nr, "ring bound all-reduce");
    cudaEventRecord(ring->ev_bound, cs);
    cudaStreamWaitEvent(st, ring->ev_bound, 0);
  }

  hs::AttnState state{};
  float* state_f = reinterpret_cast<float*>(ring->state + rows * row_bytes);
  state.o = state_f;
  state.m = state_f + rows * 64;
  state.l = state_f + rows * 65;
  for (int s = 0; s < R; ++s) {
    int src, send_to, recv_from, load, store;
    hs_ring_plan(r, R, s, &src, &send_to, &recv_from, &load, &store);
    uint32_t src_t0, src_len;
    shard_of(src, &src_t0, &src_len);
    uint8_t* cur = static_cast<uint8_t*>(ring->buf[s % 2]);
    uint8_t* nxt = static_cast<uint8_t*>(ring->buf[(s + 1) % 2]);
    if (send_to >= 0) {
      const int nsrc = (src - 1 + R) % R;  // the block the previous rank holds now
      uint32_t n_t0, n_len;
      shard_of(nsrc, &n_t0, &n_len);
      if (s == 0) cudaStreamWaitEvent(cs, ring->ev_block0, 0);
      if (s >= 1) cudaStreamWaitEvent(cs, ring->ev_compute[(s - 1) % 2], 0);  // nxt was read by step s-1
      hs::ProfScope prof(ctx, cs, "ring_transfer");
      ncclResult_t nr = n.GroupStart();
      if (nr == ncclSuccess) nr = n.Send(cur, 2ull * H * src_len * row_bytes, ncclUint8, send_to, ring->comm, cs);
      if (nr == ncclSuccess) nr = n.Recv(nxt, 2ull * H * n_len * row_bytes, ncclUint8, recv_from, ring->comm, cs);
      ncclResult_t ge = n.GroupEnd();
      if (nr != ncclSuccess) return nccl_fail(nr, "ring send/recv");
      if (ge != ncclSuccess) return nccl_fail(ge, "ring group");
      cudaEventRecord(ring->ev_recv[s % 2], cs);
    }
    if (s >= 1) cudaStreamWaitEvent(st, ring->ev_recv[(s - 1) % 2], 0);
    state.load = load;
    state.store = store;
    std::string err;
    {
      hs::ProfScope prof(ctx, st, "attention");
      hs::AttnIO io;
      io.q = q_use;
      io.lq = bounded ? hs::RowLayout::head_major(H, tr) : given(tr);
      io.k = cur;
      io.lk = bounded ? hs::RowLayout::head_major(H, src_len) : given(src_len);
      io.v = cur + static_cast<size_t>(H) * src_len * row_bytes;
      io.lv = given(src_len);
      io.out = out;
      io.lo = given(tr);
      io.out_code = code;
      const uint32_t ctas = static_cast<uint32_t>(ctx->sm_count) - ring->reserved_sms;
      e = hs::launch_attention_sm100(st, code, io, 1, H, tr, src_len, scale, state, ctas, ctx->d_status, ctx->d_sched,
                                     bounded ? ring->norm2 : nullptr, true, hs::ctx_timeout_ns(ctx), &err);
    }
    if (e != cudaSuccess)
      return hs::abi_fail(HS_ERR_CUDA, std::string(name) + ": " + (err.empty() ? cudaGetErrorString(e) : err));
    cudaEventRecord(ring->ev_compute[s % 2], st);
  }
  cudaEventRecord(ring->ev_done, st);
  return HS_OK;
}

// Head-parallel global attention (sequence parallelism by an all-to-all over
// heads): rank r holds tokens shard(T, R, r) of all H heads, as for the ring.
// The Q'/K' prep runs on the local shard (global RoPE positions), then one
// all-to-all gives every rank the whole sequence of its H / R heads, one
// attention launch computes them with nothing carried between launches, and a
// second all-to-all returns each rank's tokens of every head.  Per rank it
// moves 3 (R-1)/R of its q, k, v shard in and (R-1)/R of its output back,
// against (R-1) K/V blocks for the ring; H must be a multiple of R.
hs_status ulysses_attention(hs_ring* ring, const void* q, const void* k, const void* v, void* out, uint32_t H,
                            uint32_t T_total, uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                            const float* q_norm_b, const float* k_norm_w, const float* k_norm_b, float eps,
                            const float* rope_sin, const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                            uint32_t tokens_per_frame, const char* name) {
  if (!ring) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": null ring");
  if (ring->aborted) return hs::abi_fail(HS_ERR_NCCL, std::string(name) + ": ring was aborted");
  hs_ctx* ctx = ring->ctx;
  const int R = ring->world, r = ring->rank;
  if (ctx->cancel.load()) return hs::abi_fail(HS_ERR_CANCELLED, std::string(name) + ": cancelled");
  if (dtype != HS_F16 && dtype != HS_BF16)
    return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": f16/bf16 storage only");
  if (D != 64) return hs::abi_fail(HS_ERR_UNSUPPORTED, std::string(name) + ": head_dim must be 64");
  if (H == 0 || H > 65535 || H % static_cast<uint32_t>(R) != 0)
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": H must be a positive multiple of the ring size");
  if (T_total < static_cast<uint32_t>(R))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": need one token per rank");
  if (R == 1)
    return hs_attention_fused(ctx, q, k, v, out, 1, H, T_total, D, dtype, scale, q_norm_w, q_norm_b, k_norm_w,
                              k_norm_b, eps, rope_sin, rope_cos, rope_rows, prefix, tokens_per_frame);
  if (!q || !k || !v || !out) return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": tensor pointers must be 16-byte aligned");
  const bool ln = q_norm_w != nullptr;
  if (ln != (k_norm_w != nullptr) || (ln && (!q_norm_b || !k_norm_b)))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": QK-norm needs all of q/k weight and bias, or none");
  const bool rope = rope_sin != nullptr;
  const uint32_t tpf = tokens_per_frame ? tokens_per_frame : T_total;
  if (rope && (!rope_cos || prefix > tpf || rope_rows < tpf - prefix || !aligned16(rope_sin) || !aligned16(rope_cos)))
    return hs::abi_fail(HS_ERR_INVALID, std::string(name) + ": bad RoPE tables / prefix");
  if (!(scale > 0.f) || !isfinite(scale)) scale = 1.0f / sqrtf(static_cast<float>(D));

  cudaSetDevice(ctx->device);
  NcclApi& n = nccl();
  cudaStream_t st = hs::ctx_stream(ctx);
  cudaStream_t cs = ring->comm_stream;
  const int code = static_cast<int>(dtype);
  const size_t row_bytes = 64 * 2;
  const uint32_t G = H / static_cast<uint32_t>(R);  // heads per rank
  uint32_t t0, tr;
  shard(T_total, R, r, &t0, &tr);
  const uint32_t tmax = (T_total + R - 1) / R;
  const size_t local_rows = static_cast<size_t>(H) * tmax;
  const size_t full_rows = static_cast<size_t>(G) * T_total;
  const size_t need = (2 * local_rows + 4 * full_rows) * row_bytes;
  cudaError_t e;
  if (ring->uly_bytes < need) {
    cudaStreamSynchronize(st);
    cudaStreamSynchronize(cs);
    if (ring->uly) cudaFree(ring->uly);
    ring->uly = nullptr;
    ring->uly_bytes = 0;
    e = cudaMalloc(&ring->uly, need);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "head-parallel buffers");
    ring->uly_bytes = need;
  }
  uint8_t* lq = ring->uly;                   // (H, tr) Q' of this rank's tokens
  uint8_t* lk = lq + local_rows * row_bytes;  // (H, tr) K'
  uint8_t* fq = lk + local_rows * row_bytes;  // (G, T_total) Q' of this rank's heads
  uint8_t* fk = fq + full_rows * row_bytes;
  uint8_t* fv = fk + full_rows * row_bytes;
  uint8_t* fo = fv + full_rows * row_bytes;   // (G, T_total) output of this rank's heads

  // Q' and K' of the local tokens, with global RoPE positions, and their
  // largest row norms: an all-ranks max bounds every score (fixed offset).
  const bool bounded = ln || rope;
  const void* src_q = q;
  const void* src_k = k;
  if (bounded) {
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
    qp.pos_offset = t0;
    hs::QkPrologue kp = qp;
    kp.ln_w = k_norm_w;
    kp.ln_b = k_norm_b;
    e = cudaMemsetAsync(ring->norm2, 0, 2 * sizeof(unsigned int), st);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "head-parallel bound reset");
    qp.norm2_max = ring->norm2;
    kp.norm2_max = ring->norm2 + 1;
    const hs::RowLayout rows_in = hs::RowLayout::head_major(H, tr);
    const hs::PrepJob jobs[2] = {{k, rows_in, lk, kp}, {q, rows_in, lq, qp}};
    {
      hs::ProfScope prof(ctx, st, "qk_prep");
      e = hs::launch_qk_prep(st, code, code, 1, H, tr, jobs, 2, ctx->d_status, hs::ctx_timeout_ns(ctx));
    }
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "head-parallel Q'/K' prep");
    src_q = lq;
    src_k = lk;
  }
  cudaEventRecord(ring->ev_block0, st);
  cudaStreamWaitEvent(cs, ring->ev_block0, 0);
  if (bounded) {
    ncclResult_t nr = n.AllReduce(ring->norm2, ring->norm2, 2, ncclUint32, ncclMax, ring->comm, cs);
    if (nr != ncclSuccess) return nccl_fail(nr, "head-parallel bound all-reduce");
  }

  // Inbound all-to-all.  To each rank p this rank sends its rows of head
  // p*G + j (tr contiguous rows of its head-major (H, tr) shard), which p
  // stores at rows [t0, t0 + tr) of its head j; from each p it receives p's
  // rows of head r*G + j into rows [t0_p, t0_p + tr_p) of its own head j.
  // Every pair issues its sends and receives in the same (tensor, head) order.
  const void* src[3] = {src_q, src_k, v};
  uint8_t* dst[3] = {fq, fk, fv};
  {
    hs::ProfScope prof(ctx, cs, "ring_transfer");
    ncclResult_t nr = n.GroupStart();
    for (int x = 0; x < 3 && nr == ncclSuccess; ++x) {
      const uint8_t* sx = static_cast<const uint8_t*>(src[x]);
      for (int p = 0; p < R && nr == ncclSuccess; ++p) {
        if (p == r) continue;
        uint32_t p0, pl;
        shard(T_total, R, p, &p0, &pl);
        for (uint32_t j = 0; j < G && nr == ncclSuccess; ++j) {
          const size_t send_row = (static_cast<size_t>(p) * G + j) * tr;
          nr = n.Send(sx + send_row * row_bytes, static_cast<size_t>(tr) * row_bytes, ncclUint8, p, ring->comm, cs);
          if (nr != ncclSuccess) break;
          const size_t recv_row = static_cast<size_t>(j) * T_total + p0;
          nr = n.Recv(dst[x] + recv_row * row_bytes, static_cast<size_t>(pl) * row_bytes, ncclUint8, p, ring->comm,
                      cs);
        }
      }
    }
    ncclResult_t ge = n.GroupEnd();
    if (nr != ncclSuccess) return nccl_fail(nr, "head-parallel send/recv");
    if (ge != ncclSuccess) return nccl_fail(ge, "head-parallel group");
  }
  // This rank's own rows of its heads.
  for (int x = 0; x < 3; ++x)
    for (uint32_t j = 0; j < G; ++j) {
      const size_t from = (static_cast<size_t>(r) * G + j) * tr, to = static_cast<size_t>(j) * T_total + t0;
      e = cudaMemcpyAsync(dst[x] + to * row_bytes, static_cast<const uint8_t*>(src[x]) + from * row_bytes,
                          static_cast<size_t>(tr) * row_bytes, cudaMemcpyDeviceToDevice, cs);
      if (e != cudaSuccess) return hs::abi_cuda_fail(e, "head-parallel local rows");
    }
  cudaEventRecord(ring->ev_in, cs);
  cudaStreamWaitEvent(st, ring->ev_in, 0);

  // One launch over the whole sequence of this rank's heads.
  std::string err;
  {
    hs::ProfScope prof(ctx, st, "attention");
    hs::AttnIO io;
    const hs::RowLayout full = hs::RowLayout::head_major(G, T_total);
    io.q = fq;
    io.lq = full;
    io.k = fk;
    io.lk = full;
    io.v = fv;
    io.lv = full;
    io.out = fo;
    io.lo = full;
    io.out_code = code;
    e = hs::launch_attention_sm100(st, code, io, 1, G, T_total, T_total, scale, hs::AttnState{}, 0, ctx->d_status,
                                   ctx->d_sched, bounded ? ring->norm2 : nullptr, true, hs::ctx_timeout_ns(ctx),
                                   &err);
  }
  if (e != cudaSuccess)
    return hs::abi_fail(HS_ERR_CUDA, std::string(name) + ": " + (err.empty() ? cudaGetErrorString(e) : err));
  cudaEventRecord(ring->ev_attn, st);
  cudaStreamWaitEvent(cs, ring->ev_attn, 0);

  // Outbound all-to-all: rows [t0_p, t0_p + tr_p) of each of this rank's heads
  // go to rank p, which stores them as its head r*G + j.
  uint8_t* o = static_cast<uint8_t*>(out);
  {
    hs::ProfScope prof(ctx, cs, "ring_transfer");
    ncclResult_t nr = n.GroupStart();
    for (int p = 0; p < R && nr == ncclSuccess; ++p) {
      if (p == r) continue;
      uint32_t p0, pl;
      shard(T_total, R, p, &p0, &pl);
      for (uint32_t j = 0; j < G && nr == ncclSuccess; ++j) {
        const size_t send_row = static_cast<size_t>(j) * T_total + p0;
        nr = n.Send(fo + send_row * row_bytes, static_cast<size_t>(pl) * row_bytes, ncclUint8, p, ring->comm, cs);
        if (nr != ncclSuccess) break;
        const size_t recv_row = (static_cast<size_t>(p) * G + j) * tr;
        nr = n.Recv(o + recv_row * row_bytes, static_cast<size_t>(tr) * row_bytes, ncclUint8, p, ring->comm, cs);
      }
    }
    ncclResult_t ge = n.GroupEnd();
    if (nr != ncclSuccess) return nccl_fail(nr, "head-parallel output send/recv");
    if (ge != ncclSuccess) return nccl_fail(ge, "head-parallel output group");
  }
  for (uint32_t j = 0; j < G; ++j) {
    const size_t from = static_cast<size_t>(j) * T_total + t0, to = (static_cast<size_t>(r) * G + j) * tr;
    e = cudaMemcpyAsync(o + to * row_bytes, fo + from * row_bytes, static_cast<size_t>(tr) * row_bytes,
                        cudaMemcpyDeviceToDevice, cs);
    if (e != cudaSuccess) return hs::abi_cuda_fail(e, "head-parallel local output rows");
  }
  cudaEventRecord(ring->ev_done, cs);
  cudaStreamWaitEvent(st, ring->ev_done, 0);
  return HS_OK;
}

}  // namespace

extern "C" {

hs_status hs_ring_attention_fused(hs_ring* ring, const void* q, const void* k, const void* v, void* out, uint32_t H,
                                  uint32_t T_total, uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                                  const float* q_norm_b, const float* k_norm_w, const float* k_norm_b, float eps,
                                  const float* rope_sin, const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                  uint32_t tokens_per_frame) {
  return ring_attention(ring, q, k, v, out, H, T_total, D, dtype, scale, q_norm_w, q_norm_b, k_norm_w, k_norm_b, eps,
                        rope_sin, rope_cos, rope_rows, prefix, tokens_per_frame, false, 1,
                        "hs_ring_attention_fused");
}

hs_status hs_ring_attention_block_fused(hs_ring* ring, const void* q, const void* k, const void* v, void* out,
                                        uint32_t H, uint32_t T_total, uint32_t D, hs_dtype dtype, float scale,
                                        const float* q_norm_w, const float* q_norm_b, const float* k_norm_w,
                                        const float* k_norm_b, float eps, const float* rope_sin,
                                        const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                        uint32_t tokens_per_frame, uint32_t shard_unit) {
  return ring_attention(ring, q, k, v, out, H, T_total, D, dtype, scale, q_norm_w, q_norm_b, k_norm_w, k_norm_b, eps,
                        rope_sin, rope_cos, rope_rows, prefix, tokens_per_frame, true, shard_unit,
                        "hs_ring_attention_block_fused");
}

hs_status hs_ring_ulysses_attention_fused(hs_ring* ring, const void* q, const void* k, const void* v, void* out,
                                          uint32_t H, uint32_t T_total, uint32_t D, hs_dtype dtype, float scale,
                                          const float* q_norm_w, const float* q_norm_b, const float* k_norm_w,
                                          const float* k_norm_b, float eps, const float* rope_sin,
                                          const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                          uint32_t tokens_per_frame) {
  return ulysses_attention(ring, q, k, v, out, H, T_total, D, dtype, scale, q_norm_w, q_norm_b, k_norm_w, k_norm_b,
                           eps, rope_sin, rope_cos, rope_rows, prefix, tokens_per_frame,
                           "hs_ring_ulysses_attention_fused");
}

hs_status hs_ring_sync(hs_ring* ring, uint32_t timeout_ms) {
  if (!ring) return hs::abi_fail(HS_ERR_INVALID, "hs_ring_sync: null ring");
  if (ring->aborted) return hs::abi_fail(HS_ERR_NCCL, "hs_ring_sync: ring was aborted");
  NcclApi& n = nccl();
  cudaSetDevice(ring->ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q1 = cudaStreamQuery(ring->comm_stream);
    cudaError_t q2 = cudaStreamQuery(hs::ctx_stream(ring->ctx));
    if (q1 == cudaSuccess && q2 == cudaSuccess) break;
    if ((q1 != cudaSuccess && q1 != cudaErrorNotReady) || (q2 != cudaSuccess && q2 != cudaErrorNotReady))
      return hs::abi_cuda_fail(q1 != cudaSuccess && q1 != cudaErrorNotReady ? q1 : q2, "hs_ring_sync");
    ncclResult_t async_err = ncclSuccess;
    n.CommGetAsyncError(ring->comm, &async_err);
    const double waited =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if ((async_err != ncclSuccess && async_err != ncclInProgress) || waited > timeout_ms) {
      n.CommAbort(ring->comm);
      ring->comm = nullptr;
      ring->aborted = true;
      if (async_err != ncclSuccess && async_err != ncclInProgress) return nccl_fail(async_err, "hs_ring_sync");
      return hs::abi_fail(HS_ERR_TIMEOUT, "hs_ring_sync: ring did not finish in time; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  return hs_sync(ring->ctx);
}

}  // extern "C"
