/*
 * headshot_cuda.h — C ABI of the B200 (sm_100a) attention path for
 * headshot-server's aggregator.
 *
 * Drop-in boundary: each entry point replaces one `GpuContext` op of the
 * reference engine (Feilkin/headshot, crates/headshot-server/src/engine/),
 * keeping its tensor layouts and argument meaning.  Plain pointers and sizes
 * only; device pointers come from hs_alloc (or any CUDA allocation on the
 * context's device).  Every call is asynchronous on the context's stream;
 * hs_sync waits and reports deferred device errors, like the reference's
 * flush/download (src/engine/mod.rs:261-284).
 *
 * Errors: where the reference panics through assert! (shape, dtype, table
 * size), these functions return HS_ERR_INVALID and leave a message for
 * hs_last_error(); they never abort or throw across the ABI.
 *
 * Layouts (as in the reference):
 *   head-major  (S, H, T, D)  contiguous — attention q/k/v/out
 *   token-major (S*T, H*D)    contiguous — GEMM activations
 *   RoPE tables (P, 64) f32, P = patch rows
 */
#ifndef HEADSHOT_CUDA_H
#define HEADSHOT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HS_ABI_VERSION 2u

#if defined(__GNUC__)
#define HS_API __attribute__((visibility("default")))
#else
#define HS_API
#endif

typedef enum hs_status {
  HS_OK = 0,
  HS_ERR_INVALID = 1,     /* contract violated; the reference would panic */
  HS_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  HS_ERR_CUDA = 3,        /* CUDA runtime error */
  HS_ERR_OOM = 4,         /* device allocation failed */
  HS_ERR_TIMEOUT = 5,     /* a kernel's bounded wait gave up; context stays usable */
  HS_ERR_NCCL = 6,        /* NCCL error in a multi-GPU call */
  HS_ERR_CANCELLED = 7    /* cancellation requested (src/engine/mod.rs:102-106) */
} hs_status;

/* Storage types: the reference's Dtype::{F32,F16} (src/engine/tensor.rs:13-16) plus bf16. */
typedef enum hs_dtype { HS_F32 = 0, HS_F16 = 1, HS_BF16 = 2 } hs_dtype;

typedef struct hs_ctx hs_ctx;

/* ------------------------------------------------------------ context --- */

HS_API uint32_t hs_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
HS_API const char* hs_last_error(void);

/* Replaces GpuContext::new (src/engine/mod.rs:111-211): binds `device`,
 * creates the context's stream and device status word. */
HS_API hs_status hs_ctx_create(int device, hs_ctx** out);
HS_API hs_status hs_ctx_destroy(hs_ctx* ctx);

/* Run subsequent calls on a caller-owned cudaStream_t (NULL is the legacy
 * default stream); hs_ctx_use_own_stream returns to the context's stream. */
HS_API hs_status hs_ctx_set_stream(hs_ctx* ctx, void* stream);
HS_API hs_status hs_ctx_use_own_stream(hs_ctx* ctx);
HS_API void* hs_ctx_stream(hs_ctx* ctx);

/* Upper bound for every in-kernel wait, in milliseconds (default 2000).
 * A wait that gives up records a site code; the kernel's CTAs then stop,
 * let their own copies and tensor-core work in flight finish (a fixed bound
 * of 4 s of their own) and exit, and hs_sync returns HS_ERR_TIMEOUT with the
 * context still usable.  ms = 0 means "do not wait": a wait whose condition
 * does not already hold gives up at once, which drives every call into that
 * path deterministically (for testing the timeout handling). */
HS_API hs_status hs_ctx_set_wait_timeout_ms(hs_ctx* ctx, uint32_t ms);

/* Cooperative cancellation (src/engine/mod.rs:92-95, :286-304): multi-step
 * calls check the flag between steps and return HS_ERR_CANCELLED. */
HS_API hs_status hs_ctx_request_cancel(hs_ctx* ctx);
HS_API hs_status hs_ctx_clear_cancel(hs_ctx* ctx);

/* Per-kernel timing (the reference's unused TIMESTAMP_QUERY, mod.rs:137):
 * when enabled, every kernel launch is bracketed by CUDA events on its
 * stream.  hs_prof_read synchronises and returns the summed device time and
 * launch count of `kernel` ("attention", "qk_prep", "layernorm",
 * "rope_apply", "permute", or "*" for all). */
HS_API hs_status hs_prof_enable(hs_ctx* ctx, int on);
HS_API hs_status hs_prof_reset(hs_ctx* ctx);
HS_API hs_status hs_prof_read(hs_ctx* ctx, const char* kernel, double* total_ms, uint64_t* launches);

/* ------------------------------------------------------------- memory --- */

/* Stream-ordered device pool; replaces GpuContext::empty_typed /
 * create_buffer (src/engine/tensor.rs:59-63, :132-140).  Memory is NOT
 * zero-filled (the reference zero-fills; call hs_memset where it matters). */
HS_API hs_status hs_alloc(hs_ctx* ctx, size_t bytes, void** out);
HS_API hs_status hs_free(hs_ctx* ctx, void* ptr);
HS_API hs_status hs_memset(hs_ctx* ctx, void* dst, int value, size_t bytes);
/* Replaces tensor_from_f32 upload (tensor.rs:66-89) and download (tensor.rs:163-198). */
HS_API hs_status hs_memcpy_h2d(hs_ctx* ctx, void* dst_device, const void* src_host, size_t bytes);
HS_API hs_status hs_memcpy_d2h(hs_ctx* ctx, void* dst_host, const void* src_device, size_t bytes);
/* Replaces GpuContext::flush + sync (src/engine/mod.rs:261-284): waits for
 * the stream and returns HS_ERR_TIMEOUT if a kernel's bounded wait fired. */
HS_API hs_status hs_sync(hs_ctx* ctx);

/* -------------------------------------------------------------- ops ---- */

/* Replaces GpuContext::attention (src/engine/ops.rs:228-253).
 * q, k, v, out: (S, H, T, D) of `dtype`; D is 64 or 128; S*H <= 65535.
 * scale <= 0 selects 1/sqrt(D) as the reference does (ops.rs:244).
 * D = 64: f16/bf16 inputs compute on tcgen05 in that type with f32
 * softmax; f32 inputs are rounded to bf16 for the tensor core, out stays
 * f32.  D = 128 (the camera head's "attention_d128", ops.rs:236): f32
 * arithmetic for every storage type; the fused entry points take it only
 * without a QK-norm/RoPE prologue (the camera head has none). */
HS_API hs_status hs_attention(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S, uint32_t H,
                       uint32_t T, uint32_t D, hs_dtype dtype, float scale);

/* The attention section of Block::forward (src/model/block.rs:136-148) as
 * one op: QK-norm (LayerNorm over D with f32 weight/bias, eps) on q and k,
 * then 2D RoPE (rotate-half, src/engine/rope.rs:48-55) on q and k, then
 * attention.  Q and K are normalised/rotated once into context scratch
 * (one pass each), which also bounds every score for the softmax.
 *   q_norm_w == NULL: no QK-norm (k_norm_w must then be NULL too).
 *   rope_sin == NULL: no RoPE.  Otherwise the table row of token t is
 *   (t mod tokens_per_frame) - prefix and tokens with (t mod tokens_per_frame)
 *   < prefix pass through; tokens_per_frame == 0 means T (the reference's
 *   rope_apply, ops.rs:202-223).  rope_rows >= tokens_per_frame - prefix. */
HS_API hs_status hs_attention_fused(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t S,
                             uint32_t H, uint32_t T, uint32_t D, hs_dtype dtype, float scale, const float* q_norm_w,
                             const float* q_norm_b, const float* k_norm_w, const float* k_norm_b, float eps,
                             const float* rope_sin, const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                             uint32_t tokens_per_frame);

/* Block::forward's whole attention section (src/model/block.rs:130-149) in
 * the layout the projections produce and consume: q, k, v are the three
 * (S*T, H*D) outputs of the q/k/v linears (token-major, the input of
 * split_heads, ops.rs:185-200) and out is (S*T, H*D), the output of
 * attn_merge (ops.rs:255-267) that the proj linear reads.  Same arguments
 * and results as hs_attention_fused otherwise; the split, QK-norm, RoPE,
 * attention and merge run as one prep pass per q/k and one attention
 * kernel reading v and writing out in place (no head-major copies of v or
 * out).  Note the argument order S, T, H, D of split_heads. */
HS_API hs_status hs_attention_block_fused(hs_ctx* ctx, const void* q, const void* k, const void* v, void* out,
                                          uint32_t S, uint32_t T, uint32_t H, uint32_t D, hs_dtype dtype,
                                          float scale, const float* q_norm_w, const float* q_norm_b,
                                          const float* k_norm_w, const float* k_norm_b, float eps,
                                          const float* rope_sin, const float* rope_cos, uint32_t rope_rows,
                                          uint32_t prefix, uint32_t tokens_per_frame);

/* No counterpart in the reference.  hs_attention_fused for callers that
 * cannot let the library allocate device memory: hosts whose device memory
 * belongs to their own allocator or a pool reserved up front, and session
 * loops that must not stall or fail on an allocation once running.  Same
 * arguments and results as hs_attention_fused (f16/bf16 storage only), but
 * no hs_ctx: work goes on `stream` (a cudaStream_t, NULL = legacy default
 * stream) of the current device, and the normalised Q and K live in a fixed
 * array inside the library — 2 x HS_NOALLOC_MAX_ROWS rows of 128 bytes
 * (64 MiB), held by every GPU that loads the library until the process exits.
 * With a QK-norm or RoPE prologue, S*H*T above HS_NOALLOC_MAX_ROWS returns
 * HS_ERR_INVALID; without either, q and k are read in place and the array
 * is not used for rows, so there is no row limit.
 * The first call on a device looks up that array's device address (no
 * allocation by this library); make that first call before any stream
 * capture.  All calls on a device share the array, so calls whose work
 * overlaps on the GPU race; order them on one stream.  `status` (device
 * int) is zeroed by each call and receives a nonzero site code if an
 * in-kernel wait timed out.  With status == NULL the site code goes to a
 * word inside the library that nothing reads: timeouts are then not
 * reported and the call's output may be incomplete without notice, so pass
 * a status word wherever a timeout must be seen. */
#define HS_NOALLOC_MAX_ROWS 262144u
HS_API hs_status hs_attention_fused_noalloc(void* stream, int* status, const void* q, const void* k, const void* v,
                                            void* out, uint32_t S, uint32_t H, uint32_t T, uint32_t D,
                                            hs_dtype dtype, float scale, const float* q_norm_w,
                                            const float* q_norm_b, const float* k_norm_w, const float* k_norm_b,
                                            float eps, const float* rope_sin, const float* rope_cos,
                                            uint32_t rope_rows, uint32_t prefix, uint32_t tokens_per_frame);

/* Replaces GpuContext::linear (src/engine/ops.rs:87-128) and fuses the
 * element-wise op that follows each linear in Block::forward:
 *   out (M, N) = x (M, K) . w (N, K)^T [+ bias (N, f32)], then
 *   HS_LINEAR_PLAIN       nothing                      (qkv projections)
 *   HS_LINEAR_GELU        erf GELU (shaders/gelu.wesl) (MLP fc1 + gelu, block.rs:173-174)
 *   HS_LINEAR_RESIDUAL_LS out = residual + gamma (.) out (proj/fc2 + residual_ls,
 *                         shaders/residual_ls.wesl); residual (M, N), gamma (N, f32).
 * f16/bf16 storage on tcgen05 with f32 accumulation (the fused epilogue
 * works on the f32 sum; the reference rounds the linear's output first).
 * K and N must be multiples of 8 for 16-bit storage.  f32 storage (the
 * reference's DINO and camera head) computes in f32 on the CUDA cores, any
 * K and N, M <= 65535 * 128.
 * All pointers 16-byte aligned; bias may be NULL.  out may alias residual. */
#define HS_LINEAR_PLAIN 0
#define HS_LINEAR_GELU 1
#define HS_LINEAR_RESIDUAL_LS 2
HS_API hs_status hs_linear(hs_ctx* ctx, const void* x, const void* w, const float* bias, void* out, uint64_t M,
                           uint32_t K, uint32_t N, hs_dtype dtype, int epilogue, const void* residual,
                           const float* gamma);

/* Replaces GpuContext::layernorm (src/engine/ops.rs:130-153), with eps an
 * argument (the reference fixes 1e-5, ops.rs:139).  w, b: (dim) f32. */
HS_API hs_status hs_layernorm(hs_ctx* ctx, const void* x, const float* w, const float* b, void* out, uint64_t rows,
                       uint32_t dim, float eps, hs_dtype dtype);

/* Replaces GpuContext::rope_apply (src/engine/ops.rs:202-223): in place on
 * (S, H, T, D); tables (rope_rows, D) f32 with rope_rows == T - prefix. */
HS_API hs_status hs_rope_apply(hs_ctx* ctx, void* x, const float* rope_sin, const float* rope_cos, uint32_t rope_rows,
                        uint32_t S, uint32_t H, uint32_t T, uint32_t D, uint32_t prefix, hs_dtype dtype);

/* Replaces GpuContext::split_heads (src/engine/ops.rs:185-200): (S*T, H*D) -> (S, H, T, D). */
HS_API hs_status hs_split_heads(hs_ctx* ctx, const void* x, void* out, uint32_t S, uint32_t T, uint32_t H, uint32_t D,
                         hs_dtype dtype);

/* Replaces GpuContext::attn_merge (src/engine/ops.rs:255-267): (S, H, T, D) -> (S*T, H*D). */
HS_API hs_status hs_attn_merge(hs_ctx* ctx, const void* x, void* out, uint32_t S, uint32_t H, uint32_t T, uint32_t D,
                        hs_dtype dtype);

/* --------------------------------------- multi-GPU session (ring) ------ */

/* The reference is single-device; this layer is new.  Global attention over
 * one sequence of T_total tokens is split into `world` contiguous shards
 * (hs_ring_shard); rank r owns q, k, v, out of shape (H, T_r, 64).  K is
 * normalised/rotated once by its owner, then [K'|V] blocks rotate around the
 * ring over NCCL send/recv, overlapped with the attention kernel; the
 * running softmax state stays on each rank in f32. */
typedef struct hs_ring hs_ring;

/* [start, start+len) of rank's shard; the first n % world ranks get one extra token. */
HS_API hs_status hs_ring_shard(uint32_t n, int world, int rank, uint32_t* start, uint32_t* len);
/* Step `step` of the ring on `rank`: which block it attends to, its peers
 * (-1 on the last step: nothing to send), and whether the kernel loads /
 * stores the carried softmax state. */
HS_API hs_status hs_ring_plan(int rank, int world, int step, int* src_block, int* send_to, int* recv_from,
                              int* load_state, int* store_state);
HS_API size_t hs_ring_id_bytes(void);
/* Rank 0 creates the id and shares its bytes with the other ranks out of band. */
HS_API hs_status hs_ring_unique_id(void* id_out);
/* Collective over all ranks; one rank per GPU, ctx bound to that GPU. */
HS_API hs_status hs_ring_create(hs_ctx* ctx, int rank, int world, const void* id, hs_ring** out);
HS_API hs_status hs_ring_destroy(hs_ring* ring);
/* SMs the ring's attention launches leave free, so that the NCCL kernel
 * moving the next [K'|V] block runs alongside the attention kernel instead
 * of between launches; 0 (the default) gives attention every SM.  Must
 * leave at least one SM for attention. */
HS_API hs_status hs_ring_set_reserved_sms(hs_ring* ring, uint32_t sms);
/* Global attention over the ring, arguments as hs_attention_fused with
 * S = 1; RoPE positions use each token's global index. f16/bf16 only. */
HS_API hs_status hs_ring_attention_fused(hs_ring* ring, const void* q, const void* k, const void* v, void* out,
                                         uint32_t H, uint32_t T_total, uint32_t D, hs_dtype dtype, float scale,
                                         const float* q_norm_w, const float* q_norm_b, const float* k_norm_w,
                                         const float* k_norm_b, float eps, const float* rope_sin,
                                         const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                         uint32_t tokens_per_frame);
/* hs_ring_attention_fused on Block::forward's layout (block.rs:130-149),
 * for a trunk whose tokens are sharded across ranks by whole frames: q, k, v
 * are this rank's (T_r, H*D) rows of the q/k/v linears and out its (T_r,
 * H*D) merged attention output (the proj linear's input).  Rank r owns the
 * tokens of units shard(T_total / shard_unit, world, r) (hs_ring_shard's
 * rule over units; shard_unit = tokens per frame keeps frames whole);
 * T_total must be a multiple of shard_unit.  Every rank passes the same
 * T_total, shard_unit and prologue. */
HS_API hs_status hs_ring_attention_block_fused(hs_ring* ring, const void* q, const void* k, const void* v, void* out,
                                               uint32_t H, uint32_t T_total, uint32_t D, hs_dtype dtype, float scale,
                                               const float* q_norm_w, const float* q_norm_b, const float* k_norm_w,
                                               const float* k_norm_b, float eps, const float* rope_sin,
                                               const float* rope_cos, uint32_t rope_rows, uint32_t prefix,
                                               uint32_t tokens_per_frame, uint32_t shard_unit);
/* hs_ring_attention_fused's contract (each rank's (1, H, T_r, 64) shard of
 * hs_ring_shard's tokens in and out, global RoPE positions, f16/bf16), by
 * head parallelism instead of the ring: the Q'/K' prep runs on the local
 * shard, an all-to-all over NCCL gives each rank the whole sequence of its
 * H / world heads, one attention launch computes them (no softmax state
 * carried between launches), and a second all-to-all returns every rank's
 * tokens of all heads.  H must be a multiple of the ring's world size.  New
 * (the reference is single-device, src/model/trunk.rs:92-144). */
HS_API hs_status hs_ring_ulysses_attention_fused(hs_ring* ring, const void* q, const void* k, const void* v,
                                                 void* out, uint32_t H, uint32_t T_total, uint32_t D, hs_dtype dtype,
                                                 float scale, const float* q_norm_w, const float* q_norm_b,
                                                 const float* k_norm_w, const float* k_norm_b, float eps,
                                                 const float* rope_sin, const float* rope_cos, uint32_t rope_rows,
                                                 uint32_t prefix, uint32_t tokens_per_frame);
/* Waits for the ring's work with a host-side watchdog: on an NCCL async
 * error or after timeout_ms the communicator is aborted and the ring
 * becomes unusable (HS_ERR_NCCL / HS_ERR_TIMEOUT). */
HS_API hs_status hs_ring_sync(hs_ring* ring, uint32_t timeout_ms);

/* ------------------------------------------------------ host helpers --- */

/* Trunk glue (src/model/trunk.rs:78-84 and 105-122, GpuContext::copy_rows at
 * src/engine/tensor.rs:148-160):
 * for g < groups, rows [g*src_stride_rows, +rows) of src (row width `cols`
 * elements of dtype) are copied to rows [g*dst_stride_rows, +rows) of dst.
 * The register gather is (groups = N, src stride T, dst stride 17, rows 17);
 * the scatter back swaps the strides; groups = 1 is copy_rows.  Rows must
 * be 16-byte multiples and pointers 16-byte aligned.  src_stride_rows = 0
 * copies the same source rows into every group (the per-frame camera and
 * register tokens of trunk.rs:78-84, the cls/storage tokens of dino.rs). */
HS_API hs_status hs_copy_row_blocks(hs_ctx* ctx, const void* src, void* dst, uint64_t groups,
                                    uint64_t src_stride_rows, uint64_t dst_stride_rows, uint64_t rows,
                                    uint32_t cols, hs_dtype dtype);

/* Patch embedding front half (GpuContext::im2col_patch, ops.rs:271-300 ->
 * im2col_patch.wesl): images (n, 3, height, width) f32 in [0, 1] -> out
 * (n * (height/patch) * (width/patch), row_stride) of dtype, row = one patch
 * (frame-major, then patch row, patch column), column c*patch*patch +
 * ky*patch + kx = (pixel - mean[c]) / std[c]; columns from 3*patch*patch to
 * row_stride are written as zero (a K padded for the patch GEMM).  mean and
 * std are host arrays of 3, or NULL for the ImageNet statistics.  The
 * reference fixes patch = 16 and row_stride = 768. */
HS_API hs_status hs_im2col_patch(hs_ctx* ctx, const float* images, void* out, uint32_t n, uint32_t height,
                                 uint32_t width, uint32_t patch, uint32_t row_stride, const float* mean,
                                 const float* std_dev, hs_dtype dtype);

/* Head-input cache (src/model/cache.rs:25-52: concat_channels + cast_to_f32):
 * out (rows, cols_frame + cols_global) f32 = [frame_out row | global_out row]
 * for rows of dtype.  One buffer (no 2 GiB chunking on this device). */
HS_API hs_status hs_cache_build(hs_ctx* ctx, const void* frame_out, const void* global_out, float* out,
                                uint64_t rows, uint32_t cols_frame, uint32_t cols_global, hs_dtype dtype);

/* Replaces rope::periods (src/engine/rope.rs:8-10): 100^(2i/32), i < 16. */
HS_API hs_status hs_rope_periods(float* out16);

/* Replaces rope::tables (src/engine/rope.rs:15-44): host (P, 64) sin/cos,
 * P = h_p*w_p; periods == NULL uses hs_rope_periods. */
HS_API hs_status hs_rope_tables(const float* periods, uint32_t h_p, uint32_t w_p, float* sin_out, float* cos_out);

#ifdef __cplusplus
}
#endif

#endif /* HEADSHOT_CUDA_H */
