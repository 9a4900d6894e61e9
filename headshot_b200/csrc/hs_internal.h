// hs_internal.h — launchers shared between the kernel files and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace hs {

// Storage element codes used inside the library (match hs_dtype).
enum ElemCode : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

inline size_t elem_bytes(int code) { return code == kF32 ? 4 : 2; }

// QK-norm + 2D RoPE applied to a head vector (D = 64) in f32, in the order
// of the reference block (LayerNorm, then rotate-half RoPE).
struct QkPrologue {
  const float* ln_w = nullptr;  // (64) f32, used when ln != 0
  const float* ln_b = nullptr;  // (64) f32
  float eps = 1e-5f;
  int ln = 0;
  const float* sin_t = nullptr;  // (P, 64) f32, used when rope != 0
  const float* cos_t = nullptr;
  uint32_t prefix = 0;            // tokens [0, prefix) of every frame pass through
  uint32_t tokens_per_frame = 0;  // table row of token t is (t mod tpf) - prefix
  int rope = 0;
  uint32_t pos_offset = 0;  // global index of this shard's token 0 (ring shards)
  // When set, raised (atomicMax on the f32 bit pattern) to the largest
  // squared norm of the rows written, as stored (after 16-bit rounding).
  unsigned int* norm2_max = nullptr;
};

// Running softmax state for attention split over several launches (ring
// steps): per query row the unnormalised f32 accumulator O (64), the running
// max m (log2 domain, scaled) and the running sum l.
struct AttnState {
  float* o = nullptr;  // (SH, T, 64) f32
  float* m = nullptr;  // (SH, T) f32
  float* l = nullptr;  // (SH, T) f32
  int load = 0;        // read the state before the first KV tile
  int store = 0;       // write the state instead of the normalised output
};

// Where row (s, h, t) of a (S, H, T, 64) tensor starts, in elements: the
// strides of t, h and s (the 64 elements of a row are contiguous).
struct RowLayout {
  uint64_t t = 64, h = 0, s = 0;
  // (S, H, T, 64) contiguous, the reference's attention layout (ops.rs:228).
  static RowLayout head_major(uint32_t H, uint32_t T) {
    return RowLayout{64, static_cast<uint64_t>(T) * 64, static_cast<uint64_t>(H) * T * 64};
  }
  // (S*T, H*64) rows of `row_elems` >= H*64 elements (projection outputs and
  // the merged attention output, ops.rs:185-200 / 255-267).
  static RowLayout token_major(uint32_t H, uint32_t T, uint64_t row_elems) {
    return RowLayout{row_elems, 64, static_cast<uint64_t>(T) * row_elems};
  }
  __host__ __device__ uint64_t at(uint64_t s_, uint64_t h_, uint64_t t_) const { return s_ * s + h_ * h + t_ * t; }
};

// Operands of one attention launch: 16-bit q, k, v rows of type `elem` and
// the output (kF32 or `elem`), each with its own row layout.
struct AttnIO {
  const void* q = nullptr;
  RowLayout lq;
  const void* k = nullptr;
  RowLayout lk;
  const void* v = nullptr;
  RowLayout lv;
  void* out = nullptr;
  RowLayout lo;
  int out_code = 0;
};

// cuTensorMapEncodeTiled, looked up once through the runtime's driver entry
// point (null if the driver does not provide it).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// (S, H, T, 64) 16-bit rows in layout `l` as a 4-D tensor map (64, T, H, S)
// with box_rows x 64 boxes and 128-byte swizzle; rows past T inside a
// sequence read as zeros.  base must be 16-byte aligned and the strides of
// `l` multiples of 8 elements.
bool make_row_map(CUtensorMap* map, const void* base, const RowLayout& l, bool bf16, uint32_t t, uint32_t heads,
                  uint32_t seqs, uint32_t box_rows, std::string* err);

// SMs of the current device (cached per device; 148 if the query fails).
int current_sm_count();

// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device (once per kernel and device).
cudaError_t ensure_dynamic_smem(const void* func, int bytes);

// Flash attention on tcgen05 (D = 64), persistent: at most `max_ctas` CTAs
// (0 = one per SM) take the (sequence, 256-row) work items from the counter
// pair `sched` (2 x u32, zero before the launch; the kernel leaves it zero,
// so launches sharing it must be ordered on one stream).  q, k and v are
// 16-bit rows of `elem` (kF16 or kBF16) with any QK-norm/RoPE already
// applied (qk_prep); out is written in `out_code` (kF32 or `elem`).
// `qk_norm2` (2 x u32 or null): the max squared row norms of q and k as
// qk_prep recorded them; when they bound every score tightly enough the
// softmax uses a fixed offset instead of a running max.  Zeroed by the
// kernel unless `norm2_shared`: then the caller guarantees they bound every
// launch that carries the same state `st` (all ring steps) and resets them.
// S sequences of H heads; the state arrays are indexed head-major.
// head_dim 128 (the camera head's attention), f32 arithmetic on the CUDA
// cores; q/k/v/out of storage type `code` (kF32/kF16/kBF16) at the strides of
// their RowLayouts (rows of 128 elements).
cudaError_t launch_attention_d128(cudaStream_t stream, int code, const AttnIO& io, uint32_t S, uint32_t H, uint32_t T,
                                  float scale);
cudaError_t launch_attention_sm100(cudaStream_t stream, int elem, const AttnIO& io, uint32_t S, uint32_t H,
                                   uint32_t t_q, uint32_t t_kv, float scale, const AttnState& st, uint32_t max_ctas,
                                   int* status, uint32_t* sched, unsigned int* qk_norm2, bool norm2_shared,
                                   uint64_t timeout_ns, std::string* err);

// Row prep for K (and for casts): out = RoPE(LN(x)) in `out_code` storage.
// Trunk glue (ops.cu): strided row-block copies (register gather/scatter,
// copy_rows) and the f32 head-input cache row build.  Rows are 16-byte
// multiples; pointers 16-byte aligned.
cudaError_t launch_copy_row_blocks(cudaStream_t stream, const void* src, void* dst, uint64_t groups,
                                   uint64_t src_stride_rows, uint64_t dst_stride_rows, uint64_t rows,
                                   uint64_t row_bytes);
cudaError_t launch_im2col_patch(cudaStream_t stream, const float* images, void* out, int code, uint32_t n,
                                uint32_t height, uint32_t width, uint32_t patch, uint32_t row_stride,
                                const float mean[3], const float inv_std[3]);
cudaError_t launch_cache_build(cudaStream_t stream, const void* a, const void* b, float* out, int code,
                               uint64_t rows, uint32_t ca, uint32_t cb);

// Epilogues of the block's linears (gemm_sm100.cu).
enum LinearEpilogue : int { kEpiNone = 0, kEpiGelu = 1, kEpiResidual = 2 };

// out (m, n) = x (m, k) . w (n, k)^T [+ bias] then the epilogue, 16-bit
// `elem` storage, f32 accumulation; k and n multiples of 8, 16-byte
// aligned rows.  kEpiResidual reads res (m, n) and gamma (n).
cudaError_t launch_linear_sm100(cudaStream_t stream, int elem, const void* x, const void* w, const float* bias,
                                void* out, uint64_t m, uint32_t k, uint32_t n, int epi, const void* res,
                                const float* gamma, int* status, uint64_t timeout_ns, std::string* err);

// The same op for f32 storage, f32 arithmetic on the CUDA cores (gemm_f32.cu):
// any m, k, n; m <= 65535 * 128.
cudaError_t launch_linear_f32(cudaStream_t stream, const float* x, const float* w, const float* bias, float* out,
                              uint64_t m, uint32_t k, uint32_t n, int epi, const float* res, const float* gamma);

// One tensor of a qk_prep launch: x (S, H, T, 64) in layout `lx` in, head-
// major rows out, with its own prologue.
struct PrepJob {
  const void* x = nullptr;
  RowLayout lx;
  void* out = nullptr;
  QkPrologue p;
};
constexpr int kMaxPrepJobs = 3;
struct PrepJobs {
  PrepJob job[kMaxPrepJobs];
};
// Up to kMaxPrepJobs tensors of the same shape and types in one launch.
// 16-bit rows in and out of the same type stream through shared memory by
// TMA (bounded waits: on a timeout a site code goes to `status`); f32 rows
// in or out take a register-only kernel.
cudaError_t launch_qk_prep(cudaStream_t stream, int in_code, int out_code, uint32_t S, uint32_t H, uint32_t t,
                           const PrepJob* jobs, int n_jobs, int* status, uint64_t timeout_ns);

// Reads x (S, H, T, 64) in layout `lx`, writes head-major 16-bit or f32
// rows.
cudaError_t launch_qk_prep(cudaStream_t stream, const void* x, int in_code, const RowLayout& lx, void* out,
                           int out_code, uint32_t S, uint32_t H, uint32_t t, const QkPrologue& p, int* status,
                           uint64_t timeout_ns);

// Companion ops of the reference engine.
cudaError_t launch_layernorm(cudaStream_t stream, const void* x, void* out, int code, const float* w,
                             const float* b, uint64_t rows, uint32_t dim, float eps);
cudaError_t launch_rope_apply(cudaStream_t stream, void* x, int code, const float* sin_t, const float* cos_t,
                              uint32_t s, uint32_t h, uint32_t t, uint32_t d, uint32_t prefix,
                              uint32_t tokens_per_frame);
cudaError_t launch_split_heads(cudaStream_t stream, const void* x, void* out, int code, uint32_t s, uint32_t t,
                               uint32_t h, uint32_t d);
cudaError_t launch_attn_merge(cudaStream_t stream, const void* x, void* out, int code, uint32_t s, uint32_t h,
                              uint32_t t, uint32_t d);

}  // namespace hs
