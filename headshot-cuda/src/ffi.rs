//! Raw bindings of libheadshot_cuda.so: one declaration per entry point of
//! include/headshot_cuda.h, same order, same C types (`uint32_t` -> `u32`,
//! `const T*` -> `*const T`, `void*` -> `*mut c_void`, enums -> `c_int`).
//! tests/test_c_consumer.py parses this file and checks every declaration
//! against the header, so the binding cannot drift from the C ABI.
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub type hs_status = c_int;            // HS_OK = 0, HS_ERR_INVALID = 1, ... HS_ERR_CANCELLED = 7
pub type hs_dtype = c_int;             // HS_F32 = 0, HS_F16 = 1, HS_BF16 = 2
#[repr(C)] pub struct hs_ctx { _p: [u8; 0] }
#[repr(C)] pub struct hs_ring { _p: [u8; 0] }

#[link(name = "headshot_cuda")]
unsafe extern "C" {
    // context
    pub fn hs_abi_version() -> u32;
    pub fn hs_last_error() -> *const c_char;
    pub fn hs_ctx_create(device: c_int, out: *mut *mut hs_ctx) -> hs_status;
    pub fn hs_ctx_destroy(ctx: *mut hs_ctx) -> hs_status;
    pub fn hs_ctx_set_stream(ctx: *mut hs_ctx, stream: *mut c_void) -> hs_status;
    pub fn hs_ctx_use_own_stream(ctx: *mut hs_ctx) -> hs_status;
    pub fn hs_ctx_stream(ctx: *mut hs_ctx) -> *mut c_void;
    pub fn hs_ctx_set_wait_timeout_ms(ctx: *mut hs_ctx, ms: u32) -> hs_status;
    pub fn hs_ctx_request_cancel(ctx: *mut hs_ctx) -> hs_status;
    pub fn hs_ctx_clear_cancel(ctx: *mut hs_ctx) -> hs_status;
    pub fn hs_prof_enable(ctx: *mut hs_ctx, on: c_int) -> hs_status;
    pub fn hs_prof_reset(ctx: *mut hs_ctx) -> hs_status;
    pub fn hs_prof_read(ctx: *mut hs_ctx, kernel: *const c_char, total_ms: *mut f64,
                        launches: *mut u64) -> hs_status;
    // memory
    pub fn hs_alloc(ctx: *mut hs_ctx, bytes: usize, out: *mut *mut c_void) -> hs_status;
    pub fn hs_free(ctx: *mut hs_ctx, ptr: *mut c_void) -> hs_status;
    pub fn hs_memset(ctx: *mut hs_ctx, dst: *mut c_void, value: c_int, bytes: usize) -> hs_status;
    pub fn hs_memcpy_h2d(ctx: *mut hs_ctx, dst_device: *mut c_void, src_host: *const c_void,
                         bytes: usize) -> hs_status;
    pub fn hs_memcpy_d2h(ctx: *mut hs_ctx, dst_host: *mut c_void, src_device: *const c_void,
                         bytes: usize) -> hs_status;
    pub fn hs_sync(ctx: *mut hs_ctx) -> hs_status;
    // ops
    pub fn hs_attention(ctx: *mut hs_ctx, q: *const c_void, k: *const c_void, v: *const c_void,
                        out: *mut c_void, s: u32, h: u32, t: u32, d: u32, dtype: hs_dtype,
                        scale: f32) -> hs_status;
    pub fn hs_attention_fused(ctx: *mut hs_ctx, q: *const c_void, k: *const c_void, v: *const c_void,
                              out: *mut c_void, s: u32, h: u32, t: u32, d: u32, dtype: hs_dtype, scale: f32,
                              q_norm_w: *const f32, q_norm_b: *const f32, k_norm_w: *const f32,
                              k_norm_b: *const f32, eps: f32, rope_sin: *const f32, rope_cos: *const f32,
                              rope_rows: u32, prefix: u32, tokens_per_frame: u32) -> hs_status;
    pub fn hs_attention_block_fused(ctx: *mut hs_ctx, q: *const c_void, k: *const c_void, v: *const c_void,
                                    out: *mut c_void, s: u32, t: u32, h: u32, d: u32, dtype: hs_dtype,
                                    scale: f32, q_norm_w: *const f32, q_norm_b: *const f32,
                                    k_norm_w: *const f32, k_norm_b: *const f32, eps: f32,
                                    rope_sin: *const f32, rope_cos: *const f32, rope_rows: u32, prefix: u32,
                                    tokens_per_frame: u32) -> hs_status;
    pub fn hs_attention_fused_noalloc(stream: *mut c_void, status: *mut c_int, q: *const c_void,
                                      k: *const c_void, v: *const c_void, out: *mut c_void, s: u32, h: u32,
                                      t: u32, d: u32, dtype: hs_dtype, scale: f32, q_norm_w: *const f32,
                                      q_norm_b: *const f32, k_norm_w: *const f32, k_norm_b: *const f32,
                                      eps: f32, rope_sin: *const f32, rope_cos: *const f32, rope_rows: u32,
                                      prefix: u32, tokens_per_frame: u32) -> hs_status;
    pub fn hs_linear(ctx: *mut hs_ctx, x: *const c_void, w: *const c_void, bias: *const f32, out: *mut c_void,
                     m: u64, k: u32, n: u32, dtype: hs_dtype, epilogue: c_int, residual: *const c_void,
                     gamma: *const f32) -> hs_status;
    pub fn hs_layernorm(ctx: *mut hs_ctx, x: *const c_void, w: *const f32, b: *const f32, out: *mut c_void,
                        rows: u64, dim: u32, eps: f32, dtype: hs_dtype) -> hs_status;
    pub fn hs_rope_apply(ctx: *mut hs_ctx, x: *mut c_void, rope_sin: *const f32, rope_cos: *const f32,
                         rope_rows: u32, s: u32, h: u32, t: u32, d: u32, prefix: u32,
                         dtype: hs_dtype) -> hs_status;
    pub fn hs_split_heads(ctx: *mut hs_ctx, x: *const c_void, out: *mut c_void, s: u32, t: u32, h: u32,
                          d: u32, dtype: hs_dtype) -> hs_status;
    pub fn hs_attn_merge(ctx: *mut hs_ctx, x: *const c_void, out: *mut c_void, s: u32, h: u32, t: u32, d: u32,
                         dtype: hs_dtype) -> hs_status;
    // multi-GPU session (ring)
    pub fn hs_ring_shard(n: u32, world: c_int, rank: c_int, start: *mut u32, len: *mut u32) -> hs_status;
    pub fn hs_ring_plan(rank: c_int, world: c_int, step: c_int, src_block: *mut c_int, send_to: *mut c_int,
                        recv_from: *mut c_int, load_state: *mut c_int, store_state: *mut c_int) -> hs_status;
    pub fn hs_ring_id_bytes() -> usize;
    pub fn hs_ring_unique_id(id_out: *mut c_void) -> hs_status;
    pub fn hs_ring_create(ctx: *mut hs_ctx, rank: c_int, world: c_int, id: *const c_void,
                          out: *mut *mut hs_ring) -> hs_status;
    pub fn hs_ring_destroy(ring: *mut hs_ring) -> hs_status;
    pub fn hs_ring_attention_fused(ring: *mut hs_ring, q: *const c_void, k: *const c_void, v: *const c_void,
                                   out: *mut c_void, h: u32, t_total: u32, d: u32, dtype: hs_dtype,
                                   scale: f32, q_norm_w: *const f32, q_norm_b: *const f32,
                                   k_norm_w: *const f32, k_norm_b: *const f32, eps: f32, rope_sin: *const f32,
                                   rope_cos: *const f32, rope_rows: u32, prefix: u32,
                                   tokens_per_frame: u32) -> hs_status;
    pub fn hs_ring_attention_block_fused(ring: *mut hs_ring, q: *const c_void, k: *const c_void,
                                         v: *const c_void, out: *mut c_void, h: u32, t_total: u32, d: u32,
                                         dtype: hs_dtype, scale: f32, q_norm_w: *const f32,
                                         q_norm_b: *const f32, k_norm_w: *const f32, k_norm_b: *const f32,
                                         eps: f32, rope_sin: *const f32, rope_cos: *const f32, rope_rows: u32,
                                         prefix: u32, tokens_per_frame: u32, shard_unit: u32) -> hs_status;
    pub fn hs_ring_ulysses_attention_fused(ring: *mut hs_ring, q: *const c_void, k: *const c_void,
                                           v: *const c_void, out: *mut c_void, h: u32, t_total: u32, d: u32,
                                           dtype: hs_dtype, scale: f32, q_norm_w: *const f32,
                                           q_norm_b: *const f32, k_norm_w: *const f32, k_norm_b: *const f32,
                                           eps: f32, rope_sin: *const f32, rope_cos: *const f32,
                                           rope_rows: u32, prefix: u32, tokens_per_frame: u32) -> hs_status;
    pub fn hs_ring_set_reserved_sms(ring: *mut hs_ring, sms: u32) -> hs_status;
    pub fn hs_ring_sync(ring: *mut hs_ring, timeout_ms: u32) -> hs_status;
    // trunk glue and host helpers
    pub fn hs_copy_row_blocks(ctx: *mut hs_ctx, src: *const c_void, dst: *mut c_void, groups: u64,
                              src_stride_rows: u64, dst_stride_rows: u64, rows: u64, cols: u32,
                              dtype: hs_dtype) -> hs_status;
    pub fn hs_im2col_patch(ctx: *mut hs_ctx, images: *const f32, out: *mut c_void, n: u32, height: u32,
                           width: u32, patch: u32, row_stride: u32, mean: *const f32, std_dev: *const f32,
                           dtype: hs_dtype) -> hs_status;
    pub fn hs_cache_build(ctx: *mut hs_ctx, frame_out: *const c_void, global_out: *const c_void, out: *mut f32,
                          rows: u64, cols_frame: u32, cols_global: u32, dtype: hs_dtype) -> hs_status;
    pub fn hs_rope_periods(out16: *mut f32) -> hs_status;
    pub fn hs_rope_tables(periods: *const f32, h_p: u32, w_p: u32, sin_out: *mut f32,
                          cos_out: *mut f32) -> hs_status;
}
