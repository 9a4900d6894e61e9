//! Safe layer over libheadshot_cuda.so for headshot-server's engine.
//!
//! `Context` replaces the wgpu device behind `GpuContext` (src/engine/mod.rs)
//! and `CudaTensor` replaces `GpuTensor`'s `wgpu::Buffer` storage
//! (src/engine/tensor.rs:27-31): a device allocation from the context's
//! stream-ordered pool, with the same shape and dtype bookkeeping, freed on
//! drop after the work queued before the drop.  The ops keep the reference's
//! contract: shapes are asserted (a mismatch panics, as `assert!` does in
//! src/engine/ops.rs), every call is asynchronous on the context's stream and
//! `sync`/`download` report deferred device errors.
//!
//! Calls on one context are serialised by a lock inside `Context` (the
//! reference serialises inference with its engine's compute lock); the C
//! library keeps one stream per context.
//!
//! Not compiled in this repository's build container (it has no Rust
//! toolchain); tests/test_c_consumer.py checks `ffi.rs` against the header.

pub mod ffi;

use std::ffi::CStr;
use std::fmt;
use std::os::raw::{c_int, c_void};
use std::ptr;
use std::sync::{Arc, Mutex, MutexGuard};

/// Storage type of a tensor (src/engine/tensor.rs:13-16, plus bf16).
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum Dtype {
    F32,
    F16,
    Bf16,
}

impl Dtype {
    pub fn size(self) -> usize {
        match self {
            Dtype::F32 => 4,
            Dtype::F16 | Dtype::Bf16 => 2,
        }
    }

    fn code(self) -> ffi::hs_dtype {
        match self {
            Dtype::F32 => 0,
            Dtype::F16 => 1,
            Dtype::Bf16 => 2,
        }
    }
}

/// A non-OK `hs_status` with the library's message for it.
#[derive(Debug, Clone, PartialEq, Eq)]
pub struct Error {
    pub status: i32,
    pub message: String,
}

impl Error {
    pub const INVALID: i32 = 1;
    pub const UNSUPPORTED: i32 = 2;
    pub const CUDA: i32 = 3;
    pub const OOM: i32 = 4;
    pub const TIMEOUT: i32 = 5;
    pub const NCCL: i32 = 6;
    pub const CANCELLED: i32 = 7;
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "headshot_cuda status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

/// Message of the last failed call on this thread.
pub fn last_error() -> String {
    // SAFETY: the library returns a NUL-terminated thread-local string that
    // stays valid until the next failing call on this thread.
    unsafe { CStr::from_ptr(ffi::hs_last_error()).to_string_lossy().into_owned() }
}

fn check(status: ffi::hs_status) -> Result<(), Error> {
    if status == 0 { Ok(()) } else { Err(Error { status, message: last_error() }) }
}

/// Panics with the library's message, as the reference's ops panic on a
/// violated contract.
fn expect(status: ffi::hs_status, op: &str) {
    if let Err(e) = check(status) {
        panic!("{op}: {e}");
    }
}

struct RawCtx(*mut ffi::hs_ctx);
// SAFETY: the pointer is only used while holding `Inner::raw`'s lock.
unsafe impl Send for RawCtx {}

struct Inner {
    raw: Mutex<RawCtx>,
}

impl Drop for Inner {
    fn drop(&mut self) {
        let raw = self.raw.get_mut().map(|r| r.0).unwrap_or(ptr::null_mut());
        if !raw.is_null() {
            // SAFETY: last reference; every tensor holds an Arc to this context.
            unsafe { ffi::hs_ctx_destroy(raw) };
        }
    }
}

/// One device and its stream (GpuContext::new, src/engine/mod.rs:111-211).
#[derive(Clone)]
pub struct Context(Arc<Inner>);

/// QK-norm weights of a block (src/model/block.rs:35-40): f32 (64) tensors.
pub struct QkNorm<'a> {
    pub q_w: &'a CudaTensor,
    pub q_b: &'a CudaTensor,
    pub k_w: &'a CudaTensor,
    pub k_b: &'a CudaTensor,
    pub eps: f32,
}

/// 2D RoPE of a block (src/model/block.rs:42-47): f32 (rows, 64) tables.
pub struct Rope<'a> {
    pub sin: &'a CudaTensor,
    pub cos: &'a CudaTensor,
    pub prefix: usize,
    /// 0: the whole sequence is one frame (the reference's rope_apply).
    pub tokens_per_frame: usize,
}

impl Context {
    pub fn new(device: i32) -> Result<Self, Error> {
        let mut raw = ptr::null_mut();
        // SAFETY: `raw` is a valid out-pointer.
        check(unsafe { ffi::hs_ctx_create(device as c_int, &mut raw) })?;
        Ok(Context(Arc::new(Inner { raw: Mutex::new(RawCtx(raw)) })))
    }

    fn lock(&self) -> MutexGuard<'_, RawCtx> {
        self.0.raw.lock().unwrap_or_else(|p| p.into_inner())
    }

    /// Waits for the stream; `Error::TIMEOUT` if a kernel's bounded wait gave up.
    pub fn sync(&self) -> Result<(), Error> {
        let g = self.lock();
        check(unsafe { ffi::hs_sync(g.0) })
    }

    pub fn set_wait_timeout_ms(&self, ms: u32) -> Result<(), Error> {
        let g = self.lock();
        check(unsafe { ffi::hs_ctx_set_wait_timeout_ms(g.0, ms) })
    }

    /// Cooperative cancellation between steps (src/engine/mod.rs:92-106).
    pub fn request_cancel(&self) -> Result<(), Error> {
        let g = self.lock();
        check(unsafe { ffi::hs_ctx_request_cancel(g.0) })
    }

    pub fn clear_cancel(&self) -> Result<(), Error> {
        let g = self.lock();
        check(unsafe { ffi::hs_ctx_clear_cancel(g.0) })
    }

    /// empty_typed (src/engine/tensor.rs:132-140); the memory is not zero-filled.
    pub fn empty(&self, shape: &[usize], dtype: Dtype) -> Result<CudaTensor, Error> {
        let bytes = shape.iter().product::<usize>() * dtype.size();
        let mut p: *mut c_void = ptr::null_mut();
        let g = self.lock();
        check(unsafe { ffi::hs_alloc(g.0, bytes.max(1), &mut p) })?;
        Ok(CudaTensor { ptr: p, ctx: self.clone(), shape: shape.to_vec(), dtype })
    }

    /// Copies host bytes (already in the tensor's storage type) into `t`.
    pub fn upload(&self, t: &CudaTensor, bytes: &[u8]) -> Result<(), Error> {
        assert_eq!(bytes.len(), t.byte_len(), "upload size");
        let g = self.lock();
        check(unsafe { ffi::hs_memcpy_h2d(g.0, t.ptr, bytes.as_ptr().cast(), bytes.len()) })
    }

    /// download (src/engine/tensor.rs:163-198): the tensor's bytes, after its producers finished.
    pub fn download(&self, t: &CudaTensor) -> Result<Vec<u8>, Error> {
        let mut host = vec![0u8; t.byte_len()];
        let g = self.lock();
        check(unsafe { ffi::hs_memcpy_d2h(g.0, host.as_mut_ptr().cast(), t.ptr, host.len()) })?;
        check(unsafe { ffi::hs_sync(g.0) })?;
        Ok(host)
    }

    /// GpuContext::attention (src/engine/ops.rs:225-253): non-causal attention over
    /// head-major q, k, v (S, H, T, D), D = 64 or 128; softmax statistics in f32.
    pub fn attention(&self, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor) -> CudaTensor {
        let [s, h, t, d] = q.shape[..] else { panic!("attention wants (S,H,T,D)") };
        assert_eq!(q.shape, k.shape);
        assert_eq!(q.shape, v.shape);
        assert!(q.dtype == k.dtype && q.dtype == v.dtype, "attention: mixed dtypes");
        assert!(s * h <= 65535, "attention grid y overflow");
        let out = self.empty(&q.shape, q.dtype).unwrap_or_else(|e| panic!("attention: {e}"));
        let g = self.lock();
        expect(
            unsafe {
                ffi::hs_attention(g.0, q.ptr, k.ptr, v.ptr, out.ptr, s as u32, h as u32, t as u32, d as u32,
                                  q.dtype.code(), 0.0)
            },
            "attention",
        );
        out
    }

    /// Block::forward's QK-norm -> RoPE -> attention (src/model/block.rs:136-148) as one op.
    pub fn attention_fused(&self, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor, qk_norm: Option<&QkNorm<'_>>,
                           rope: Option<&Rope<'_>>) -> CudaTensor {
        let [s, h, t, d] = q.shape[..] else { panic!("attention wants (S,H,T,D)") };
        assert_eq!(q.shape, k.shape);
        assert_eq!(q.shape, v.shape);
        let out = self.empty(&q.shape, q.dtype).unwrap_or_else(|e| panic!("attention_fused: {e}"));
        let null = ptr::null::<f32>();
        let (qw, qb, kw, kb, eps) = match qk_norm {
            Some(n) => (n.q_w.f32_ptr(), n.q_b.f32_ptr(), n.k_w.f32_ptr(), n.k_b.f32_ptr(), n.eps),
            None => (null, null, null, null, 1e-5),
        };
        let (sin, cos, rows, prefix, tpf) = match rope {
            Some(r) => (r.sin.f32_ptr(), r.cos.f32_ptr(), r.sin.len() / 64, r.prefix, r.tokens_per_frame),
            None => (null, null, 0, 0, 0),
        };
        let g = self.lock();
        expect(
            unsafe {
                ffi::hs_attention_fused(g.0, q.ptr, k.ptr, v.ptr, out.ptr, s as u32, h as u32, t as u32, d as u32,
                                        q.dtype.code(), 0.0, qw, qb, kw, kb, eps, sin, cos, rows as u32,
                                        prefix as u32, tpf as u32)
            },
            "attention_fused",
        );
        out
    }

    /// GpuContext::layernorm (src/engine/ops.rs:130-153) with eps an argument.
    pub fn layernorm(&self, x: &CudaTensor, w: &CudaTensor, b: &CudaTensor, eps: f32) -> CudaTensor {
        let dim = *x.shape.last().expect("layernorm wants a shape");
        assert_eq!(w.len(), dim);
        assert_eq!(b.len(), dim);
        assert_eq!(w.dtype, Dtype::F32, "norm weight must be f32");
        assert_eq!(b.dtype, Dtype::F32, "norm bias must be f32");
        let out = self.empty(&x.shape, x.dtype).unwrap_or_else(|e| panic!("layernorm: {e}"));
        let g = self.lock();
        expect(
            unsafe {
                ffi::hs_layernorm(g.0, x.ptr, w.f32_ptr(), b.f32_ptr(), out.ptr, (x.len() / dim) as u64, dim as u32,
                                  eps, x.dtype.code())
            },
            "layernorm",
        );
        out
    }

    /// GpuContext::rope_apply (src/engine/ops.rs:202-223), in place.
    pub fn rope_apply(&self, x: &CudaTensor, sin: &CudaTensor, cos: &CudaTensor, prefix: usize) {
        let [s, h, t, d] = x.shape[..] else { panic!("rope_apply wants (S,H,T,D)") };
        assert_eq!(sin.len(), (t - prefix) * d, "table size");
        assert_eq!(sin.dtype, Dtype::F32, "rope tables must be f32");
        assert_eq!(cos.dtype, Dtype::F32, "rope tables must be f32");
        let g = self.lock();
        expect(
            unsafe {
                ffi::hs_rope_apply(g.0, x.ptr, sin.f32_ptr(), cos.f32_ptr(), (t - prefix) as u32, s as u32, h as u32,
                                   t as u32, d as u32, prefix as u32, x.dtype.code())
            },
            "rope_apply",
        );
    }
}

/// A device tensor: pool allocation + shape + dtype (GpuTensor, src/engine/tensor.rs:27-31).
pub struct CudaTensor {
    ptr: *mut c_void,
    ctx: Context,
    pub shape: Vec<usize>,
    pub dtype: Dtype,
}

// SAFETY: the allocation belongs to the context, whose calls are serialised by its lock.
unsafe impl Send for CudaTensor {}
unsafe impl Sync for CudaTensor {}

impl CudaTensor {
    pub fn len(&self) -> usize {
        self.shape.iter().product()
    }

    pub fn is_empty(&self) -> bool {
        self.len() == 0
    }

    pub fn byte_len(&self) -> usize {
        self.len() * self.dtype.size()
    }

    /// Device address (for the engine's own kernels on the context's stream).
    pub fn as_ptr(&self) -> *const c_void {
        self.ptr
    }

    fn f32_ptr(&self) -> *const f32 {
        assert_eq!(self.dtype, Dtype::F32);
        self.ptr as *const f32
    }

    /// Reinterpret the shape (same element count), as GpuTensor::reshaped.
    pub fn reshaped(mut self, shape: &[usize]) -> Self {
        assert_eq!(self.len(), shape.iter().product::<usize>(), "reshape element count");
        self.shape = shape.to_vec();
        self
    }
}

impl Drop for CudaTensor {
    fn drop(&mut self) {
        let g = self.ctx.lock();
        // SAFETY: stream-ordered free, after the work already queued that uses the tensor.
        unsafe { ffi::hs_free(g.0, self.ptr) };
    }
}

/// One rank of the multi-GPU ring (global attention over NCCL; one process per GPU).
/// hs_ring_attention_fused and hs_ring_ulysses_attention_fused share one signature.
type GlobalFn = unsafe extern "C" fn(*mut ffi::hs_ring, *const c_void, *const c_void, *const c_void, *mut c_void, u32,
                                     u32, u32, ffi::hs_dtype, f32, *const f32, *const f32, *const f32, *const f32,
                                     f32, *const f32, *const f32, u32, u32, u32) -> ffi::hs_status;

pub struct Ring {
    raw: *mut ffi::hs_ring,
    ctx: Context,
}

unsafe impl Send for Ring {}

impl Ring {
    /// Rank 0 creates the id and shares its bytes with the other ranks out of band.
    pub fn unique_id() -> Result<Vec<u8>, Error> {
        let mut id = vec![0u8; unsafe { ffi::hs_ring_id_bytes() }];
        check(unsafe { ffi::hs_ring_unique_id(id.as_mut_ptr().cast()) })?;
        Ok(id)
    }

    /// Collective over all ranks.
    pub fn new(ctx: &Context, rank: i32, world: i32, id: &[u8]) -> Result<Self, Error> {
        assert_eq!(id.len(), unsafe { ffi::hs_ring_id_bytes() }, "ring id size");
        let mut raw = ptr::null_mut();
        let g = ctx.lock();
        check(unsafe { ffi::hs_ring_create(g.0, rank, world, id.as_ptr().cast(), &mut raw) })?;
        drop(g);
        Ok(Ring { raw, ctx: ctx.clone() })
    }

    /// SMs the attention launches leave to the block transfers (default 0).
    pub fn set_reserved_sms(&self, sms: u32) -> Result<(), Error> {
        check(unsafe { ffi::hs_ring_set_reserved_sms(self.raw, sms) })
    }

    /// Global attention over this rank's shard (S = 1): q, k, v, out (H, T_r, 64), by the K/V ring.
    pub fn attention_fused(&self, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor, out: &CudaTensor, t_total: usize,
                           qk_norm: Option<&QkNorm<'_>>, rope: Option<&Rope<'_>>) -> Result<(), Error> {
        self.global(ffi::hs_ring_attention_fused, q, k, v, out, t_total, qk_norm, rope)
    }

    /// The same contract by head parallelism: an all-to-all gathers the whole sequence of
    /// H / world heads on each rank, one attention launch, an all-to-all back (H a multiple of world).
    pub fn attention_ulysses(&self, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor, out: &CudaTensor,
                             t_total: usize, qk_norm: Option<&QkNorm<'_>>, rope: Option<&Rope<'_>>)
                             -> Result<(), Error> {
        self.global(ffi::hs_ring_ulysses_attention_fused, q, k, v, out, t_total, qk_norm, rope)
    }

    fn global(&self, call: GlobalFn, q: &CudaTensor, k: &CudaTensor, v: &CudaTensor, out: &CudaTensor,
              t_total: usize, qk_norm: Option<&QkNorm<'_>>, rope: Option<&Rope<'_>>) -> Result<(), Error> {
        let h = q.shape[q.shape.len() - 3];
        let null = ptr::null::<f32>();
        let (qw, qb, kw, kb, eps) = match qk_norm {
            Some(n) => (n.q_w.f32_ptr(), n.q_b.f32_ptr(), n.k_w.f32_ptr(), n.k_b.f32_ptr(), n.eps),
            None => (null, null, null, null, 1e-5),
        };
        let (sin, cos, rows, prefix, tpf) = match rope {
            Some(r) => (r.sin.f32_ptr(), r.cos.f32_ptr(), r.sin.len() / 64, r.prefix, r.tokens_per_frame),
            None => (null, null, 0, 0, 0),
        };
        let _g = self.ctx.lock();
        check(unsafe {
            call(self.raw, q.ptr, k.ptr, v.ptr, out.ptr, h as u32, t_total as u32, 64, q.dtype.code(), 0.0, qw, qb, kw,
                 kb, eps, sin, cos, rows as u32, prefix as u32, tpf as u32)
        })
    }

    /// Waits with the library's watchdog; on a timeout or NCCL error the ring is aborted.
    pub fn sync(&self, timeout_ms: u32) -> Result<(), Error> {
        let _g = self.ctx.lock();
        check(unsafe { ffi::hs_ring_sync(self.raw, timeout_ms) })
    }
}

impl Drop for Ring {
    fn drop(&mut self) {
        let _g = self.ctx.lock();
        unsafe { ffi::hs_ring_destroy(self.raw) };
    }
}

/// rope::tables (src/engine/rope.rs:15-44) on the host: (sin, cos), each h_p*w_p rows of 64.
pub fn rope_tables(h_p: u32, w_p: u32) -> Result<(Vec<f32>, Vec<f32>), Error> {
    let n = (h_p * w_p) as usize * 64;
    let (mut sin, mut cos) = (vec![0f32; n], vec![0f32; n]);
    check(unsafe { ffi::hs_rope_tables(ptr::null(), h_p, w_p, sin.as_mut_ptr(), cos.as_mut_ptr()) })?;
    Ok((sin, cos))
}

/// The library's ABI version (HS_ABI_VERSION).
pub fn abi_version() -> u32 {
    unsafe { ffi::hs_abi_version() }
}
