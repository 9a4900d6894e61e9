// Replacement fragments for headshot-server's engine (crates/headshot-server/src/engine/),
// written against this crate.  Each fragment names the reference lines it replaces; the
// rest of the engine keeps its call sites, since the op signatures do not change.
// (Only the new code is given here, not the reference's own lines.)

// ---- src/engine/tensor.rs:27-31 — GpuTensor storage -------------------------
//
// The wgpu buffer becomes a device allocation of the CUDA context; shape and dtype
// bookkeeping stay.  `Dtype` gains `Bf16` (the B200 path's 16-bit type besides f16).

pub struct GpuTensor {
    pub buffer: headshot_cuda::CudaTensor,
    pub shape: Vec<usize>,
    pub dtype: Dtype,
}

// ---- src/engine/tensor.rs:132-140 — GpuContext::empty_typed ----------------

impl GpuContext {
    pub fn empty_typed(&self, shape: &[usize], dtype: Dtype) -> GpuTensor {
        let buffer = self.cuda.empty(shape, dtype.into()).unwrap_or_else(|e| panic!("empty_typed: {e}"));
        GpuTensor { buffer, shape: shape.to_vec(), dtype }
    }
}

// ---- src/engine/ops.rs:225-253 — GpuContext::attention ----------------------
//
// Same contract: head-major (S, H, T, D) q, k, v; D = 64 (trunk, DINO) or 128 (camera
// head); out allocated here; scale 1/sqrt(D); a violated shape contract panics.  The
// dispatch that picked a WGSL entry point by (D, dtype) moves into the library
// (hs_attention: tcgen05 kernel for D = 64, f32 CUDA-core kernel for D = 128).

impl GpuContext {
    pub fn attention(&self, q: &GpuTensor, k: &GpuTensor, v: &GpuTensor) -> GpuTensor {
        let out = self.cuda.attention(&q.buffer, &k.buffer, &v.buffer);
        let shape = out.shape.clone();
        GpuTensor { buffer: out, shape, dtype: q.dtype }
    }
}

// ---- src/model/block.rs:136-148 — the block's QK-norm, RoPE and attention ----
//
// Three engine calls (layernorm on q and k, rope_apply on q and k, attention) become one:
// the library normalises and rotates Q and K once, bounds every score from the stored
// rows' norms and runs the attention kernel.  The reference's LayerNorm eps is fixed at
// 1e-5 (ops.rs:139), so that is what the block passes.

impl Block {
    fn attention_section(&self, ctx: &GpuContext, q: &GpuTensor, k: &GpuTensor, v: &GpuTensor,
                         rope: Option<&Rope<'_>>) -> GpuTensor {
        let norm = self.qk_norm.as_ref().map(|n| headshot_cuda::QkNorm {
            q_w: &n.q_w.buffer,
            q_b: &n.q_b.buffer,
            k_w: &n.k_w.buffer,
            k_b: &n.k_b.buffer,
            eps: 1e-5,
        });
        let rope = rope.map(|r| headshot_cuda::Rope {
            sin: &r.sin.buffer,
            cos: &r.cos.buffer,
            prefix: r.prefix,
            tokens_per_frame: 0,
        });
        let out = ctx.cuda.attention_fused(&q.buffer, &k.buffer, &v.buffer, norm.as_ref(), rope.as_ref());
        let shape = out.shape.clone();
        GpuTensor { buffer: out, shape, dtype: q.dtype }
    }
}

// ---- src/engine/mod.rs:111-211 — GpuContext::new -----------------------------
//
// The wgpu adapter/device/queue set-up becomes one CUDA context on the chosen device:
//
//     let cuda = headshot_cuda::Context::new(device_index)?;
//
// and `flush`/`sync` (mod.rs:261-284) become `cuda.sync()`, which also reports a kernel
// whose bounded wait gave up (Error::TIMEOUT) with the context still usable.
