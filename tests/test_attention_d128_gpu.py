"""The camera head's head_dim-128 attention (GpuContext::attention's
"attention_d128" variant, src/engine/ops.rs:233-237; used by
src/model/camera_head.rs:68-72 over one sequence of N*17 prefix tokens)
against the oracle's restatement of attention.wesl at DV = 32.

f32 storage computes in f32, so the gate is the reference's own attention
tolerance (kernels.rs:184-239: |diff| < 1e-4); 16-bit storage uses the
north-star gate on inputs rounded to the storage type."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from headshot_b200._lib import HsError
from headshot_b200.engine import QkNorm

pytestmark = pytest.mark.gpu
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(TORCH[dtype])


def host(t):
    return t.float().cpu().numpy()


def inputs(s, h, t, dtype, seed):
    vals = oracle.rng_uniform(seed, 3 * s * h * t * 128)
    n = s * h * t * 128
    q, k, v = (vals[i * n:(i + 1) * n].reshape(s, h, t, 128) for i in range(3))
    if dtype != "f32":
        q, k, v = (oracle.round_to(dtype, x) for x in (q, k, v))
    return q, k, v


@pytest.mark.parametrize("s,h,t", [(2, 3, 17), (2, 3, 64), (2, 3, 150), (1, 16, 1700), (1, 2, 33), (3, 1, 1)])
def test_d128_f32_within_reference_tolerance(gpu_ctx, s, h, t):
    q, k, v = inputs(s, h, t, "f32", 5 + t)
    out = gpu_ctx.attention(dev(q, "f32"), dev(k, "f32"), dev(v, "f32"))
    ref = oracle.attention(q, k, v)
    gpu_ctx.sync()
    assert np.abs(host(out) - ref).max() < 1e-4


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_d128_16bit_storage(gpu_ctx, dtype):
    q, k, v = inputs(1, 4, 700, dtype, 9)
    out = gpu_ctx.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype))
    ref = oracle.attention(q, k, v)
    gpu_ctx.sync()
    oracle.gate(oracle.compare(host(out), ref), 0.9999, 1e-2)


def test_d128_block_layout(gpu_ctx):
    """Camera-head Block::forward shape: dim 2048 = 16 heads x 128, projection layout in,
    merged layout out (split_heads -> attention -> attn_merge in one call)."""
    s, t, h = 1, 3 * 17, 16
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((s * t, h * 128)).astype(np.float32) for _ in range(3))
    out = gpu_ctx.attention_block(dev(q, "f32"), dev(k, "f32"), dev(v, "f32"), s, t, h)
    sp = [oracle.split_heads(x, s, t, h, 128) for x in (q, k, v)]
    ref = oracle.attn_merge(oracle.attention(*sp))
    gpu_ctx.sync()
    assert np.abs(host(out) - ref).max() < 1e-4


def test_d128_rejects_prologue(gpu_ctx):
    q = torch.zeros((1, 1, 8, 128), device="cuda")
    w = torch.ones(128, device="cuda")
    b = torch.zeros(128, device="cuda")
    with pytest.raises(HsError):
        gpu_ctx.attention_fused(q, q, q, qk_norm=QkNorm(w, b, w, b))
