"""Trunk glue on the GPU, bit-exact against the oracle: the register-layer
gather and scatter of the 17 prefix tokens per frame (src/model/trunk.rs:
105-122, GpuContext::copy_rows) and the f32 head-input cache build
(src/model/cache.rs:25-52: concat_channels + cast_to_f32)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from headshot_b200 import _lib
from headshot_b200.engine import GpuContext

pytestmark = pytest.mark.gpu
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(TORCH[dtype])


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_register_gather_scatter(gpu_ctx: GpuContext, dtype):
    n, t, prefix, c = 7, 1374, 17, 1024
    rng = np.random.default_rng(3)
    x = oracle.round_to(dtype, rng.standard_normal((n * t, c)).astype(np.float32)) if dtype != "f32" else \
        rng.standard_normal((n * t, c)).astype(np.float32)
    xd = dev(x, dtype)
    reg = gpu_ctx.gather_prefix(xd, n, t, prefix)
    exp = oracle.copy_row_blocks(x, np.zeros((n * prefix, c), np.float32), n, t, prefix, prefix)
    gpu_ctx.sync()
    assert np.array_equal(reg.float().cpu().numpy(), exp)
    # scatter a transformed copy back: prefix rows change, patch rows must not
    new = rng.standard_normal((n * prefix, c)).astype(np.float32)
    new = oracle.round_to(dtype, new) if dtype != "f32" else new
    gpu_ctx.scatter_prefix(dev(new, dtype), xd, n, t, prefix)
    exp_x = oracle.copy_row_blocks(new, x.copy(), n, prefix, t, prefix)
    gpu_ctx.sync()
    assert np.array_equal(xd.float().cpu().numpy(), exp_x)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_cache_build(gpu_ctx, dtype):
    rows, c = 3 * 1374, 1024
    rng = np.random.default_rng(4)
    a, b = (rng.standard_normal((rows, c)).astype(np.float32) for _ in range(2))
    if dtype != "f32":
        a, b = oracle.round_to(dtype, a), oracle.round_to(dtype, b)
    out = gpu_ctx.cache_build(dev(a, dtype), dev(b, dtype))
    gpu_ctx.sync()
    assert out.dtype == torch.float32 and out.shape == (rows, 2 * c)
    assert np.array_equal(out.cpu().numpy(), oracle.cache_build(a, b))


def test_glue_rejects_bad_shapes(gpu_ctx):
    x = torch.zeros((10, 12), device="cuda", dtype=torch.float16)  # 24-byte rows
    with pytest.raises(_lib.HsError):
        gpu_ctx.copy_row_blocks(x, torch.zeros_like(x), 1, 0, 0, 10)
