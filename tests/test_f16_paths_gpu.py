"""The reference's f16-versus-f32 known-answer tests, restated for this library's ops.

- tests/kernels.rs:376-401 (`attention_f16_matches_f32`): Rng(9), (S, H, T, D) = (1, 2, 33,
  64); the f16 path on f16-rounded inputs must land within 5e-3 (abs + rel, kernels.rs:35-43)
  of f32 attention on the unrounded inputs (here the oracle's restatement of attention.wesl).
- tests/f16_ops.rs:35-109 (`every_op_f16_matches_f32`): (S, H, T, D) = (2, 4, 21, 64) with
  values every storage type holds exactly (f16_ops.rs:7-19's own generator); each op's f16
  result against its f32 result: LayerNorm within 2e-2, RoPE (4x4 grid, prefix T - 16) within
  2e-3, split_heads / attn_merge exact (max difference below 1e-6).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

S, H, T, D = 2, 4, 21, 64


def _dev(a: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(dtype)


def _host(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def _max_diff(a: np.ndarray, b: np.ndarray) -> float:
    """f16_ops.rs:21-33: the max absolute difference, with neither side all zero."""
    assert np.count_nonzero(b) > 0, "f32 result is all zero"
    assert np.count_nonzero(a) > 0, "f16 result is all zero"
    return float(np.abs(a - b).max())


def test_attention_f16_matches_f32(gpu_ctx):
    s, h, t, d = 1, 2, 33, 64
    n = s * h * t * d
    vals = oracle.rng_uniform(9, 3 * n)  # one Rng(9) stream: q, then k, then v
    q, k, v = (vals[i * n:(i + 1) * n].reshape(s, h, t, d) for i in range(3))
    want = oracle.attention(q, k, v)
    got = gpu_ctx.attention(_dev(q, torch.float16), _dev(k, torch.float16), _dev(v, torch.float16))
    gpu_ctx.sync()
    tol = 5e-3
    excess = np.abs(_host(got) - want) - (tol + tol * np.abs(want))
    assert excess.max() <= 0, f"max excess {excess.max():.3g}"


def test_layernorm_f16_matches_f32(gpu_ctx):
    rows, c = S * T, H * D
    x = oracle.rng_f16_exact(1, rows * c).reshape(rows, c)
    w = torch.from_numpy(oracle.rng_f16_exact(2, c)).cuda()
    b = torch.from_numpy(oracle.rng_f16_exact(3, c)).cuda()
    f32 = gpu_ctx.layernorm(_dev(x, torch.float32), w, b)  # eps 1e-5, ops.rs:139
    f16 = gpu_ctx.layernorm(_dev(x, torch.float16), w, b)
    gpu_ctx.sync()
    assert _max_diff(_host(f16), _host(f32)) < 2e-2
    assert np.abs(_host(f32) - oracle.layernorm(x, _host(w), _host(b), 1e-5)).max() < 1e-4


def test_rope_apply_f16_matches_f32(gpu_ctx):
    sin, cos = oracle.rope_tables(4, 4)  # 16 rows: prefix = T - 16
    prefix = T - 16
    x = oracle.rng_f16_exact(7, S * H * T * D).reshape(S, H, T, D)
    g32, g16 = _dev(x, torch.float32), _dev(x, torch.float16)
    sin_d, cos_d = torch.from_numpy(sin).cuda(), torch.from_numpy(cos).cuda()
    gpu_ctx.rope_apply(g32, sin_d, cos_d, prefix)
    gpu_ctx.rope_apply(g16, sin_d, cos_d, prefix)
    gpu_ctx.sync()
    assert _max_diff(_host(g16), _host(g32)) < 2e-3
    assert np.abs(_host(g32) - oracle.rope_apply(x, sin, cos, prefix)).max() < 1e-5


def test_split_merge_f16_matches_f32(gpu_ctx):
    rows, c = S * T, H * D
    qkv = oracle.rng_f16_exact(6, rows * c).reshape(rows, c)
    q32 = gpu_ctx.split_heads(_dev(qkv, torch.float32), S, T, H, D)
    q16 = gpu_ctx.split_heads(_dev(qkv, torch.float16), S, T, H, D)
    m32, m16 = gpu_ctx.attn_merge(q32), gpu_ctx.attn_merge(q16)
    gpu_ctx.sync()
    assert _max_diff(_host(q16), _host(q32)) < 1e-6
    assert _max_diff(_host(m16), _host(m32)) < 1e-6
    np.testing.assert_array_equal(_host(q32), oracle.split_heads(qkv, S, T, H, D))
