"""The block's linears (hs_linear: tcgen05 for f16/bf16, f32 on the CUDA cores)
against the CPU oracle.

Restated cases from the reference's own tests (tests/kernels.rs:313-374,
linear_f16_and_wmma_match_cpu: f16-rounded inputs, f64 sums, f16 output,
abs+rel tolerance as kernels.rs:35-43) and the trunk's shapes (d = 1024,
MLP 4096) with each fused epilogue: GELU (gelu.wesl) and the LayerScale
residual (residual_ls.wesl).  The reference rounds the linear's output to
the storage type before those element-wise kernels; the fused epilogue does
not, so the gate compares against the oracle on the unrounded sum with the
storage type's rounding as tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from headshot_b200 import _lib
from headshot_b200.engine import GpuContext

pytestmark = pytest.mark.gpu

TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(TORCH[dtype])


def close(got, exp, tol):
    err = np.abs(got - exp) - (tol + tol * np.abs(exp))
    assert np.all(err <= 0), f"max excess {err.max():.3g} at {np.unravel_index(np.argmax(err), err.shape)}"


def test_linear_reference_f16_case(gpu_ctx: GpuContext):
    # kernels.rs:313-374: Rng(8), (m, k, n) = (37, 96, 128) with bias, tol 1e-2;
    # the same x against the first 48 rows of w without bias, tol 2e-3.
    m, k, n = 37, 96, 128
    vals = oracle.rng_uniform(8, m * k + n * k + n)
    x = oracle.round_to("f16", vals[:m * k].reshape(m, k))
    w = oracle.round_to("f16", vals[m * k:m * k + n * k].reshape(n, k))
    b = vals[m * k + n * k:]
    exp = oracle.round_to("f16", (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32) + b)
    out = gpu_ctx.linear(dev(x, "f16"), dev(w, "f16"), torch.from_numpy(b).cuda())
    gpu_ctx.sync()
    close(out.float().cpu().numpy(), exp, 1e-2)
    n2 = 48
    exp2 = oracle.round_to("f16", (x.astype(np.float64) @ w[:n2].astype(np.float64).T).astype(np.float32))
    out2 = gpu_ctx.linear(dev(x, "f16"), dev(w[:n2], "f16"))
    gpu_ctx.sync()
    close(out2.float().cpu().numpy(), exp2, 2e-3)


def _case(dtype, m, k, n, seed):
    rng = np.random.default_rng(seed)
    x = oracle.round_to(dtype, rng.standard_normal((m, k)).astype(np.float32))
    w = oracle.round_to(dtype, (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32))
    b = (0.1 * rng.standard_normal(n)).astype(np.float32)
    return x, w, b


def _tol(dtype):
    return 8e-3 if dtype == "bf16" else 1e-3  # about one rounding of the 16-bit output


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("m,k,n", [(300, 1024, 1024), (1374, 1024, 4096), (517, 4096, 1024), (130, 64, 1000),
                                   (5, 8, 8)])
def test_linear_plain(gpu_ctx, dtype, m, k, n):
    x, w, b = _case(dtype, m, k, n, m + k + n)
    ref = oracle.linear(x, w, b)
    out = gpu_ctx.linear(dev(x, dtype), dev(w, dtype), torch.from_numpy(b).cuda())
    gpu_ctx.sync()
    close(out.float().cpu().numpy(), ref, _tol(dtype))


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_linear_gelu_epilogue(gpu_ctx, dtype):
    m, k, n = 700, 1024, 4096  # MLP fc1 shape
    x, w, b = _case(dtype, m, k, n, 11)
    ref = oracle.gelu(oracle.linear(x, w, b))
    out = gpu_ctx.linear(dev(x, dtype), dev(w, dtype), torch.from_numpy(b).cuda(), epilogue="gelu")
    gpu_ctx.sync()
    close(out.float().cpu().numpy(), ref, _tol(dtype))


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("inplace", [False, True])
def test_linear_residual_ls_epilogue(gpu_ctx, dtype, inplace):
    m, k, n = 700, 4096, 1024  # MLP fc2 shape; proj is k = 1024
    x, w, b = _case(dtype, m, k, n, 12)
    rng = np.random.default_rng(13)
    res = oracle.round_to(dtype, rng.standard_normal((m, n)).astype(np.float32))
    gamma = (0.5 * rng.standard_normal(n)).astype(np.float32)
    ref = oracle.residual_ls(res, oracle.linear(x, w, b), gamma)
    res_d = dev(res, dtype)
    out = gpu_ctx.linear(dev(x, dtype), dev(w, dtype), torch.from_numpy(b).cuda(), epilogue="residual_ls",
                         residual=res_d, gamma=torch.from_numpy(gamma).cuda(), out=res_d if inplace else None)
    gpu_ctx.sync()
    close(out.float().cpu().numpy(), ref, _tol(dtype))


def test_linear_reference_f32_case(gpu_ctx):
    """kernels.rs:63-100 (linear_matches_cpu): Rng(2), (m, k, n) = (37, 53, 29), f32, against
    f64 sums with and without bias, tolerance 1e-4 (abs + rel, kernels.rs:35-43)."""
    m, k, n = 37, 53, 29
    vals = oracle.rng_uniform(2, m * k + n * k + n)
    x = vals[:m * k].reshape(m, k)
    w = vals[m * k:m * k + n * k].reshape(n, k)
    b = vals[m * k + n * k:]
    exp = (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32) + b
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = gpu_ctx.linear(xd, wd, torch.from_numpy(b).cuda())
    out_nb = gpu_ctx.linear(xd, wd)
    gpu_ctx.sync()
    close(out.cpu().numpy(), exp, 1e-4)
    close(out_nb.cpu().numpy(), exp - b, 1e-4)


@pytest.mark.parametrize("epilogue", ["none", "gelu", "residual_ls"])
@pytest.mark.parametrize("m,k,n", [(300, 1024, 1024), (129, 768, 4096), (1, 1, 1), (257, 130, 67)])
def test_linear_f32(gpu_ctx, epilogue, m, k, n):
    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
    b = (0.1 * rng.standard_normal(n)).astype(np.float32)
    ref = oracle.linear(x, w, b)
    kw = {}
    if epilogue == "gelu":
        ref = oracle.gelu(ref)
    elif epilogue == "residual_ls":
        res = rng.standard_normal((m, n)).astype(np.float32)
        gamma = (0.5 * rng.standard_normal(n)).astype(np.float32)
        ref = oracle.residual_ls(res, ref, gamma)
        kw = {"residual": torch.from_numpy(res).cuda(), "gamma": torch.from_numpy(gamma).cuda()}
    out = gpu_ctx.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda(),
                         epilogue=epilogue, **kw)
    gpu_ctx.sync()
    close(out.cpu().numpy(), ref, 1e-5)


def test_linear_rejects_unsupported(gpu_ctx):
    x = torch.zeros((4, 12), device="cuda", dtype=torch.float16)  # K = 12: not a multiple of 8
    w = torch.zeros((16, 12), device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.HsError):
        gpu_ctx.linear(x, w)
