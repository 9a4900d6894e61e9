"""hs_attention_fused_noalloc against hs_attention_fused, through the C ABI.

The no-allocation variant serves callers that cannot let the library call
cudaMalloc (their device memory belongs to their own allocator or a pool
reserved up front, or they must not stall or fail on an allocation while a
session runs).  It must give the same results as the allocating entry point:
checked here on two calls in a row (the second reuses the library's fixed
scratch array, which still holds the first call's rows), with the tolerance
the other parity tests use.  Collected last on purpose (file name).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from headshot_b200 import _lib
from headshot_b200.engine import GpuContext, QkNorm, Rope

pytestmark = pytest.mark.gpu

COS_MIN, ABS_MAX = 0.9999, 1e-2
HS_NOALLOC_MAX_ROWS = 262144  # include/headshot_cuda.h
_vp, _u32, _f32, _i = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float, ctypes.c_int


def _noalloc():
    fn = _lib.lib().hs_attention_fused_noalloc
    fn.restype = _i
    fn.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp, _vp, _f32, _vp, _vp,
                   _u32, _u32, _u32]
    return fn


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_noalloc_matches_allocating_entry_point(dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s, h, t, d, prefix = 2, 16, 1374, 64, 5
    g = torch.Generator(device=dev).manual_seed(21)
    q, k, v = (torch.randn((s, h, t, d), device=dev, generator=g).to(dtype) for _ in range(3))
    qw, kw = (1.0 + 0.2 * torch.randn(d, device=dev, generator=g) for _ in range(2))
    qb, kb = (0.1 * torch.randn(d, device=dev, generator=g) for _ in range(2))
    sin, cos = oracle.rope_tables(37, 37)
    sin_d, cos_d = torch.from_numpy(sin).to(dev), torch.from_numpy(cos).to(dev)
    eps = 1e-6

    ctx = GpuContext(0)
    ref = ctx.attention_fused(q, k, v, qk_norm=QkNorm(qw, qb, kw, kb, eps), rope=Rope(sin_d, cos_d, prefix, t))
    ctx.sync()
    ref_h = ref.float().cpu().numpy()

    fn = _noalloc()
    code = _lib.HS_BF16 if dtype == torch.bfloat16 else _lib.HS_F16
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = fn(stream, _p(status), _p(q), _p(k), _p(v), _p(out), s, h, t, d, code, 0.0, _p(qw), _p(qb), _p(kw),
                _p(kb), eps, _p(sin_d), _p(cos_d), sin.shape[0], prefix, t)
        assert rc == _lib.HS_OK, _lib.last_error()
        torch.cuda.synchronize(dev)
        assert int(status.item()) == 0, "an in-kernel wait timed out"
        m = oracle.compare(out.float().cpu().numpy(), ref_h)
        oracle.gate(m, COS_MIN, ABS_MAX)
    ctx.close()


def test_noalloc_rejects_oversized_requests():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fn = _noalloc()
    rows = HS_NOALLOC_MAX_ROWS + 1
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    rc = fn(None, None, _p(dummy), _p(dummy), _p(dummy), _p(dummy), 1, 1, rows, 64, _lib.HS_BF16, 0.0, None, None,
            None, None, 1e-6, None, None, 0, 0, 0)
    assert rc == _lib.HS_ERR_INVALID
    assert "exceeds the fixed scratch" in _lib.last_error()
