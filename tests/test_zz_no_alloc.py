"""hs_attention_fused_noalloc against hs_attention_fused and the oracle, through the C ABI.

The no-allocation variant serves callers that cannot let the library call
cudaMalloc: hosts whose device memory belongs to their own allocator or to a
pool reserved up front, and session loops that must not stall or fail on an
allocation while a session runs.  It runs the same QK prep and attention
kernels on the same bytes as the allocating entry point, only with its
scratch in a fixed array inside the library, so its output must equal that
entry point's bit for bit: checked here on two calls in a row (the second
reuses the array, which still holds the first call's rows).  One case is
also gated against the CPU oracle with the tolerance the other parity tests
use, so the check does not rest on another GPU path alone.  Collected last
on purpose (file name).
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


def _inputs(dev, dtype, s, h, t, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    q, k, v = (torch.randn((s, h, t, 64), device=dev, generator=g).to(dtype) for _ in range(3))
    qw, kw = (1.0 + 0.2 * torch.randn(64, device=dev, generator=g) for _ in range(2))
    qb, kb = (0.1 * torch.randn(64, device=dev, generator=g) for _ in range(2))
    return q, k, v, (qw, qb, kw, kb)


def _call(fn, dev, dtype, q, k, v, status, norm, rope, prefix, tpf):
    """One no-alloc call on torch's current stream; returns the output tensor."""
    code = _lib.HS_BF16 if dtype == torch.bfloat16 else _lib.HS_F16
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    s, h, t, d = q.shape
    out = torch.full_like(q, float("nan"))
    qw, qb, kw, kb = norm if norm is not None else (None,) * 4
    sin, cos = rope if rope is not None else (None, None)
    rc = fn(stream, _p(status), _p(q), _p(k), _p(v), _p(out), s, h, t, d, code, 0.0, _p(qw), _p(qb), _p(kw), _p(kb),
            1e-6, _p(sin), _p(cos), 0 if sin is None else sin.shape[0], prefix, tpf)
    assert rc == _lib.HS_OK, _lib.last_error()
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_noalloc_equals_allocating_entry_point(dtype):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s, h, t, prefix = 2, 16, 1374, 5
    q, k, v, (qw, qb, kw, kb) = _inputs(dev, dtype, s, h, t, 21)
    sin, cos = (torch.from_numpy(a).to(dev) for a in oracle.rope_tables(37, 37))

    ctx = GpuContext(0)
    ref = ctx.attention_fused(q, k, v, qk_norm=QkNorm(qw, qb, kw, kb, 1e-6), rope=Rope(sin, cos, prefix, t))
    ctx.sync()

    fn = _noalloc()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for call in range(2):
        out = _call(fn, dev, dtype, q, k, v, status, (qw, qb, kw, kb), (sin, cos), prefix, t)
        torch.cuda.synchronize(dev)
        assert int(status.item()) == 0, "an in-kernel wait timed out"
        assert torch.equal(out, ref), f"call {call + 1} differs from hs_attention_fused"
    ctx.close()


def test_noalloc_without_prologue_equals_plain_attention():
    # No QK-norm and no RoPE: q and k go to the attention kernel in place (no
    # scratch rows), the running-max softmax; the same bytes as hs_attention.
    # The second call passes no status word (timeouts go to the library's
    # own word).
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dtype = torch.bfloat16
    q, k, v, _ = _inputs(dev, dtype, 3, 4, 777, 22)
    ctx = GpuContext(0)
    ref = ctx.attention(q, k, v)
    ctx.sync()
    fn = _noalloc()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for st in (status, None):
        out = _call(fn, dev, dtype, q, k, v, st, None, None, 0, 0)
        torch.cuda.synchronize(dev)
        assert torch.equal(out, ref)
    assert int(status.item()) == 0
    ctx.close()


def test_noalloc_matches_oracle():
    # The fused case against the CPU oracle (attention.wesl, layernorm.wesl,
    # rope_apply.wesl restated), q' and k' rounded to the storage type as the
    # reference's separate kernels store them; no status word on this call.
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dtype, s, h, t, prefix = torch.float16, 2, 3, 1374, 5
    q, k, v, (qw, qb, kw, kb) = _inputs(dev, dtype, s, h, t, 23)
    sin_h, cos_h = oracle.rope_tables(37, 37)
    sin, cos = torch.from_numpy(sin_h).to(dev), torch.from_numpy(cos_h).to(dev)
    out = _call(_noalloc(), dev, dtype, q, k, v, None, (qw, qb, kw, kb), (sin, cos), prefix, t)
    torch.cuda.synchronize(dev)
    hq, hk, hv = (x.float().cpu().numpy() for x in (q, k, v))
    w = [x.float().cpu().numpy() for x in (qw, qb, kw, kb)]
    qn = oracle.round_to("f16", oracle.qk_prep(hq, w[0], w[1], 1e-6, sin_h, cos_h, prefix, t))
    kn = oracle.round_to("f16", oracle.qk_prep(hk, w[2], w[3], 1e-6, sin_h, cos_h, prefix, t))
    m = oracle.compare(out.float().cpu().numpy(), oracle.attention(qn, kn, hv))
    oracle.gate(m, COS_MIN, ABS_MAX)


def test_noalloc_rejects_oversized_requests():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fn = _noalloc()
    rows = HS_NOALLOC_MAX_ROWS + 1
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(64, device="cuda")
    rc = fn(None, None, _p(dummy), _p(dummy), _p(dummy), _p(dummy), 1, 1, rows, 64, _lib.HS_BF16, 0.0, _p(w), _p(w),
            _p(w), _p(w), 1e-6, None, None, 0, 0, 0)
    assert rc == _lib.HS_ERR_INVALID
    assert "exceeds the fixed scratch" in _lib.last_error()
