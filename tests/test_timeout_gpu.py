"""The in-kernel bounded waits give up cleanly and leave the context usable.

The reference's contract for a step that cannot finish is an error between
steps with the engine still usable (cancellation, src/engine/mod.rs:102-106;
srv/tests/session.rs:186-231).  Here every spin-wait in a kernel is bounded:
on expiry it records a site code in the context's status word, the CTAs stop,
drain their own TMA loads and MMAs (with a fixed teardown bound of their own)
and exit, and hs_sync returns HS_ERR_TIMEOUT.

A wait timeout of 0 makes every wait whose condition does not already hold
give up at once, so a fused call is driven into that path deterministically
(the first score tile of every item depends on TMA loads and an MMA issued
after the kernel starts), without faulting or hanging anything.  The next
call with the default timeout must then pass the parity gate on the same
context.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from headshot_b200 import _lib
from headshot_b200.engine import GpuContext, QkNorm, Rope

pytestmark = pytest.mark.gpu


def _case(dtype=torch.bfloat16, s=1, h=4, t=4122, seed=5):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    q, k, v = (torch.randn((s, h, t, 64), device=dev, generator=g).to(dtype) for _ in range(3))
    w = torch.ones(64, device=dev)
    b = torch.zeros(64, device=dev)
    sin, cos = (torch.from_numpy(a).to(dev) for a in oracle.rope_tables(37, 37))
    return q, k, v, QkNorm(w, b, w, b, 1e-6), Rope(sin, cos, 5, 1374)


def _oracle(q, k, v, dtype="bf16"):
    qh, kh, vh = (x.float().cpu().numpy() for x in (q, k, v))
    w, b = np.ones(64, np.float32), np.zeros(64, np.float32)
    sin, cos = oracle.rope_tables(37, 37)
    qn = oracle.round_to(dtype, oracle.qk_prep(qh, w, b, 1e-6, sin, cos, 5, 1374))
    kn = oracle.round_to(dtype, oracle.qk_prep(kh, w, b, 1e-6, sin, cos, 5, 1374))
    return oracle.attention(qn, kn, vh)


def test_timeout_is_reported_and_the_context_recovers():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    q, k, v, norm, rope = _case()
    ctx = GpuContext(0)
    try:
        ctx.set_wait_timeout_ms(0)
        ctx.attention_fused(q, k, v, qk_norm=norm, rope=rope)
        with pytest.raises(_lib.HsError) as err:
            ctx.sync()
        assert err.value.status == _lib.HS_ERR_TIMEOUT
        assert "site 0x" in err.value.message
        # hs_sync cleared the status word: nothing further is pending
        ctx.sync()

        ctx.set_wait_timeout_ms(2000)
        out = ctx.attention_fused(q, k, v, qk_norm=norm, rope=rope)
        ctx.sync()
        m = oracle.compare(out.float().cpu().numpy(), _oracle(q, k, v))
        oracle.gate(m, 0.9999, 1e-2)
        # and a plain attention on the same context: the work counter and the
        # score-bound words the aborted launch left behind were reset
        plain = ctx.attention(q, k, v)
        ctx.sync()
        qh, kh, vh = (x.float().cpu().numpy() for x in (q, k, v))
        oracle.gate(oracle.compare(plain.float().cpu().numpy(), oracle.attention(qh, kh, vh)), 0.9999, 1e-2)
    finally:
        ctx.close()


def test_timeout_in_the_linear_leaves_the_context_usable():
    # The block linears' persistent GEMM takes the same path (its epilogue
    # still waits for the output stores it issued before leaving).
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn((4096, 1024), device=dev, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn((2048, 1024), device=dev, generator=g)).to(torch.bfloat16)
    ctx = GpuContext(0)
    try:
        ctx.set_wait_timeout_ms(0)
        ctx.linear(x, w)
        with pytest.raises(_lib.HsError) as err:
            ctx.sync()
        assert err.value.status == _lib.HS_ERR_TIMEOUT
        ctx.set_wait_timeout_ms(2000)
        out = ctx.linear(x, w)
        ctx.sync()
        ref = oracle.linear(x.float().cpu().numpy(), w.float().cpu().numpy())
        # bf16 output rounding as the tolerance (abs + rel), as the linear's own parity tests
        tol = 8e-3
        excess = np.abs(out.float().cpu().numpy() - ref) - (tol + tol * np.abs(ref))
        assert excess.max() <= 0, f"max excess {excess.max():.3g}"
    finally:
        ctx.close()
