"""Parity of the tcgen05 attention path against the CPU oracle (a
restatement of shaders/attention.wesl, layernorm.wesl, rope_apply.wesl).

Method: seeded f32 inputs are rounded to the storage dtype first, so the
oracle and the GPU see identical values; the oracle computes in f32, the GPU
on tensor cores in that dtype with f32 softmax statistics.  Gate (the
north-star tolerance for bf16/fp16 compute): cosine >= 0.9999 and
max |diff| <= 1e-2, NaN-proof (src/parity.rs:85-103).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from headshot_b200.engine import GpuContext, QkNorm, Rope

pytestmark = pytest.mark.gpu

TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
COS_MIN, ABS_MAX = 0.9999, 1e-2


def dev(x: np.ndarray, dtype: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(TORCH[dtype])


def host(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def rounded(x: np.ndarray, dtype: str) -> np.ndarray:
    return x if dtype == "f32" else oracle.round_to(dtype, x)


def gate(ours, ref, cos_min=COS_MIN, abs_max=ABS_MAX):
    m = oracle.compare(ours, ref)
    oracle.gate(m, cos_min, abs_max)
    return m


# ---- the reference's own known-answer cases (tests/kernels.rs:184-239) ----

@pytest.mark.parametrize("t", [17, 64, 150])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_attention_kernels_rs_cases(gpu_ctx: GpuContext, t, dtype):
    # S=2, H=3, D=64; SplitMix64 seed 5+T, q, k, v drawn in that order from one stream.
    s, h, d = 2, 3, 64
    vals = oracle.rng_uniform(5 + t, 3 * s * h * t * d)
    q, k, v = (rounded(vals[i * s * h * t * d:(i + 1) * s * h * t * d].reshape(s, h, t, d), dtype) for i in range(3))
    ref = oracle.attention(q, k, v)
    out = gpu_ctx.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype))
    gpu_ctx.sync()
    gate(host(out), ref)


@pytest.mark.parametrize("t", [1, 2, 100, 127, 128, 129, 255, 256, 257, 383, 1374])
def test_attention_tails_bf16(gpu_ctx, t):
    s, h, d = 1, 2, 64
    rng = np.random.default_rng(100 + t)
    q, k, v = (rounded(rng.standard_normal((s, h, t, d), np.float32), "bf16") for _ in range(3))
    ref = oracle.attention(q, k, v)
    out = gpu_ctx.attention(dev(q, "bf16"), dev(k, "bf16"), dev(v, "bf16"))
    gpu_ctx.sync()
    gate(host(out), ref)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("jump", [12.0, 40.0])
def test_attention_running_max_jump(gpu_ctx, dtype, jump):
    # Key 530 (tile 5 of 96-key tiles) scores `jump` log2 units above what
    # any query saw before, so the running max moves past the lazy-rescale
    # threshold (2^8) in a later tile: that tile's row max replaces the
    # running one and O and l are rescaled before its PV product.  At 40 a P
    # taken against the old max would overflow f16 (2^40).
    s, h, t, d = 1, 2, 700, 64
    rng = np.random.default_rng(11)
    u = rng.standard_normal(d).astype(np.float32)
    u /= np.linalg.norm(u)
    c = 0.125 * 1.4426950408889634
    q = u * 8 + 0.3 * rng.standard_normal((s, h, t, d)).astype(np.float32)
    k = 0.5 * rng.standard_normal((s, h, t, d)).astype(np.float32)
    k[:, :, 530, :] = u * (jump / c / 8)
    v = rng.standard_normal((s, h, t, d)).astype(np.float32)
    q, k, v = (rounded(x, dtype) for x in (q, k, v))
    ref = oracle.attention(q, k, v)
    out = gpu_ctx.attention(dev(q, dtype), dev(k, dtype), dev(v, dtype))
    gpu_ctx.sync()
    gate(host(out), ref)


def test_attention_f32_storage(gpu_ctx):
    # f32 callers: tensor cores see bf16-rounded q, k, v; out stays f32.
    s, h, t, d = 2, 2, 300, 64
    rng = np.random.default_rng(7)
    q, k, v = (rng.standard_normal((s, h, t, d), np.float32) for _ in range(3))
    ref = oracle.attention(q, k, v)
    out = gpu_ctx.attention(dev(q, "f32"), dev(k, "f32"), dev(v, "f32"))
    gpu_ctx.sync()
    assert out.dtype == torch.float32
    gate(host(out), ref)


# ---- fused QK-norm + RoPE (block.rs:136-148) --------------------------------

def _fused_case(gpu_ctx, s, h, t, dtype, prefix, tpf, grid, seed, ln_random=True, rope=True, ln_gain=None,
                ln_shift=0.0, round_qk=False):
    d = 64
    rng = np.random.default_rng(seed)
    q, k, v = (rounded(rng.standard_normal((s, h, t, d), np.float32), dtype) for _ in range(3))
    if ln_gain is not None:
        # Shared bias along one unit direction: it raises |q'| and |k'| (and
        # so the kernel's score bound) while its q'.k' term is the same for
        # every key and cancels in the softmax.
        u = rng.standard_normal(d).astype(np.float32)
        u /= np.linalg.norm(u)
        qw = kw = np.full(d, ln_gain, np.float32)
        qb = kb = (ln_shift * u).astype(np.float32)
    elif ln_random:
        qw, qb, kw, kb = (rng.uniform(0.5, 1.5, d).astype(np.float32), rng.uniform(-0.2, 0.2, d).astype(np.float32),
                          rng.uniform(0.5, 1.5, d).astype(np.float32), rng.uniform(-0.2, 0.2, d).astype(np.float32))
    else:
        qw = kw = np.ones(d, np.float32)
        qb = kb = np.zeros(d, np.float32)
    eps = 1e-6
    sin = cos = None
    if rope:
        sin, cos = oracle.rope_tables(*grid)
    qn = oracle.qk_prep(q, qw, qb, eps, sin, cos, prefix, tpf)
    kn = oracle.qk_prep(k, kw, kb, eps, sin, cos, prefix, tpf)
    if round_qk:  # the reference stores q', k' in the tensor dtype between its kernels
        qn, kn = rounded(qn, dtype), rounded(kn, dtype)
    ref = oracle.attention(qn, kn, v)
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = gpu_ctx.attention_fused(
        dev(q, dtype), dev(k, dtype), dev(v, dtype), qk_norm=QkNorm(c(qw), c(qb), c(kw), c(kb), eps),
        rope=Rope(c(sin), c(cos), prefix, tpf) if rope else None)
    gpu_ctx.sync()
    return host(out), ref


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fused_frame_reference_shape(gpu_ctx, dtype):
    # Reference trunk frame block: prefix 17, P = 4x4 patches -> T = 33.
    ours, ref = _fused_case(gpu_ctx, 3, 4, 33, dtype, prefix=17, tpf=33, grid=(4, 4), seed=11)
    gate(ours, ref)


def test_fused_frame_baseline_shape(gpu_ctx):
    # BASELINE frame attention: 37x37 grid + 5 special tokens, T = 1374, fp16.
    ours, ref = _fused_case(gpu_ctx, 2, 16, 1374, "f16", prefix=5, tpf=1374, grid=(37, 37), seed=2)
    gate(ours, ref)


def test_fused_global_multi_frame(gpu_ctx):
    # Global attention over 3 frames of 1374 tokens with per-frame RoPE positions.
    ours, ref = _fused_case(gpu_ctx, 1, 2, 3 * 1374, "bf16", prefix=5, tpf=1374, grid=(37, 37), seed=3,
                            ln_random=False)
    gate(ours, ref)


def test_fused_no_rope(gpu_ctx):
    ours, ref = _fused_case(gpu_ctx, 1, 3, 500, "bf16", prefix=0, tpf=500, grid=(1, 1), seed=4, rope=False)
    gate(ours, ref)


@pytest.mark.parametrize("gain,shift", [(0.25, 0.0), (1.0, 0.0), (1.0, 14.0)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fused_score_bound_modes(gpu_ctx, dtype, gain, shift):
    # The kernel bounds every score by max|q'| * max|k'| * scale * log2(e)
    # (qk_prep records the norms; here |q'|, |k'| <= 8 * gain + shift).  A
    # small bound selects the fixed-offset softmax (no running max): bf16 up
    # to 48, f16 up to 14 (bounds 0.72 and 11.5 here); the shifted case
    # (bound 63) takes the running-max path in both types.  The oracle
    # rounds q', k' to the dtype, as the reference's separate kernels store
    # them.
    ours, ref = _fused_case(gpu_ctx, 1, 4, 1374, dtype, prefix=5, tpf=1374, grid=(37, 37), seed=9, ln_gain=gain,
                            ln_shift=shift, round_qk=True)
    gate(ours, ref)


def test_fused_f32_storage(gpu_ctx):
    ours, ref = _fused_case(gpu_ctx, 2, 2, 199, "f32", prefix=17, tpf=199, grid=(13, 14), seed=5)
    gate(ours, ref)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("s,h,t", [(3, 3, 32), (1, 9, 31), (2, 5, 65), (17, 1, 96)])
def test_fused_prep_unit_edges(gpu_ctx, dtype, s, h, t):
    # The QK prep moves 32 tokens of 8 sequences per unit through shared
    # memory: sequence counts just past a multiple of 8, and token counts at,
    # below and above the 32-token unit, leave partial units both ways.
    ours, ref = _fused_case(gpu_ctx, s, h, t, dtype, prefix=5, tpf=t, grid=(37, 37), seed=40 + s * h + t)
    gate(ours, ref)


# ---- companion ops -----------------------------------------------------------

@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_layernorm(gpu_ctx, dtype):
    # kernels.rs:100-126 shape (19 x 300, dim > 256) plus the QK-norm shape.
    for rows, dim, seed in ((19, 300, 3), (1000, 64, 4)):
        x = rounded(oracle.rng_uniform(seed, rows * dim).reshape(rows, dim), dtype)
        w = oracle.rng_uniform(seed + 100, dim)
        b = oracle.rng_uniform(seed + 200, dim)
        ref = oracle.layernorm(x, w, b, 1e-5)
        out = gpu_ctx.layernorm(dev(x, dtype), torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda())
        gpu_ctx.sync()
        tol = 1e-4 if dtype == "f32" else 2e-2 * max(1.0, float(np.abs(ref).max()))
        assert np.abs(host(out) - ref).max() <= tol


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_rope_apply(gpu_ctx, dtype):
    # kernels.rs:149-182: prefix 5 on a 2x3 grid, s=2, h=3, t=11.
    s, h, t, d, prefix = 2, 3, 11, 64, 5
    sin, cos = oracle.rope_tables(2, 3)
    x = rounded(oracle.rng_uniform(4, s * h * t * d).reshape(s, h, t, d), dtype)
    ref = oracle.rope_apply(x, sin, cos, prefix)
    g = dev(x, dtype)
    gpu_ctx.rope_apply(g, torch.from_numpy(sin).cuda(), torch.from_numpy(cos).cuda(), prefix)
    gpu_ctx.sync()
    tol = 1e-5 if dtype == "f32" else 2e-2
    assert np.abs(host(g) - ref).max() <= tol * max(1.0, float(np.abs(ref).max()))


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_split_merge_roundtrip(gpu_ctx, dtype):
    # kernels.rs:241-274, exact.
    for s, t, h, d in ((2, 5, 4, 8), (3, 17, 16, 64)):
        x = rounded(oracle.rng_uniform(6, s * t * h * d).reshape(s * t, h * d), dtype)
        heads = gpu_ctx.split_heads(dev(x, dtype), s, t, h, d)
        gpu_ctx.sync()
        np.testing.assert_array_equal(host(heads), oracle.split_heads(x, s, t, h, d))
        merged = gpu_ctx.attn_merge(heads)
        gpu_ctx.sync()
        np.testing.assert_array_equal(host(merged), x)


# ---- the block's attention section on the projection layout (f1) ------------

def _block_inputs(s, h, t, dtype, seed):
    d = 64
    rng = np.random.default_rng(seed)
    # the three (S*T, H*D) projection outputs Block::forward feeds split_heads
    qt, kt, vt = (rounded(rng.standard_normal((s * t, h * d), np.float32), dtype) for _ in range(3))
    qw, kw = (rng.uniform(0.5, 1.5, d).astype(np.float32) for _ in range(2))
    qb, kb = (rng.uniform(-0.2, 0.2, d).astype(np.float32) for _ in range(2))
    return qt, kt, vt, (qw, qb, kw, kb)


@pytest.mark.parametrize("dtype,s,t,tpf", [("bf16", 2, 1374, 1374), ("f16", 3, 1374, 1374), ("bf16", 1, 2748, 1374)])
def test_block_fused_matches_oracle(gpu_ctx, dtype, s, t, tpf):
    # split_heads -> QK-norm -> RoPE -> attention -> attn_merge (block.rs:130-149)
    # in one call on the token-major layout, against the oracle's five steps.
    h, d, prefix, eps = 4, 64, 5, 1e-6
    qt, kt, vt, (qw, qb, kw, kb) = _block_inputs(s, h, t, dtype, 31 + t)
    sin, cos = oracle.rope_tables(37, 37)
    q, k, v = (oracle.split_heads(x, s, t, h, d) for x in (qt, kt, vt))
    qn = rounded(oracle.qk_prep(q, qw, qb, eps, sin, cos, prefix, tpf), dtype)
    kn = rounded(oracle.qk_prep(k, kw, kb, eps, sin, cos, prefix, tpf), dtype)
    ref = oracle.attn_merge(oracle.attention(qn, kn, v))
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = gpu_ctx.attention_block(dev(qt, dtype), dev(kt, dtype), dev(vt, dtype), s, t, h,
                                  qk_norm=QkNorm(c(qw), c(qb), c(kw), c(kb), eps),
                                  rope=Rope(c(sin), c(cos), prefix, tpf))
    gpu_ctx.sync()
    assert out.shape == (s * t, h * d)
    gate(host(out), ref)


@pytest.mark.parametrize("dtype,s,h,t", [("bf16", 3, 3, 33), ("f16", 1, 9, 95)])
def test_block_fused_prep_unit_edges(gpu_ctx, dtype, s, h, t):
    # The prep's partial units on the token-major projection layout (row
    # stride H*64, so the tensor map steps heads by one 128-byte row).
    d, prefix, eps = 64, 5, 1e-6
    qt, kt, vt, (qw, qb, kw, kb) = _block_inputs(s, h, t, dtype, 71 + t)
    sin, cos = oracle.rope_tables(37, 37)
    q, k, v = (oracle.split_heads(x, s, t, h, d) for x in (qt, kt, vt))
    qn = rounded(oracle.qk_prep(q, qw, qb, eps, sin, cos, prefix, t), dtype)
    kn = rounded(oracle.qk_prep(k, kw, kb, eps, sin, cos, prefix, t), dtype)
    ref = oracle.attn_merge(oracle.attention(qn, kn, v))
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = gpu_ctx.attention_block(dev(qt, dtype), dev(kt, dtype), dev(vt, dtype), s, t, h,
                                  qk_norm=QkNorm(c(qw), c(qb), c(kw), c(kb), eps),
                                  rope=Rope(c(sin), c(cos), prefix, t))
    gpu_ctx.sync()
    gate(host(out), ref)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_block_plain_reads_token_major_directly(gpu_ctx, dtype):
    # No QK-norm/RoPE: the kernel's tensor maps read q, k, v straight from the
    # token-major rows (no prep pass) and the epilogue writes merged rows.
    s, h, t, d = 2, 3, 777, 64
    qt, kt, vt, _ = _block_inputs(s, h, t, dtype, 5)
    q, k, v = (oracle.split_heads(x, s, t, h, d) for x in (qt, kt, vt))
    ref = oracle.attn_merge(oracle.attention(q, k, v))
    out = gpu_ctx.attention_block(dev(qt, dtype), dev(kt, dtype), dev(vt, dtype), s, t, h)
    gpu_ctx.sync()
    gate(host(out), ref)


def test_block_fused_equals_split_fused_merge_on_gpu(gpu_ctx):
    # Same kernel, two layouts: the block entry point must reproduce
    # split_heads + attention_fused + attn_merge bit for bit.
    s, h, t, d, prefix, eps = 2, 4, 1374, 64, 5, 1e-6
    qt, kt, vt, (qw, qb, kw, kb) = _block_inputs(s, h, t, "bf16", 77)
    sin, cos = oracle.rope_tables(37, 37)
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    norm, rope = QkNorm(c(qw), c(qb), c(kw), c(kb), eps), Rope(c(sin), c(cos), prefix, t)
    qd, kd, vd = (dev(x, "bf16") for x in (qt, kt, vt))
    merged = gpu_ctx.attention_block(qd, kd, vd, s, t, h, qk_norm=norm, rope=rope)
    heads = [gpu_ctx.split_heads(x, s, t, h, d) for x in (qd, kd, vd)]
    two_step = gpu_ctx.attn_merge(gpu_ctx.attention_fused(*heads, qk_norm=norm, rope=rope))
    gpu_ctx.sync()
    assert torch.equal(merged, two_step.reshape(merged.shape))


def test_block_fused_f32_storage(gpu_ctx):
    s, h, t, d, prefix, eps = 1, 2, 500, 64, 5, 1e-6
    qt, kt, vt, (qw, qb, kw, kb) = _block_inputs(s, h, t, "f32", 8)
    sin, cos = oracle.rope_tables(37, 37)
    q, k, v = (oracle.split_heads(x, s, t, h, d) for x in (qt, kt, vt))
    ref = oracle.attn_merge(oracle.attention(oracle.qk_prep(q, qw, qb, eps, sin, cos, prefix, t),
                                             oracle.qk_prep(k, kw, kb, eps, sin, cos, prefix, t), v))
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = gpu_ctx.attention_block(dev(qt, "f32"), dev(kt, "f32"), dev(vt, "f32"), s, t, h,
                                  qk_norm=QkNorm(c(qw), c(qb), c(kw), c(kb), eps), rope=Rope(c(sin), c(cos), prefix, t))
    gpu_ctx.sync()
    assert out.dtype == torch.float32
    gate(host(out), ref)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_repeated_calls_are_bit_identical(gpu_ctx, dtype):
    # The kernel's barriers must not depend on timing: warps of a warpgroup
    # drift apart by up to a tile (the last tile's epilogue once read O
    # early when a fast warp got there before the item's second-to-last PV
    # product was issued).  Many identical calls, all equal bit for bit.
    s, h, t, d, prefix, eps = 2, 16, 1374, 64, 5, 1e-6
    rng = np.random.default_rng(123)
    q, k, v = (rounded(rng.standard_normal((s, h, t, d), np.float32), dtype) for _ in range(3))
    qw, kw = (rng.uniform(0.8, 1.6, d).astype(np.float32) for _ in range(2))
    qb, kb = (rng.uniform(-0.1, 0.1, d).astype(np.float32) for _ in range(2))
    sin, cos = oracle.rope_tables(37, 37)
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    norm, rope = QkNorm(c(qw), c(qb), c(kw), c(kb), eps), Rope(c(sin), c(cos), prefix, t)
    qd, kd, vd = (dev(x, dtype) for x in (q, k, v))
    first = gpu_ctx.attention_fused(qd, kd, vd, qk_norm=norm, rope=rope)
    for i in range(64):
        again = gpu_ctx.attention_fused(qd, kd, vd, qk_norm=norm, rope=rope)
        gpu_ctx.sync()
        assert torch.equal(first, again), f"call {i + 1} differs from the first"


@pytest.mark.parametrize("s,h,t", [
    (1, 3, 1374),  # frames' 94-row last items (warpgroup 1 idle), odd sequence count
    (2, 16, 100),  # one short item per sequence
    (1, 4, 128),   # last item exactly one 128-row tile
    (1, 2, 129),   # one row into the second tile
    (1, 5, 300),
    (1, 1, 1374),  # a single sequence
])
def test_short_last_items(gpu_ctx, s, h, t):
    # Items whose second 128-row tile lies past the sequence end: that
    # warpgroup and its MMA warp skip the item and only release its K/V stages.
    rng = np.random.default_rng(s * 1000 + h * 10 + t)
    q, k, v = (rounded(rng.standard_normal((s, h, t, 64), np.float32), "bf16") for _ in range(3))
    out = gpu_ctx.attention(*(dev(x, "bf16") for x in (q, k, v)))
    gpu_ctx.sync()
    gate(host(out), oracle.attention(q, k, v))


def test_long_sequence_alternating_kv_direction(gpu_ctx):
    # Past 1024 key tiles (24 MiB of K and V per sequence) every other wave of
    # items walks K/V last tile to first, so the partial last tile (67 keys
    # here) is the first one such an item masks.  Rows from forward and
    # backward items against the oracle over all keys, and the order is a
    # function of the item index alone: repeated calls agree bit for bit.
    s, h, t = 1, 2, 100_003
    rng = np.random.default_rng(77)
    q, k, v = (rounded(rng.standard_normal((s, h, t, 64), np.float32), "bf16") for _ in range(3))
    qd, kd, vd = (dev(x, "bf16") for x in (q, k, v))
    out = gpu_ctx.attention(qd, kd, vd)
    again = gpu_ctx.attention(qd, kd, vd)
    gpu_ctx.sync()
    assert torch.equal(out, again)
    items = -(-t // 256)
    # first rows of items in waves 0, 1 and 2 of 148 (head 0) and of head 1's first item, plus random rows
    starts = [0, 147 * 256, 148 * 256, 295 * 256, 296 * 256, (items - 1) * 256, t + 0, t + 200 * 256]
    rows = {r + d for r in starts for d in (0, 5, 128, 255) if (r % t) + d < t}
    rows |= {int(x) for x in rng.integers(0, s * h * t, 256)}
    rows = np.array(sorted(rows), np.int64)
    ours = host(out.reshape(-1, 64)[torch.from_numpy(rows).cuda()])
    gate(ours, oracle.attention_rows(q, k, v, rows))


# ---- BASELINE configurations at their own sizes (sampled query rows) --------
#
# The bench's workloads, generated exactly as bench.py generates them on rank 0
# (torch generator on the device, seed * 1000, N(0,1) f32 rounded to the
# storage type), run through hs_attention_fused at full size.  Rows are
# independent, so a fixed sample of query rows (spread over sequences, the
# first and last 256-row items, the short tail item, frame boundaries and the
# unrotated special tokens) is checked against the oracle over every key of
# its sequence (oracle.attention_rows, attention.wesl:36-82).

def _config_inputs(s, h, t, dtype, seed):
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(seed * 1000)
    return tuple(torch.randn((s, h, t, 64), device=dev, dtype=torch.float32, generator=g).to(TORCH[dtype])
                 for _ in range(3))


def _sample_rows(s, h, t, tpf, prefix, n=512, seed=0):
    """Flattened (s*h + head) * t + token indices: fixed edge positions plus random fill."""
    rng = np.random.default_rng(seed)
    seqs = s * h
    tail0 = (t // 256) * 256 if t % 256 else t - 256  # first row of the last (short) 256-row item
    edge_tokens = sorted({0, 1, prefix - 1, prefix, 127, 128, 255, 256, tail0, tail0 + 1, t - 2, t - 1,
                          tpf - 1, min(tpf, t - 1), min(tpf + prefix, t - 1), t // 2} & set(range(t)))
    edge_seqs = sorted({0, 1, h - 1, seqs // 2, seqs - 1})
    rows = {sq * t + tok for sq in edge_seqs for tok in edge_tokens}
    rows |= {int(sq) * t + int(tok) for sq, tok in zip(rng.integers(0, seqs, 64), rng.integers(tail0, t, 64))}
    while len(rows) < n:
        rows.add(int(rng.integers(0, seqs)) * t + int(rng.integers(0, t)))
    return np.array(sorted(rows)[:n], np.int64)


@pytest.mark.parametrize("name,s,h,t,dtype,seed,gain", [
    ("config2_global43k", 1, 16, 32 * 1374, "bf16", 1, 1.0),
    ("config3_frames200", 200, 16, 1374, "f16", 2, 1.0),
    ("config4_global274k", 1, 16, 200 * 1374, "bf16", 3, 1.0),
    # QK-norm gain 1.2 lifts the f16 score bound to ~16.6 > 14: the running-max softmax at config 3's size
    ("config3_running_max", 200, 16, 1374, "f16", 2, 1.2),
])
def test_baseline_config_full_size(gpu_ctx, name, s, h, t, dtype, seed, gain):
    tpf, prefix, eps = 1374, 5, 1e-6
    q, k, v = _config_inputs(s, h, t, dtype, seed)
    sin, cos = oracle.rope_tables(37, 37)
    w = np.full(64, gain, np.float32)
    b = np.zeros(64, np.float32)
    c = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = gpu_ctx.attention_fused(q, k, v, qk_norm=QkNorm(c(w), c(b), c(w), c(b), eps),
                                  rope=Rope(c(sin), c(cos), prefix, tpf))
    gpu_ctx.sync()
    rows = _sample_rows(s, h, t, tpf, prefix)
    ours = host(out.reshape(-1, 64)[torch.from_numpy(rows).cuda()])
    del out
    qh, kh, vh = (host(x) for x in (q, k, v))
    del q, k, v
    # q' and k' rounded to the storage type, as the reference's separate kernels store them
    qn = rounded(oracle.qk_prep(qh, w, b, eps, sin, cos, prefix, tpf), dtype)
    del qh
    kn = rounded(oracle.qk_prep(kh, w, b, eps, sin, cos, prefix, tpf), dtype)
    del kh
    ref = oracle.attention_rows(qn, kn, vh, rows)
    gate(ours, ref)
