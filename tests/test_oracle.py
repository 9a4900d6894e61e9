"""Pins the CPU oracle (oracle/headshot_oracle.c) before it is trusted as
the parity checker: the reference's own known-answer tests restated
(src/engine/rope.rs:57-104, tests/kernels.rs:100-274), plus the golden
fixtures of tests/golden/make_golden.py (an independent numpy restatement).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


# ---- RNG (tests/kernels.rs:7-23) --------------------------------------------

@pytest.mark.parametrize("seed", [1, 3, 4, 22, 69, 155])
def test_rng_matches_golden(seed):
    np.testing.assert_array_equal(oracle.rng_uniform(seed, 64), GOLDEN[f"rng_{seed}"])


def test_rng_f16_exact_generator():
    """tests/f16_ops.rs:7-19: SplitMix64 without the final xorshift, (z>>40)/2^24*2-1, rounded
    to f16; restated here independently with Python integers for the first values."""
    mask = (1 << 64) - 1
    s, want = 7, []
    for _ in range(64):
        s = (s + 0x9E3779B97F4A7C15) & mask
        z = ((s ^ (s >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        want.append(np.float16(np.float32((z >> 40) / float(1 << 24) * 2.0 - 1.0)))
    got = oracle.rng_f16_exact(7, 64)
    np.testing.assert_array_equal(got, np.array(want, np.float32))
    many = oracle.rng_f16_exact(1, 1 << 16)
    assert many.min() >= -1.0 and many.max() <= 1.0
    np.testing.assert_array_equal(many, many.astype(np.float16).astype(np.float32))


def test_rng_normal_moments():
    x = oracle.rng_normal(1, 200_000)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01
    np.testing.assert_array_equal(x[:10], oracle.rng_normal(1, 10))


# ---- RoPE (src/engine/rope.rs:57-104) ----------------------------------------

def test_periods_formula():
    p = oracle.rope_periods()
    assert p[0] == 1.0
    assert abs(p[8] - 10.0) < 1e-4  # i=8: 100^(16/32) = 10
    assert abs(p[15] - np.float32(100.0) ** np.float32(30.0 / 32.0)) < 1e-3
    np.testing.assert_allclose(p, GOLDEN["periods"], rtol=1e-6)


def test_table_values():
    sin, cos = oracle.rope_tables(2, 3)
    assert sin.shape == (6, 64)
    angle = np.float32(2 * np.pi) * np.float32(2.0 * (2.5 / 3.0) - 1.0)
    idx = 5  # token (row 1, col 2)
    assert abs(sin[idx, 16] - np.sin(angle)) < 1e-6
    assert abs(cos[idx, 16] - np.cos(angle)) < 1e-6
    assert abs(sin[idx, 0]) < 1e-6 and abs(cos[idx, 0] - 1.0) < 1e-6
    np.testing.assert_array_equal(sin[:, :32], sin[:, 32:])
    np.testing.assert_array_equal(cos[:, :32], cos[:, 32:])
    for g in ("2x3", "4x4"):
        s, c = oracle.rope_tables(*map(int, g.split("x")))
        np.testing.assert_allclose(s, GOLDEN[f"sin_{g}"], atol=2e-7)
        np.testing.assert_allclose(c, GOLDEN[f"cos_{g}"], atol=2e-7)


def test_rotation_preserves_norm():
    sin, cos = oracle.rope_tables(4, 4)
    x = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.37)).astype(np.float32)
    y = oracle.rope_apply_row(x, sin, cos, 7)
    for i in range(32):
        assert abs(np.hypot(x[i], x[i + 32]) - np.hypot(y[i], y[i + 32])) < 1e-5


def test_rope_apply_matches_apply_cpu():
    # tests/kernels.rs:149-182
    s, h, t, d, prefix = 2, 3, 11, 64, 5
    sin, cos = oracle.rope_tables(2, 3)
    x = oracle.rng_uniform(4, s * h * t * d).reshape(s, h, t, d)
    got = oracle.rope_apply(x, sin, cos, prefix)
    for si in range(s):
        for hi in range(h):
            for ti in range(t):
                want = x[si, hi, ti] if ti < prefix else oracle.rope_apply_row(x[si, hi, ti], sin, cos, ti - prefix)
                np.testing.assert_allclose(got[si, hi, ti], want, atol=1e-5, rtol=1e-5)


def test_rope_tokens_per_frame_extension():
    # With tokens_per_frame == T the extension is the reference's rope_apply;
    # with several frames each frame restarts its positions.
    sin, cos = oracle.rope_tables(2, 3)
    x = oracle.rng_uniform(9, 1 * 2 * 33 * 64).reshape(1, 2, 33, 64)
    np.testing.assert_array_equal(oracle.rope_apply(x[:, :, :11], sin, cos, 5, 11),
                                  oracle.rope_apply(x[:, :, :11], sin, cos, 5))
    multi = oracle.rope_apply(x, sin, cos, 5, 11)
    for f in range(3):
        np.testing.assert_array_equal(multi[:, :, 11 * f:11 * (f + 1)],
                                      oracle.rope_apply(x[:, :, 11 * f:11 * (f + 1)], sin, cos, 5))


# ---- LayerNorm (tests/kernels.rs:100-126) -------------------------------------

def test_layernorm_matches_naive():
    rows, dim = 19, 300
    x = oracle.rng_uniform(3, rows * dim).reshape(rows, dim)
    w = oracle.rng_uniform(103, dim)
    b = oracle.rng_uniform(203, dim)
    got = oracle.layernorm(x, w, b, 1e-5)
    np.testing.assert_allclose(got, GOLDEN["ln_19x300"], atol=1e-4, rtol=1e-4)


def test_qk_prep_is_layernorm_then_rope():
    sin, cos = oracle.rope_tables(4, 4)
    x = oracle.rng_uniform(12, 2 * 3 * 33 * 64).reshape(2, 3, 33, 64)
    w = oracle.rng_uniform(13, 64)
    b = oracle.rng_uniform(14, 64)
    want = oracle.rope_apply(oracle.layernorm(x, w, b, 1e-5), sin, cos, 17)
    np.testing.assert_array_equal(oracle.qk_prep(x, w, b, 1e-5, sin, cos, 17, 33), want)


# ---- attention (tests/kernels.rs:184-239) --------------------------------------

@pytest.mark.parametrize("t", [17, 64, 150])
def test_attention_matches_naive_softmax(t):
    s, h, d = 2, 3, 64
    vals = oracle.rng_uniform(5 + t, 3 * s * h * t * d)
    n = s * h * t * d
    q, k, v = (vals[i * n:(i + 1) * n].reshape(s, h, t, d) for i in range(3))
    got = oracle.attention(q, k, v)
    want = GOLDEN[f"attn_T{t}"]
    if t == 150:
        got = got[:, :, ::7]
    assert np.abs(got - want).max() < 1e-4


@pytest.mark.parametrize("t", [17, 150])
def test_attention_d128_matches_naive_softmax(t):
    """The camera head's head_dim-128 variant (attention.wesl with DV = 32) on the
    kernels.rs inputs, against a float64 softmax(q k^T / sqrt(128)) v."""
    s, h, d = 1, 2, 128
    vals = oracle.rng_uniform(5 + t, 3 * s * h * t * d)
    n = s * h * t * d
    q, k, v = (vals[i * n:(i + 1) * n].reshape(s, h, t, d) for i in range(3))
    got = oracle.attention(q, k, v)
    sc = np.einsum("shtd,shud->shtu", q.astype(np.float64), k.astype(np.float64)) / np.sqrt(128.0)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    want = np.einsum("shtu,shud->shtd", p / p.sum(-1, keepdims=True), v.astype(np.float64))
    assert np.abs(got - want).max() < 1e-4


def test_attention_rows_equal_full():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 3, 130, 64), np.float32) for _ in range(3))
    full = oracle.attention(q, k, v)
    rows = np.array([0, 1, 129, 130, 389, 777], np.int64)
    got = oracle.attention_rows(q, k, v, rows)
    np.testing.assert_array_equal(got, full.reshape(-1, 64)[rows])


def test_split_merge_roundtrip():
    # tests/kernels.rs:241-274
    s, t, h, d = 2, 5, 4, 8
    x = oracle.rng_uniform(6, s * t * h * d).reshape(s * t, h * d)
    heads = oracle.split_heads(x, s, t, h, d)
    for si in range(s):
        for hi in range(h):
            for ti in range(t):
                np.testing.assert_array_equal(heads[si, hi, ti], x[si * t + ti, hi * d:(hi + 1) * d])
    np.testing.assert_array_equal(oracle.attn_merge(heads), x)


# ---- storage rounding and the parity gate --------------------------------------

def test_round_to_matches_torch():
    import torch

    x = np.concatenate([oracle.rng_normal(5, 4096) * 30, [0.0, -0.0, 1e-8, 65504.0, 70000.0, 1e-5]]).astype(np.float32)
    for name, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        want = torch.from_numpy(x).to(dt).float().numpy()
        np.testing.assert_array_equal(oracle.round_to(name, x), want)


def test_gate_is_nan_proof():
    a = np.array([1.0, -2.0, 3.0, 0.5], np.float32)
    m = oracle.compare(a, a)
    assert m["max_abs"] == 0 and abs(m["cosine"] - 1) < 1e-12
    oracle.gate(m)
    with pytest.raises(AssertionError):
        oracle.gate(oracle.compare(np.full(4, np.nan, np.float32), a))
    with pytest.raises(AssertionError):
        oracle.gate(oracle.compare(-a, a))


# ---- block linears (f2): restatements of linear.wesl, gelu.wesl, residual_ls.wesl ----

def test_linear_matches_reference_known_answer():
    # tests/kernels.rs:63-98: Rng(2), (m, k, n) = (37, 53, 29), f64 reference, tol 1e-4
    # (abs + rel, kernels.rs:35-43), with and without bias.
    m, k, n = 37, 53, 29
    vals = oracle.rng_uniform(2, m * k + n * k + n)
    x = vals[:m * k].reshape(m, k)
    w = vals[m * k:m * k + n * k].reshape(n, k)
    b = vals[m * k + n * k:]
    exp = (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32) + b
    got = oracle.linear(x, w, b)
    assert np.all(np.abs(got - exp) <= 1e-4 + 1e-4 * np.abs(exp))
    got = oracle.linear(x, w)
    exp_nb = exp - b
    assert np.all(np.abs(got - exp_nb) <= 1e-4 + 1e-4 * np.abs(exp_nb))


def test_gelu_matches_erf_known_answer():
    # tests/kernels.rs:128-147: x in [-8, 8] step 0.2, within 1e-5 of the exact erf GELU.
    import math
    xs = (np.arange(-40, 41) * 0.2).astype(np.float32)
    got = oracle.gelu(xs)
    exact = np.array([0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in xs.astype(np.float64)])
    assert np.abs(got - exact).max() < 1e-5


def test_residual_ls():
    rng = np.random.default_rng(4)
    res, x = (rng.standard_normal((7, 12)).astype(np.float32) for _ in range(2))
    g = rng.standard_normal(12).astype(np.float32)
    assert np.array_equal(oracle.residual_ls(res, x, g), res + g * x)
