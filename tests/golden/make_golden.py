"""Generates tests/golden/golden.npz — independent restatements used to pin
the C oracle (oracle/headshot_oracle.c).

Everything here is written separately from the oracle, in pure Python
integers (SplitMix64) and numpy (f32 tables, f64 naive softmax), following
the reference's own CPU references:

  rng_*           tests/kernels.rs:7-23       SplitMix64 -> (z>>40)/2^23*2-1
  periods         src/engine/rope.rs:8-10     100^(2i/32)
  sin_2x3/cos_*   src/engine/rope.rs:15-44    axial tables
  attn_T*         tests/kernels.rs:184-239    naive full-matrix softmax (here f64)
  ln_*            tests/kernels.rs:100-126    naive two-pass LayerNorm (here f64)

The Rust/WGSL reference cannot run in this container (no Rust toolchain, no
Vulkan), so these fixtures restate its CPU-side references rather than
dumping its outputs.  Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "golden.npz"
MASK = (1 << 64) - 1


def splitmix_uniform(seed: int, n: int) -> np.ndarray:
    s = seed & MASK
    out = np.empty(n, np.float32)
    for i in range(n):
        s = (s + 0x9E3779B97F4A7C15) & MASK
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
        z ^= z >> 31
        out[i] = np.float32(np.float32(z >> 40) / np.float32(1 << 23)) * np.float32(2.0) - np.float32(1.0)
    return out


def periods() -> np.ndarray:
    return np.array([np.float32(100.0) ** np.float32(2.0 * i / 32.0) for i in range(16)], np.float32)


def tables(h_p: int, w_p: int):
    per = periods()
    side = np.float32(max(h_p, w_p))
    tau = np.float32(2.0 * np.pi)
    sin = np.zeros((h_p * w_p, 64), np.float32)
    cos = np.zeros((h_p * w_p, 64), np.float32)
    coord = lambda i: np.float32(2.0) * ((np.float32(i) + np.float32(0.5)) / side) - np.float32(1.0)  # noqa: E731
    for r in range(h_p):
        for c in range(w_p):
            idx = r * w_p + c
            for i in range(16):
                ah = tau * coord(r) / per[i]
                aw = tau * coord(c) / per[i]
                for off, a in ((0, ah), (16, aw)):
                    for half in (0, 32):
                        sin[idx, half + off + i] = np.sin(a, dtype=np.float32)
                        cos[idx, half + off + i] = np.cos(a, dtype=np.float32)
    return sin, cos


def naive_attention(q, k, v) -> np.ndarray:
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = np.einsum("shqd,shkd->shqk", q, k) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.einsum("shqk,shkd->shqd", p, v).astype(np.float32)


def naive_layernorm(x, w, b, eps=1e-5) -> np.ndarray:
    x = x.astype(np.float64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return ((x - mu) / np.sqrt(var + eps) * w + b).astype(np.float32)


def main() -> None:
    g = {}
    for seed in (1, 3, 4, 22, 69, 155):
        g[f"rng_{seed}"] = splitmix_uniform(seed, 64)
    g["periods"] = periods()
    g["sin_2x3"], g["cos_2x3"] = tables(2, 3)
    g["sin_4x4"], g["cos_4x4"] = tables(4, 4)
    s, h, d = 2, 3, 64
    for t in (17, 64, 150):
        vals = splitmix_uniform(5 + t, 3 * s * h * t * d)
        n = s * h * t * d
        q, k, v = (vals[i * n:(i + 1) * n].reshape(s, h, t, d) for i in range(3))
        out = naive_attention(q, k, v)
        g[f"attn_T{t}"] = out if t < 150 else out[:, :, ::7]
    rows, dim = 19, 300
    x = splitmix_uniform(3, rows * dim).reshape(rows, dim)
    w = splitmix_uniform(103, dim)
    b = splitmix_uniform(203, dim)
    g["ln_x_seed"] = np.array([3, 103, 203])
    g["ln_19x300"] = naive_layernorm(x, w, b)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
