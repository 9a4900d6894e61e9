"""CPU oracle for the attention path — TEST INFRASTRUCTURE ONLY.

ctypes bindings over headshot_oracle.c, the plain-C restatement of the
reference's f32 WGSL path (see that file's header for the file:line each
function follows).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline may import this package, and only as the checker or the timed
CPU baseline; the product library never calls it.

`build()` compiles the C source with gcc into oracle/_build/.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "headshot_oracle.c"
LIB = HERE / "_build" / "libheadshot_oracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle (no -ffast-math, no FMA contraction: f32 order as written)."""
    LIB.parent.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    cmd = [cc, "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread",
           "-fvisibility=hidden", str(SRC), "-o", str(LIB), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        u32, u64, f32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
        L.or_rng_uniform.argtypes = [u64, _f32p, u64]
        L.or_rng_normal.argtypes = [u64, _f32p, u64]
        L.or_rng_f16_exact.argtypes = [u64, _f32p, u64]
        L.or_round_to.argtypes = [ctypes.c_int, _f32p, _f32p, u64]
        L.or_rope_periods.argtypes = [_f32p]
        L.or_rope_tables.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.or_rope_apply_row.argtypes = [_f32p, _f32p, _f32p, u64, _f32p]
        L.or_rope_apply.argtypes = [_f32p, _f32p, _f32p, u32, u32, u32, u32, u32, u32]
        L.or_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, u64, u32, f32]
        L.or_qk_prep.argtypes = [_f32p, _f32p, _f32p, f32, _f32p, _f32p, ctypes.c_int, u32, u32, u32, u32, u32,
                                 u32, _f32p]
        L.or_split_heads.argtypes = [_f32p, _f32p, u32, u32, u32, u32]
        L.or_attn_merge.argtypes = [_f32p, _f32p, u32, u32, u32, u32]
        L.or_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, u32, u32, u32, u32, f32, ctypes.c_int]
        L.or_attention.restype = ctypes.c_int
        L.or_attention_rows.argtypes = [_f32p, _f32p, _f32p, _f32p, u32, u32, f32, _i64p, u64, ctypes.c_int]
        L.or_attention_rows.restype = ctypes.c_int
        L.or_linear.argtypes = [_f32p, _f32p, _f32p, _f32p, u64, u32, u32, ctypes.c_int]
        L.or_gelu.argtypes = [_f32p, _f32p, u64]
        L.or_residual_ls.argtypes = [_f32p, _f32p, _f32p, _f32p, u64, u32]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ----------------------------------------------------------------- RNG ----

def rng_uniform(seed: int, n: int) -> np.ndarray:
    """SplitMix64 -> (z>>40)/2^23*2-1 (tests/kernels.rs:7-23); spans [-1, 3) as the reference's does."""
    out = np.empty(n, np.float32)
    lib().or_rng_uniform(seed, _p(out), n)
    return out


def rng_normal(seed: int, n: int) -> np.ndarray:
    """Seeded N(0,1): SplitMix64 + Box-Muller."""
    out = np.empty(n, np.float32)
    lib().or_rng_normal(seed, _p(out), n)
    return out


def rng_f16_exact(seed: int, n: int) -> np.ndarray:
    """tests/f16_ops.rs:7-19: SplitMix64 without the final xorshift, (z>>40)/2^24*2-1 in [-1, 1),
    rounded to f16 (values every storage type holds exactly)."""
    out = np.empty(n, np.float32)
    lib().or_rng_f16_exact(seed, _p(out), n)
    return out


def round_to(dtype: str, x: np.ndarray) -> np.ndarray:
    """Round through 'f16' / 'bf16' storage (round to nearest even)."""
    code = {"f32": 0, "f16": 1, "bf16": 2}[dtype]
    x = _f32(x)
    out = np.empty_like(x)
    lib().or_round_to(code, _p(x), _p(out), x.size)
    return out


# ---------------------------------------------------------------- RoPE ----

def rope_periods() -> np.ndarray:
    out = np.empty(16, np.float32)
    lib().or_rope_periods(_p(out))
    return out


def rope_tables(h_p: int, w_p: int, periods: np.ndarray | None = None):
    per = rope_periods() if periods is None else _f32(periods)
    sin = np.empty((h_p * w_p, 64), np.float32)
    cos = np.empty((h_p * w_p, 64), np.float32)
    lib().or_rope_tables(_p(per), h_p, w_p, _p(sin), _p(cos))
    return sin, cos


def rope_apply_row(x64: np.ndarray, sin: np.ndarray, cos: np.ndarray, row: int) -> np.ndarray:
    x64 = _f32(x64)
    out = np.empty(64, np.float32)
    lib().or_rope_apply_row(_p(x64), _p(_f32(sin)), _p(_f32(cos)), row, _p(out))
    return out


def rope_apply(x: np.ndarray, sin, cos, prefix: int, tokens_per_frame: int = 0) -> np.ndarray:
    """rope_apply.wesl on a copy of x (S,H,T,D)."""
    S, H, T, D = x.shape
    out = _f32(x).copy()
    lib().or_rope_apply(_p(out), _p(_f32(sin)), _p(_f32(cos)), S, H, T, D, prefix, tokens_per_frame)
    return out


# ----------------------------------------------------------- LayerNorm ----

def layernorm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = _f32(x)
    dim = x.shape[-1]
    out = np.empty_like(x)
    lib().or_layernorm(_p(x), _p(_f32(w)), _p(_f32(b)), _p(out), x.size // dim, dim, eps)
    return out


def qk_prep(x: np.ndarray, w, b, eps: float, sin=None, cos=None, prefix: int = 0, tokens_per_frame: int = 0):
    """QK-norm then RoPE (block.rs:136-146) on (S,H,T,D)."""
    S, H, T, D = x.shape
    x = _f32(x)
    out = np.empty_like(x)
    rope_on = sin is not None
    dummy = np.zeros(64, np.float32)
    lib().or_qk_prep(_p(x), _p(_f32(w)), _p(_f32(b)), eps, _p(_f32(sin) if rope_on else dummy),
                     _p(_f32(cos) if rope_on else dummy), int(rope_on), prefix, tokens_per_frame, S, H, T, D,
                     _p(out))
    return out


# ------------------------------------------------------------ layouts -----

def split_heads(x: np.ndarray, s: int, t: int, h: int, d: int) -> np.ndarray:
    x = _f32(x)
    out = np.empty((s, h, t, d), np.float32)
    lib().or_split_heads(_p(x), _p(out), s, t, h, d)
    return out


def attn_merge(x: np.ndarray) -> np.ndarray:
    S, H, T, D = x.shape
    x = _f32(x)
    out = np.empty((S * T, H * D), np.float32)
    lib().or_attn_merge(_p(x), _p(out), S, H, T, D)
    return out


# ----------------------------------------------------------- attention ----

def attention(q, k, v, scale: float | None = None, nthreads: int | None = None) -> np.ndarray:
    """attention.wesl over (S,H,T,D) f32."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    S, H, T, D = q.shape
    out = np.empty_like(q)
    sc = float(1.0 / np.sqrt(np.float32(D))) if scale is None else scale
    rc = lib().or_attention(_p(q), _p(k), _p(v), _p(out), S, H, T, D, np.float32(sc), nthreads or threads())
    assert rc == 0
    return out


def attention_rows(q, k, v, rows, scale: float | None = None, nthreads: int | None = None) -> np.ndarray:
    """Selected query rows (flattened sh*T + t) of attention.wesl; returns (len(rows), D)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    S, H, T, D = q.shape
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((rows.size, D), np.float32)
    sc = float(1.0 / np.sqrt(np.float32(D))) if scale is None else scale
    rc = lib().or_attention_rows(_p(q), _p(k), _p(v), _p(out), T, D, np.float32(sc),
                                 rows.ctypes.data_as(_i64p), rows.size, nthreads or threads())
    assert rc == 0
    return out


# --------------------------------------------------------- parity gate ----

def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None, nthreads: int | None = None) -> np.ndarray:
    """out (M, N) = x (M, K) . w (N, K)^T [+ b] (shaders/linear.wesl)."""
    x, w = _f32(x), _f32(w)
    K = x.shape[-1]
    M = x.size // K
    N = w.shape[0]
    assert w.shape == (N, K)
    out = np.empty((M, N), np.float32)
    lib().or_linear(_p(x), _p(w), None if b is None else _p(_f32(b)), _p(out), M, K, N, nthreads or threads())
    return out


def gelu(x: np.ndarray) -> np.ndarray:
    """Erf GELU, erf by A&S 7.1.26 (shaders/gelu.wesl)."""
    x = _f32(x)
    out = np.empty_like(x)
    lib().or_gelu(_p(x), _p(out), x.size)
    return out


def residual_ls(res: np.ndarray, x: np.ndarray, gamma: np.ndarray) -> np.ndarray:
    """res + gamma * x over the last dim (shaders/residual_ls.wesl)."""
    res, x, gamma = _f32(res), _f32(x), _f32(gamma)
    out = np.empty_like(x)
    lib().or_residual_ls(_p(res), _p(x), _p(gamma), _p(out), x.size, gamma.size)
    return out


def copy_row_blocks(src: np.ndarray, dst: np.ndarray, groups: int, src_stride: int, dst_stride: int,
                    rows: int) -> np.ndarray:
    """GpuContext::copy_rows per group (trunk.rs:109-122: register gather/scatter); returns dst."""
    for g in range(groups):
        dst[g * dst_stride:g * dst_stride + rows] = src[g * src_stride:g * src_stride + rows]
    return dst


def cache_build(frame_out: np.ndarray, global_out: np.ndarray) -> np.ndarray:
    """Cache::build (cache.rs:25-52): concat_channels (concat_channels.wesl) then cast to f32
    (cast_f16_to_f32.wesl); inputs already hold the values of their storage type."""
    return np.concatenate([frame_out.astype(np.float32), global_out.astype(np.float32)], axis=-1)


def compare(ours: np.ndarray, ref: np.ndarray) -> dict:
    """src/parity.rs:35-60: max_abs, mean_abs, cosine, ref_scale in f64."""
    a = np.asarray(ours, np.float64).ravel()
    b = np.asarray(ref, np.float64).ravel()
    assert a.size == b.size and a.size > 0
    d = np.abs(a - b)
    denom = max(np.sqrt((a * a).sum()) * np.sqrt((b * b).sum()), np.finfo(np.float64).tiny)
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean()), "cosine": float((a * b).sum() / denom),
            "ref_scale": float(np.abs(b).max())}


def gate(m: dict, min_cosine: float = 0.9999, max_abs: float = 1e-2) -> None:
    """NaN-proof gate (src/parity.rs:85-103): NaN metrics always fail."""
    if not (m["cosine"] >= min_cosine):
        raise AssertionError(f"cosine {m['cosine']:.9f} !>= {min_cosine} ({m})")
    if not (m["max_abs"] <= max_abs):
        raise AssertionError(f"max_abs {m['max_abs']:.3e} !<= {max_abs} ({m})")
