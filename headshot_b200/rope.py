"""Axial 2D RoPE tables — mirror of headshot-server's engine::rope
(crates/headshot-server/src/engine/rope.rs).

`periods()` and `tables()` call the C ABI's host helpers (hs_rope_periods,
hs_rope_tables), which restate rope.rs:8-10 and :15-44 in f32.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

_fp = ctypes.POINTER(ctypes.c_float)


def periods() -> np.ndarray:
    """periods[i] = 100^(2i/32), i = 0..15 (rope.rs:8-10)."""
    out = np.empty(16, np.float32)
    _lib.check(_lib.lib().hs_rope_periods(out.ctypes.data_as(_fp)))
    return out


def tables(per: np.ndarray | None, h_p: int, w_p: int) -> tuple[np.ndarray, np.ndarray]:
    """(P, 64) sin and cos tables for an h_p x w_p patch grid (rope.rs:15-44)."""
    sin = np.empty((h_p * w_p, 64), np.float32)
    cos = np.empty((h_p * w_p, 64), np.float32)
    pp = None
    if per is not None:
        per = np.ascontiguousarray(per, np.float32)
        assert per.shape == (16,), "periods must have 16 entries"
        pp = per.ctypes.data_as(_fp)
    _lib.check(_lib.lib().hs_rope_tables(pp, h_p, w_p, sin.ctypes.data_as(_fp), cos.ctypes.data_as(_fp)))
    return sin, cos
