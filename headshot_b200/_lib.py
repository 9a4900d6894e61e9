"""ctypes loader for libheadshot_cuda.so — the package's only native path.

There is no fallback: if the library is missing or fails to load, every op
raises.  Build it with `python -m headshot_b200.build` (or
`__graft_entry__.build()`).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libheadshot_cuda.so"
HEADER = PKG.parent / "include" / "headshot_cuda.h"

HS_OK, HS_ERR_INVALID, HS_ERR_UNSUPPORTED, HS_ERR_CUDA, HS_ERR_OOM, HS_ERR_TIMEOUT, HS_ERR_NCCL, HS_ERR_CANCELLED = range(8)
HS_F32, HS_F16, HS_BF16 = 0, 1, 2

STATUS_NAMES = {
    HS_OK: "HS_OK",
    HS_ERR_INVALID: "HS_ERR_INVALID",
    HS_ERR_UNSUPPORTED: "HS_ERR_UNSUPPORTED",
    HS_ERR_CUDA: "HS_ERR_CUDA",
    HS_ERR_OOM: "HS_ERR_OOM",
    HS_ERR_TIMEOUT: "HS_ERR_TIMEOUT",
    HS_ERR_NCCL: "HS_ERR_NCCL",
    HS_ERR_CANCELLED: "HS_ERR_CANCELLED",
}


class HsError(RuntimeError):
    """A non-OK hs_status from the C ABI, with hs_last_error()'s message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


_vp, _u32, _u64, _f32, _i = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int
_fp = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); mirrors include/headshot_cuda.h
SIGNATURES = {
    "hs_abi_version": (_u32, []),
    "hs_last_error": (ctypes.c_char_p, []),
    "hs_ctx_create": (_i, [_i, ctypes.POINTER(_vp)]),
    "hs_ctx_destroy": (_i, [_vp]),
    "hs_ctx_set_stream": (_i, [_vp, _vp]),
    "hs_ctx_use_own_stream": (_i, [_vp]),
    "hs_ctx_stream": (_vp, [_vp]),
    "hs_ctx_set_wait_timeout_ms": (_i, [_vp, _u32]),
    "hs_ctx_request_cancel": (_i, [_vp]),
    "hs_ctx_clear_cancel": (_i, [_vp]),
    "hs_prof_enable": (_i, [_vp, _i]),
    "hs_prof_reset": (_i, [_vp]),
    "hs_prof_read": (_i, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_u64)]),
    "hs_alloc": (_i, [_vp, ctypes.c_size_t, ctypes.POINTER(_vp)]),
    "hs_free": (_i, [_vp, _vp]),
    "hs_memset": (_i, [_vp, _vp, _i, ctypes.c_size_t]),
    "hs_memcpy_h2d": (_i, [_vp, _vp, _vp, ctypes.c_size_t]),
    "hs_memcpy_d2h": (_i, [_vp, _vp, _vp, ctypes.c_size_t]),
    "hs_sync": (_i, [_vp]),
    "hs_attention": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i, _f32]),
    "hs_attention_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp, _vp, _f32,
                                _vp, _vp, _u32, _u32, _u32]),
    "hs_attention_block_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp,
                                      _vp, _f32, _vp, _vp, _u32, _u32, _u32]),
    "hs_linear": (_i, [_vp, _vp, _vp, _vp, _vp, _u64, _u32, _u32, _i, _i, _vp, _vp]),
    "hs_copy_row_blocks": (_i, [_vp, _vp, _vp, _u64, _u64, _u64, _u64, _u32, _i]),
    "hs_cache_build": (_i, [_vp, _vp, _vp, _vp, _u64, _u32, _u32, _i]),
    "hs_im2col_patch": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _i]),
    "hs_layernorm": (_i, [_vp, _vp, _vp, _vp, _vp, _u64, _u32, _f32, _i]),
    "hs_rope_apply": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _i]),
    "hs_split_heads": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _i]),
    "hs_attn_merge": (_i, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _i]),
    "hs_rope_periods": (_i, [_fp]),
    "hs_rope_tables": (_i, [_fp, _u32, _u32, _fp, _fp]),
}

_lib: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Every function name include/headshot_cuda.h declares."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hs_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """The loaded CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: the CUDA path is required (no CPU fallback). "
                "Build it with `python -m headshot_b200.build`.")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().hs_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != HS_OK:
        raise HsError(status, last_error())
