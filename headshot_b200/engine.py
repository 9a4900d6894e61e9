"""Host-side mirror of headshot-server's `GpuContext` attention ops.

Same op names, argument meaning and layouts as
crates/headshot-server/src/engine/ops.rs; tensors are torch CUDA tensors
(PyTorch supplies device memory and the stream — the arithmetic runs in
libheadshot_cuda.so through the C ABI).  Where the reference `assert!`s
(shape, dtype, table size) this raises AssertionError before launching;
errors reported by the library raise `HsError`.

    ctx = GpuContext()
    out = ctx.attention(q, k, v)                    # ops.rs:228-253
    q = ctx.layernorm(q, w, b)                      # ops.rs:130-153 (eps 1e-5)
    ctx.rope_apply(q, sin, cos, prefix)             # ops.rs:202-223, in place
    heads = ctx.split_heads(x, s, t, h, d)          # ops.rs:185-200
    merged = ctx.attn_merge(heads)                  # ops.rs:255-267
    out = ctx.attention_fused(q, k, v, qk_norm=QkNorm(...), rope=Rope(...))
                                                    # block.rs:136-148 as one op
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import HsError, check  # noqa: F401  (re-exported)

_DTYPES = {torch.float32: _lib.HS_F32, torch.float16: _lib.HS_F16, torch.bfloat16: _lib.HS_BF16}


def _code(t: torch.Tensor) -> int:
    assert t.dtype in _DTYPES, f"unsupported dtype {t.dtype}"
    return _DTYPES[t.dtype]


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@dataclass
class QkNorm:
    """LayerNorm(64) weights for q and k (block.rs:35-40); f32 device tensors."""

    q_w: torch.Tensor
    q_b: torch.Tensor
    k_w: torch.Tensor
    k_b: torch.Tensor
    eps: float = 1e-5


@dataclass
class Rope:
    """RoPE tables + unrotated prefix (block.rs:42-47).  `tokens_per_frame`
    extends the reference for sequences of several frames (global attention
    with per-frame positions); None means the whole sequence is one frame."""

    sin: torch.Tensor
    cos: torch.Tensor
    prefix: int
    tokens_per_frame: int | None = None


class GpuContext:
    """One device + one stream, like engine::GpuContext (src/engine/mod.rs)."""

    def __init__(self, device: int = 0):
        self._L = _lib.lib()
        h = ctypes.c_void_p()
        check(self._L.hs_ctx_create(device, ctypes.byref(h)))
        self._h = h
        self.device = torch.device("cuda", device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.hs_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def _bind_stream(self) -> None:
        # Order our launches with torch's work on the same device.
        check(self._L.hs_ctx_set_stream(self._h, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))

    def _check_tensor(self, t: torch.Tensor, name: str) -> None:
        assert t.is_cuda and t.device == self.device, f"{name} must live on {self.device}"
        assert t.is_contiguous(), f"{name} must be contiguous"

    # ------------------------------------------------------------ ops ----

    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None) -> torch.Tensor:
        """Non-causal attention over head-major (S, H, T, D); allocates `out` (ops.rs:228-253)."""
        assert q.dim() == 4, "attention wants (S,H,T,D)"
        assert q.shape == k.shape and q.shape == v.shape, "q/k/v shape mismatch"
        assert q.dtype == k.dtype == v.dtype, "q/k/v dtype mismatch"
        s, h, t, d = q.shape
        assert s * h <= 65535, "attention grid y overflow"
        for n, x in (("q", q), ("k", k), ("v", v)):
            self._check_tensor(x, n)
        out = torch.empty_like(q)
        self._bind_stream()
        check(self._L.hs_attention(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out), s, h, t, d, _code(q),
                                   0.0 if scale is None else float(scale)))
        return out

    def _prologue_args(self, d: int, t: int, qk_norm: QkNorm | None, rope: Rope | None) -> tuple:
        n_args = [None] * 4
        eps = 1e-5
        if qk_norm is not None:
            for x in (qk_norm.q_w, qk_norm.q_b, qk_norm.k_w, qk_norm.k_b):
                assert x.dtype == torch.float32 and x.numel() == d, "norm weight must be f32 (D)"
                self._check_tensor(x, "qk_norm")
            n_args = [qk_norm.q_w, qk_norm.q_b, qk_norm.k_w, qk_norm.k_b]
            eps = qk_norm.eps
        r_sin = r_cos = None
        rows = prefix = tpf = 0
        if rope is not None:
            assert rope.sin.dtype == torch.float32 and rope.cos.dtype == torch.float32, "rope tables must be f32"
            assert rope.sin.shape == rope.cos.shape and rope.sin.shape[-1] == d, "table size"
            self._check_tensor(rope.sin, "rope.sin")
            self._check_tensor(rope.cos, "rope.cos")
            r_sin, r_cos = rope.sin, rope.cos
            rows = rope.sin.numel() // d
            prefix = rope.prefix
            tpf = rope.tokens_per_frame or t
        return (*[_ptr(x) for x in n_args], float(eps), _ptr(r_sin), _ptr(r_cos), rows, prefix, tpf)

    def attention_fused(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, qk_norm: QkNorm | None = None,
                        rope: Rope | None = None, scale: float | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
        """QK-norm -> RoPE -> attention (block.rs:136-148) in one call."""
        assert q.dim() == 4, "attention wants (S,H,T,D)"
        assert q.shape == k.shape and q.shape == v.shape, "q/k/v shape mismatch"
        assert q.dtype == k.dtype == v.dtype, "q/k/v dtype mismatch"
        s, h, t, d = q.shape
        for n, x in (("q", q), ("k", k), ("v", v)):
            self._check_tensor(x, n)
        if out is None:
            out = torch.empty_like(q)
        assert out.shape == q.shape and out.dtype == q.dtype
        pro = self._prologue_args(d, t, qk_norm, rope)
        self._bind_stream()
        check(self._L.hs_attention_fused(
            self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out), s, h, t, d, _code(q),
            0.0 if scale is None else float(scale), *pro))
        return out

    def attention_block(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, s: int, t: int, heads: int,
                        qk_norm: QkNorm | None = None, rope: Rope | None = None, scale: float | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
        """Block::forward's attention section (block.rs:130-149) on the projection layout:
        q, k, v are the (S*T, H*D) outputs of the q/k/v linears; returns the (S*T, H*D)
        merged attention output (what attn_merge hands to the proj linear)."""
        assert q.shape == k.shape and q.shape == v.shape, "q/k/v shape mismatch"
        assert q.dtype == k.dtype == v.dtype, "q/k/v dtype mismatch"
        assert q.numel() % (s * t * heads) == 0, "shape"
        d = q.numel() // (s * t * heads)
        assert q.shape[-1] == heads * d and q.numel() == s * t * heads * d, "q must be (S*T, H*D)"
        for n, x in (("q", q), ("k", k), ("v", v)):
            self._check_tensor(x, n)
        if out is None:
            out = torch.empty_like(q)
        assert out.shape == q.shape and out.dtype == q.dtype
        pro = self._prologue_args(d, t, qk_norm, rope)
        self._bind_stream()
        check(self._L.hs_attention_block_fused(
            self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out), s, t, heads, d, _code(q),
            0.0 if scale is None else float(scale), *pro))
        return out

    _EPILOGUES = {"none": 0, "gelu": 1, "residual_ls": 2}

    def linear(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
               epilogue: str = "none", residual: torch.Tensor | None = None, gamma: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """out (M, N) = x (M, K) @ weight (N, K)^T [+ bias] (ops.rs:87-128), then the fused
        epilogue: "gelu" (block.rs:173-174) or "residual_ls": residual + gamma * out
        (ops.rs:168-183)."""
        k = x.shape[-1]
        m = x.numel() // k
        assert weight.dim() == 2 and weight.shape[1] == k, "weight k mismatch"
        assert weight.dtype == x.dtype, "weight/activation dtype"
        n = weight.shape[0]
        self._check_tensor(x, "x")
        self._check_tensor(weight, "weight")
        if bias is not None:
            assert bias.numel() == n, "bias len"
            assert bias.dtype == torch.float32, "bias must be f32"
            self._check_tensor(bias, "bias")
        epi = self._EPILOGUES[epilogue]
        if epi == 2:
            assert residual is not None and gamma is not None, "residual_ls needs residual and gamma"
            assert residual.numel() == m * n and residual.dtype == x.dtype
            assert gamma.dtype == torch.float32 and gamma.numel() == n, "gamma must be f32 (N)"
            self._check_tensor(residual, "residual")
            self._check_tensor(gamma, "gamma")
        if out is None:
            out = torch.empty((*x.shape[:-1], n), dtype=x.dtype, device=x.device)
        assert out.numel() == m * n and out.dtype == x.dtype
        self._bind_stream()
        check(self._L.hs_linear(self._h, _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), m, k, n, _code(x), epi,
                                _ptr(residual), _ptr(gamma)))
        return out

    def copy_row_blocks(self, src: torch.Tensor, dst: torch.Tensor, groups: int, src_stride: int, dst_stride: int,
                        rows: int) -> torch.Tensor:
        """Rows [g*src_stride, +rows) of src -> rows [g*dst_stride, +rows) of dst for g < groups
        (trunk.rs:109-122's register gather/scatter; groups=1 is copy_rows)."""
        cols = src.shape[-1]
        assert dst.shape[-1] == cols and dst.dtype == src.dtype
        assert (groups - 1) * src_stride + rows <= src.numel() // cols, "src rows"
        assert (groups - 1) * dst_stride + rows <= dst.numel() // cols, "dst rows"
        self._check_tensor(src, "src")
        self._check_tensor(dst, "dst")
        self._bind_stream()
        check(self._L.hs_copy_row_blocks(self._h, _ptr(src), _ptr(dst), groups, src_stride, dst_stride, rows, cols,
                                         _code(src)))
        return dst

    def gather_prefix(self, x: torch.Tensor, n: int, t: int, prefix: int) -> torch.Tensor:
        """(N*T, C) -> (N*prefix, C): the prefix tokens of every frame (trunk.rs:109-113)."""
        out = torch.empty((n * prefix, x.shape[-1]), dtype=x.dtype, device=x.device)
        return self.copy_row_blocks(x, out, n, t, prefix, prefix)

    def scatter_prefix(self, reg: torch.Tensor, x: torch.Tensor, n: int, t: int, prefix: int) -> torch.Tensor:
        """Writes (N*prefix, C) back over the prefix rows of every frame of x (trunk.rs:119-121)."""
        return self.copy_row_blocks(reg, x, n, prefix, t, prefix)

    def cache_build(self, frame_out: torch.Tensor, global_out: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """(rows, C1) and (rows, C2) -> (rows, C1 + C2) f32 (cache.rs:25-52); writes into out when given."""
        assert frame_out.dtype == global_out.dtype
        c1, c2 = frame_out.shape[-1], global_out.shape[-1]
        rows = frame_out.numel() // c1
        assert global_out.numel() // c2 == rows, "row mismatch"
        self._check_tensor(frame_out, "frame_out")
        self._check_tensor(global_out, "global_out")
        if out is None:
            out = torch.empty((rows, c1 + c2), dtype=torch.float32, device=frame_out.device)
        assert out.dtype == torch.float32 and out.numel() == rows * (c1 + c2), "cache shape"
        self._check_tensor(out, "out")
        self._bind_stream()
        check(self._L.hs_cache_build(self._h, _ptr(frame_out), _ptr(global_out), _ptr(out), rows, c1, c2,
                                     _code(frame_out)))
        return out

    def im2col_patch(self, images: torch.Tensor, patch: int = 16, dtype: torch.dtype = torch.float32,
                     row_stride: int | None = None, mean=(0.485, 0.456, 0.406),
                     std=(0.229, 0.224, 0.225)) -> torch.Tensor:
        """images (N, 3, H, W) f32 -> normalised patch rows (N*P, row_stride) (ops.rs:271-300);
        row_stride defaults to 3*patch*patch, wider strides are zero-padded."""
        assert images.dim() == 4 and images.shape[1] == 3, "images (N,3,H,W)"
        assert images.dtype == torch.float32, "images are uploaded f32"
        n, _, height, width = images.shape
        assert height % patch == 0 and width % patch == 0, "image sides must be multiples of the patch"
        k = 3 * patch * patch
        row_stride = k if row_stride is None else row_stride
        assert row_stride >= k
        self._check_tensor(images, "images")
        p = (height // patch) * (width // patch)
        out = torch.empty((n * p, row_stride), dtype=dtype, device=images.device)
        m = (ctypes.c_float * 3)(*mean)
        sd = (ctypes.c_float * 3)(*std)
        self._bind_stream()
        check(self._L.hs_im2col_patch(self._h, _ptr(images), _ptr(out), n, height, width, patch, row_stride,
                                      ctypes.cast(m, ctypes.c_void_p), ctypes.cast(sd, ctypes.c_void_p),
                                      _DTYPES[dtype]))
        return out

    def layernorm(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
        """Row LayerNorm over the last dim, f32 statistics (ops.rs:130-153; the reference fixes eps 1e-5)."""
        dim = x.shape[-1]
        rows = x.numel() // dim
        assert weight.numel() == dim and bias.numel() == dim
        assert weight.dtype == torch.float32, "norm weight must be f32"
        assert bias.dtype == torch.float32, "norm bias must be f32"
        for n, t in (("x", x), ("weight", weight), ("bias", bias)):
            self._check_tensor(t, n)
        out = torch.empty_like(x)
        self._bind_stream()
        check(self._L.hs_layernorm(self._h, _ptr(x), _ptr(weight), _ptr(bias), _ptr(out), rows, dim, float(eps),
                                   _code(x)))
        return out

    def rope_apply(self, x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor, prefix: int) -> None:
        """In-place RoPE on (S,H,T,D); tables (T - prefix, D) f32 (ops.rs:202-223)."""
        assert x.dim() == 4, "rope_apply wants (S,H,T,D)"
        s, h, t, d = x.shape
        assert sin.numel() == (t - prefix) * d, "table size"
        assert sin.dtype == torch.float32 and cos.dtype == torch.float32, "rope tables must be f32"
        for n, tt in (("x", x), ("sin", sin), ("cos", cos)):
            self._check_tensor(tt, n)
        self._bind_stream()
        check(self._L.hs_rope_apply(self._h, _ptr(x), _ptr(sin), _ptr(cos), t - prefix, s, h, t, d, prefix, _code(x)))

    def split_heads(self, x: torch.Tensor, s: int, t: int, h: int, d: int) -> torch.Tensor:
        """(S*T, H*D) -> head-major (S, H, T, D) (ops.rs:185-200)."""
        assert x.numel() == s * t * h * d
        self._check_tensor(x, "x")
        out = torch.empty((s, h, t, d), dtype=x.dtype, device=x.device)
        self._bind_stream()
        check(self._L.hs_split_heads(self._h, _ptr(x), _ptr(out), s, t, h, d, _code(x)))
        return out

    def attn_merge(self, x: torch.Tensor) -> torch.Tensor:
        """(S, H, T, D) -> (S*T, H*D) (ops.rs:255-267)."""
        assert x.dim() == 4, "attn_merge wants (S,H,T,D)"
        s, h, t, d = x.shape
        self._check_tensor(x, "x")
        out = torch.empty((s * t, h * d), dtype=x.dtype, device=x.device)
        self._bind_stream()
        check(self._L.hs_attn_merge(self._h, _ptr(x), _ptr(out), s, h, t, d, _code(x)))
        return out

    def sync(self) -> None:
        """Wait for the stream; raises HsError(HS_ERR_TIMEOUT) if an in-kernel wait gave up."""
        self._bind_stream()
        check(self._L.hs_sync(self._h))

    def set_wait_timeout_ms(self, ms: int) -> None:
        check(self._L.hs_ctx_set_wait_timeout_ms(self._h, int(ms)))

    # ---------------------------------------------------- profiling ----

    def prof_enable(self, on: bool = True) -> None:
        """Bracket every launch with CUDA events on its stream."""
        check(self._L.hs_prof_enable(self._h, 1 if on else 0))

    def prof_reset(self) -> None:
        check(self._L.hs_prof_reset(self._h))

    def prof_read(self, kernel: str = "*") -> tuple[float, int]:
        """(summed device ms, launches) of `kernel` since the last reset."""
        ms = ctypes.c_double()
        n = ctypes.c_uint64()
        check(self._L.hs_prof_read(self._h, kernel.encode(), ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    # ------------------------------------------- host <-> device (C ABI) --

    def upload(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        """hs_memcpy_h2d of a contiguous host tensor into a device tensor."""
        assert src.numel() * src.element_size() == dst.numel() * dst.element_size()
        self._bind_stream()
        check(self._L.hs_memcpy_h2d(self._h, _ptr(dst), _ptr(src), dst.numel() * dst.element_size()))

    def download(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        """hs_memcpy_d2h of a device tensor into a contiguous host tensor."""
        assert src.numel() * src.element_size() == dst.numel() * dst.element_size()
        self._bind_stream()
        check(self._L.hs_memcpy_d2h(self._h, _ptr(dst), _ptr(src), dst.numel() * dst.element_size()))
