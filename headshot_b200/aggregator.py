"""The VGGT aggregator forward on libheadshot_cuda.so's ops.

Host-side mirror of headshot-server's model code, op for op:

- `Block.forward`   -> Block::forward (src/model/block.rs:121-159)
- `Dino.forward`    -> Dino::forward  (src/model/dino.rs:58-118)
- `Trunk.forward`   -> Trunk::forward (src/model/trunk.rs:55-146)
- caches            -> Cache::build   (src/model/cache.rs:25-52)

Each block is seven library calls: hs_layernorm, three hs_linear (q, k, v),
hs_attention_block_fused (split_heads + QK-norm + RoPE + attention +
attn_merge, block.rs:130-149), hs_linear with the LayerScale-residual
epilogue (proj, ops.rs:168-183), hs_layernorm, hs_linear with the GELU
epilogue (fc1) and hs_linear with the LayerScale residual (fc2).  Token
assembly, the register-layer gather/scatter and the head-input caches are
hs_copy_row_blocks / hs_cache_build; the patch embedding is hs_im2col_patch
followed by hs_linear.

Multi-GPU (one process per GPU): frames are sharded across ranks
(`shard_bounds(N, R, r)`), so DINO, the frame blocks, every linear and
LayerNorm, and the caches run on the rank's own frames with no
communication.  A global block's attention runs as the ring
(`RingSession.attention_block`, shards of whole frames); a register layer
gathers the prefix tokens of all ranks (torch.distributed all_gather, a few
hundred KB), runs that small block on every rank and keeps its own rows.

Weights are random (the checkpoint is not available): N(0, init_std) for
linear weights, class/camera/register tokens; zero biases; LayerNorm weight
1 and bias 0; LayerScale gammas `ls_init` (N(0, 0.02),
LayerScale 1e-5), drawn from a seeded torch generator on the device.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Callable

import torch

from . import rope as _rope
from .engine import GpuContext, QkNorm, Rope
from .session import shard_bounds

# headshot-shared model.rs:25-28
REGISTER_ATTENTION_LAYERS = (2, 6, 9, 14, 20)
CACHED_LAYERS = (4, 11, 17, 23)
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)

Tap = Callable[[str, torch.Tensor], None]


class Cancelled(RuntimeError):
    """Raised between blocks after `Aggregator.cancel()` (engine::Cancelled, src/engine/mod.rs:102-106)."""


@dataclass(frozen=True)
class AggregatorConfig:
    """Architecture of one aggregator.  The defaults are BASELINE config 5 (VGGT-1B at
    518x518: patch 14 -> 37x37 patches, 1 camera + 4 register tokens per frame, 24
    frame-attention / global-attention block pairs, no register-only layers).
    `headshot_shared()` is the reference server's own trunk layout: five of the 24
    inter-frame layers attend over the prefix tokens only (headshot-shared
    src/model.rs:25, trunk.rs:105-122).  The reference checkpoint's own token layout is
    patch 16, DINO prefix 5, trunk prefix 17."""

    dim: int = 1024
    heads: int = 16
    mlp_hidden: int = 4096
    patch: int = 14
    dino_layers: int = 24
    dino_prefix: int = 5  # cls + storage tokens (dino.rs:11)
    trunk_pairs: int = 24
    trunk_prefix: int = 5  # camera + register tokens (trunk.rs:15)
    register_layers: tuple = ()
    cached_layers: tuple = CACHED_LAYERS
    norm_eps: float = 1e-5  # ctx.layernorm's fixed eps (ops.rs:139)
    qk_eps: float = 1e-6
    init_std: float = 0.02
    ls_init: float = 1e-5

    @classmethod
    def headshot_shared(cls, **overrides) -> "AggregatorConfig":
        """The reference server's trunk: register-only attention at layers 2, 6, 9, 14, 20
        (headshot-shared src/model.rs:25-28), 19 global layers."""
        return cls(**{"register_layers": REGISTER_ATTENTION_LAYERS, **overrides})

    @property
    def k_patch(self) -> int:
        """Patch GEMM K: 3*patch^2 rounded up to 8 elements (16-byte rows); im2col zero-fills the rest."""
        return (3 * self.patch * self.patch + 7) // 8 * 8


@dataclass
class BlockWeights:
    """One pre-norm transformer block (block.rs:12-33); GEMM weights in the storage
    dtype, norms, biases and gammas f32."""

    norm1_w: torch.Tensor
    norm1_b: torch.Tensor
    qkv_w: list  # q, k, v: (dim, dim) each (block.rs:15-18)
    qkv_b: list
    proj_w: torch.Tensor
    proj_b: torch.Tensor
    ls1: torch.Tensor
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor
    fc1_w: torch.Tensor
    fc1_b: torch.Tensor
    fc2_w: torch.Tensor
    fc2_b: torch.Tensor
    ls2: torch.Tensor
    qk_norm: QkNorm | None

    @staticmethod
    def random(cfg: AggregatorConfig, qk_norm: bool, dtype: torch.dtype, gen: torch.Generator,
               device: torch.device) -> "BlockWeights":
        d, hid = cfg.dim, cfg.mlp_hidden
        hd = d // cfg.heads

        def w(n, k):
            return (torch.randn((n, k), generator=gen, device=device) * cfg.init_std).to(dtype)

        def f(n, v):
            return torch.full((n,), float(v), dtype=torch.float32, device=device)

        qn = None
        if qk_norm:
            qn = QkNorm(f(hd, 1), f(hd, 0), f(hd, 1), f(hd, 0), eps=cfg.qk_eps)
        return BlockWeights(
            norm1_w=f(d, 1), norm1_b=f(d, 0),
            qkv_w=[w(d, d) for _ in range(3)], qkv_b=[f(d, 0) for _ in range(3)],
            proj_w=w(d, d), proj_b=f(d, 0), ls1=f(d, cfg.ls_init),
            norm2_w=f(d, 1), norm2_b=f(d, 0),
            fc1_w=w(hid, d), fc1_b=f(hid, 0), fc2_w=w(d, hid), fc2_b=f(d, 0), ls2=f(d, cfg.ls_init),
            qk_norm=qn)


class Block:
    """Block::forward (block.rs:121-159): x += LS1(Attn(LN(x))); x += LS2(MLP(LN(x)))."""

    def __init__(self, w: BlockWeights, heads: int, norm_eps: float):
        self.w, self.heads, self.eps = w, heads, norm_eps

    def forward(self, ctx: GpuContext, x: torch.Tensor, s: int, t: int, rope: Rope | None = None,
                ring=None, t_total: int | None = None, shard_unit: int = 1) -> torch.Tensor:
        """x (S*T, C); attention runs as S sequences of T tokens.  With `ring`, x holds this
        rank's rows of one sequence of `t_total` tokens sharded in whole `shard_unit`s."""
        w = self.w
        normed = ctx.layernorm(x, w.norm1_w, w.norm1_b, self.eps)
        q, k, v = (ctx.linear(normed, w.qkv_w[i], w.qkv_b[i]) for i in range(3))
        if ring is None:
            merged = ctx.attention_block(q, k, v, s, t, self.heads, qk_norm=w.qk_norm, rope=rope)
        else:
            assert s == 1 and rope is None, "ring attention: one global sequence, no RoPE (trunk.rs:124-125)"
            merged = torch.empty_like(q)
            ring.attention_block(q, k, v, merged, t_total, self.heads, shard_unit=shard_unit, qk_norm=w.qk_norm)
        del q, k, v
        x1 = ctx.linear(merged, w.proj_w, w.proj_b, epilogue="residual_ls", residual=x, gamma=w.ls1)
        del merged
        normed2 = ctx.layernorm(x1, w.norm2_w, w.norm2_b, self.eps)
        hidden = ctx.linear(normed2, w.fc1_w, w.fc1_b, epilogue="gelu")
        del normed2
        return ctx.linear(hidden, w.fc2_w, w.fc2_b, epilogue="residual_ls", residual=x1, gamma=w.ls2)


def _rope_tables(ctx: GpuContext, h_p: int, w_p: int, prefix: int, tokens_per_frame: int) -> Rope:
    sin, cos = _rope.tables(None, h_p, w_p)
    dev = ctx.device
    return Rope(torch.from_numpy(sin).to(dev), torch.from_numpy(cos).to(dev), prefix, tokens_per_frame)


class Dino:
    """Dino::forward (dino.rs:58-118): patch embed, cls + storage tokens, RoPE blocks, final norm."""

    def __init__(self, cfg: AggregatorConfig, dtype: torch.dtype, gen: torch.Generator, device: torch.device):
        self.cfg, self.dtype = cfg, dtype
        d = cfg.dim
        k = 3 * cfg.patch * cfg.patch
        proj = torch.randn((d, k), generator=gen, device=device) * cfg.init_std
        # Conv weight (dim, 3, ps, ps) flattened, K padded with zero columns to 16-byte rows.
        self.proj_w = torch.zeros((d, cfg.k_patch), dtype=dtype, device=device)
        self.proj_w[:, :k] = proj.to(dtype)
        self.proj_b = torch.zeros(d, dtype=torch.float32, device=device)
        self.cls_token = (torch.randn((1, d), generator=gen, device=device) * cfg.init_std).to(dtype)
        self.storage_tokens = (torch.randn((cfg.dino_prefix - 1, d), generator=gen, device=device)
                               * cfg.init_std).to(dtype)
        self.blocks = [Block(BlockWeights.random(cfg, False, dtype, gen, device), cfg.heads, cfg.norm_eps)
                       for _ in range(cfg.dino_layers)]
        self.norm_w = torch.ones(d, dtype=torch.float32, device=device)
        self.norm_b = torch.zeros(d, dtype=torch.float32, device=device)

    def forward(self, ctx: GpuContext, images: torch.Tensor, tap: Tap | None = None,
                check: Callable[[], None] | None = None) -> torch.Tensor:
        """images (N, 3, H, W) f32 in [0, 1] -> patch tokens (N*P, dim)."""
        cfg = self.cfg
        n, _, height, width = images.shape
        h_p, w_p = height // cfg.patch, width // cfg.patch
        p, pre = h_p * w_p, cfg.dino_prefix
        t = p + pre
        cols = ctx.im2col_patch(images, cfg.patch, self.dtype, cfg.k_patch, IMAGENET_MEAN, IMAGENET_STD)
        embedded = ctx.linear(cols, self.proj_w, self.proj_b)
        del cols
        if tap:
            tap("dino.patch_embed", embedded)
        x = torch.empty((n * t, cfg.dim), dtype=self.dtype, device=images.device)
        ctx.copy_row_blocks(self.cls_token, x, n, 0, t, 1)
        ctx.copy_row_blocks(self.storage_tokens, x[1:], n, 0, t, pre - 1)
        ctx.copy_row_blocks(embedded, x[pre:], n, p, t, p)
        del embedded
        rope = _rope_tables(ctx, h_p, w_p, pre, t)
        for i, blk in enumerate(self.blocks):
            if check:
                check()
            x = blk.forward(ctx, x, n, t, rope)
            if tap:
                tap(f"dino.block.{i:02}", x)
        normed = ctx.layernorm(x, self.norm_w, self.norm_b, cfg.norm_eps)
        out = torch.empty((n * p, cfg.dim), dtype=self.dtype, device=images.device)
        ctx.copy_row_blocks(normed[pre:], out, n, t, p, p)
        if tap:
            tap("dino.tokens", out)
        return out


class Trunk:
    """Trunk::forward (trunk.rs:55-146): 24 frame-block / inter-frame-block pairs."""

    def __init__(self, cfg: AggregatorConfig, dtype: torch.dtype, gen: torch.Generator, device: torch.device):
        self.cfg, self.dtype = cfg, dtype
        d, reg = cfg.dim, cfg.trunk_prefix - 1
        # variant 0: frame 0, variant 1: the other frames (trunk.rs:19-20)
        self.camera_token = (torch.randn((2, d), generator=gen, device=device) * cfg.init_std).to(dtype)
        self.register_token = (torch.randn((2 * reg, d), generator=gen, device=device) * cfg.init_std).to(dtype)
        self.frame_blocks = [Block(BlockWeights.random(cfg, True, dtype, gen, device), cfg.heads, cfg.norm_eps)
                             for _ in range(cfg.trunk_pairs)]
        self.inter_blocks = [Block(BlockWeights.random(cfg, True, dtype, gen, device), cfg.heads, cfg.norm_eps)
                             for _ in range(cfg.trunk_pairs)]

    def _assemble(self, ctx: GpuContext, tokens: torch.Tensor, n: int, p: int, frame0: int) -> torch.Tensor:
        cfg = self.cfg
        pre, reg = cfg.trunk_prefix, cfg.trunk_prefix - 1
        t = p + pre
        x = torch.empty((n * t, cfg.dim), dtype=self.dtype, device=tokens.device)
        first = 1 if frame0 == 0 else 0  # global frame 0 takes variant 0 (trunk.rs:78-84)
        if first:
            ctx.copy_row_blocks(self.camera_token[0:1], x, 1, 0, t, 1)
            ctx.copy_row_blocks(self.register_token[0:reg], x[1:], 1, 0, t, reg)
        if n > first:
            rest = x[first * t:]
            ctx.copy_row_blocks(self.camera_token[1:2], rest, n - first, 0, t, 1)
            ctx.copy_row_blocks(self.register_token[reg:2 * reg], rest[1:], n - first, 0, t, reg)
        ctx.copy_row_blocks(tokens, x[pre:], n, p, t, p)
        return x

    def forward(self, ctx: GpuContext, tokens: torch.Tensor, n: int, h_p: int, w_p: int, tap: Tap | None = None,
                check: Callable[[], None] | None = None, ring=None, group=None, n_total: int | None = None,
                frame0: int = 0) -> list:
        """tokens (n*P, dim) -> the head-input caches (n*T, 2*dim) f32 of `cached_layers`.
        With `ring`, the n frames are this rank's frames [frame0, frame0 + n) of n_total."""
        cfg = self.cfg
        p, pre = h_p * w_p, cfg.trunk_prefix
        t = p + pre
        n_total = n if n_total is None else n_total
        x = self._assemble(ctx, tokens, n, p, frame0)
        rope = _rope_tables(ctx, h_p, w_p, pre, t)
        caches = []
        for k in range(cfg.trunk_pairs):
            if check:
                check()
            frame_out = self.frame_blocks[k].forward(ctx, x, n, t, rope)
            if tap:
                tap(f"trunk.frame.{k:02}", frame_out)
            if k in cfg.register_layers:
                reg = ctx.gather_prefix(frame_out, n, t, pre)
                if ring is None:
                    reg_out = self.inter_blocks[k].forward(ctx, reg, 1, n * pre)
                else:
                    all_reg = _all_gather_frames(reg, n_total, group)
                    all_out = self.inter_blocks[k].forward(ctx, all_reg, 1, n_total * pre)
                    reg_out = all_out[frame0 * pre:(frame0 + n) * pre]
                if tap:
                    tap(f"trunk.inter.{k:02}", reg_out)
                ctx.scatter_prefix(reg_out.contiguous(), frame_out, n, t, pre)
                x = frame_out
            else:
                if ring is None:
                    inter_out = self.inter_blocks[k].forward(ctx, frame_out, 1, n * t)
                else:
                    inter_out = self.inter_blocks[k].forward(ctx, frame_out, 1, n * t, ring=ring,
                                                             t_total=n_total * t, shard_unit=t)
                if tap:
                    tap(f"trunk.inter.{k:02}", inter_out)
                if k in cfg.cached_layers:
                    cache = ctx.cache_build(frame_out, inter_out)
                    if tap:
                        tap(f"cache.{k:02}", cache)
                    caches.append(cache)
                x = inter_out
            del frame_out
        return caches


def _all_gather_frames(rows: torch.Tensor, n_total: int, group) -> torch.Tensor:
    """Concatenate every rank's per-frame rows in frame order (ranks own contiguous frames,
    shard_bounds); all_gather wants equal sizes, so shares are padded to the largest."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    counts = [shard_bounds(n_total, world, r) for r in range(world)]
    per = rows.shape[0] // max(counts[rank][1] - counts[rank][0], 1)
    most = max(b - a for a, b in counts) * per
    buf = torch.zeros((most, rows.shape[1]), dtype=rows.dtype, device=rows.device)
    buf[:rows.shape[0]] = rows
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][:(b - a) * per] for r, (a, b) in enumerate(counts)]).contiguous()


class Aggregator:
    """DINO + trunk (BASELINE config 5's "full aggregator forward"), random weights."""

    def __init__(self, cfg: AggregatorConfig = AggregatorConfig(), dtype: torch.dtype = torch.bfloat16,
                 seed: int = 4, device: torch.device | int = 0):
        device = torch.device("cuda", device) if isinstance(device, int) else device
        gen = torch.Generator(device=device).manual_seed(seed)
        self.cfg, self.dtype = cfg, dtype
        self.dino = Dino(cfg, dtype, gen, device)
        self.trunk = Trunk(cfg, dtype, gen, device)
        self._cancel = threading.Event()

    def cancel(self) -> None:
        """Request cancellation; forward raises Cancelled before its next block."""
        self._cancel.set()

    def _check(self) -> None:
        if self._cancel.is_set():
            self._cancel.clear()
            raise Cancelled("aggregator forward cancelled")

    def forward(self, ctx: GpuContext, images: torch.Tensor, tap: Tap | None = None, ring=None, group=None,
                n_total: int | None = None, frame0: int = 0) -> list:
        """images (n, 3, H, W) f32 in [0, 1] -> the caches of `cfg.cached_layers`, each
        (n*T, 2*dim) f32.  With `ring`, images are this rank's frames [frame0, frame0 + n)."""
        cfg = self.cfg
        n, _, height, width = images.shape
        h_p, w_p = height // cfg.patch, width // cfg.patch
        tokens = self.dino.forward(ctx, images, tap, self._check)
        return self.trunk.forward(ctx, tokens, n, h_p, w_p, tap, self._check, ring=ring, group=group,
                                  n_total=n_total, frame0=frame0)

    def flops(self, n: int, height: int, width: int) -> dict:
        """Algorithmic FLOPs of one forward over n frames: GEMMs (2*M*N*K) and attention (4*T^2*D per
        head-sequence), the figures the frames/s roofline is built on."""
        cfg = self.cfg
        p = (height // cfg.patch) * (width // cfg.patch)
        d, hid = cfg.dim, cfg.mlp_hidden
        block_gemm = lambda rows: 2 * rows * (4 * d * d + 2 * d * hid)  # noqa: E731
        attn = lambda s, t: 4 * s * cfg.heads * t * t * (d // cfg.heads)  # noqa: E731
        td, tt = p + cfg.dino_prefix, p + cfg.trunk_prefix
        gemm = 2 * n * p * cfg.k_patch * d + cfg.dino_layers * block_gemm(n * td)
        att = cfg.dino_layers * attn(n, td)
        for k in range(cfg.trunk_pairs):
            gemm += block_gemm(n * tt)
            att += attn(n, tt)
            if k in cfg.register_layers:
                gemm += block_gemm(n * cfg.trunk_prefix)
                att += attn(1, n * cfg.trunk_prefix)
            else:
                gemm += block_gemm(n * tt)
                att += attn(1, n * tt)
        return {"gemm": gemm, "attention": att, "total": gemm + att}
