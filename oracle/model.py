"""CPU restatement of the aggregator's model code — TEST INFRASTRUCTURE ONLY.

Composes the oracle's op restatements (headshot_oracle.c via this package)
in the order headshot-server's model code calls its ops, with every op's
result rounded to the storage type as the reference's storage would hold it:

- `block_forward`  follows Block::forward (src/model/block.rs:121-159) and
                   Block::mlp's single-shot path (block.rs:166-175);
- `dino_forward`   follows Dino::forward (src/model/dino.rs:58-118);
- `trunk_forward`  follows Trunk::forward (src/model/trunk.rs:55-146) and
                   Cache::build (src/model/cache.rs:25-52);
- `im2col_patch`   follows im2col_patch.wesl (normalise, (c, ky, kx) order).

Weights are plain dicts of numpy arrays (the values the GPU side holds).
Only tests/ may call this module, as the checker.
"""
from __future__ import annotations

import numpy as np

from . import (attention, attn_merge, cache_build, gelu, layernorm, linear, residual_ls, rope_apply, rope_tables,
               round_to, split_heads)


def im2col_patch(images: np.ndarray, patch: int, mean, std, row_stride: int | None = None) -> np.ndarray:
    """images (N, 3, H, W) -> (N*P, row_stride) f32 rows, column c*ps*ps + ky*ps + kx
    (im2col_patch.wesl:33-58); columns past 3*ps*ps are zero."""
    n, c, h, w = images.shape
    hp, wp = h // patch, w // patch
    x = (images.astype(np.float32) - np.asarray(mean, np.float32)[None, :, None, None]) \
        * (np.float32(1) / np.asarray(std, np.float32))[None, :, None, None]
    x = x.reshape(n, c, hp, patch, wp, patch).transpose(0, 2, 4, 1, 3, 5).reshape(n * hp * wp, c * patch * patch)
    k = c * patch * patch
    out = np.zeros((n * hp * wp, row_stride or k), np.float32)
    out[:, :k] = x
    return out


def block_forward(x: np.ndarray, w: dict, s: int, t: int, heads: int, eps: float, store: str,
                  rope: tuple | None = None) -> np.ndarray:
    """Block::forward on (S*T, C) rows; `rope` = (sin, cos, prefix)."""
    r = lambda a: round_to(store, a)  # noqa: E731
    c = x.shape[-1]
    d = c // heads
    normed = r(layernorm(x, w["norm1_w"], w["norm1_b"], eps))
    q, k, v = (split_heads(r(linear(normed, w["qkv_w"][i], w["qkv_b"][i])), s, t, heads, d) for i in range(3))
    if w.get("qk_norm") is not None:
        qw, qb, kw, kb, qk_eps = w["qk_norm"]
        q = r(layernorm(q, qw, qb, qk_eps))
        k = r(layernorm(k, kw, kb, qk_eps))
    if rope is not None:
        sin, cos, prefix = rope
        q = r(rope_apply(q, sin, cos, prefix))
        k = r(rope_apply(k, sin, cos, prefix))
    merged = attn_merge(r(attention(q, k, v)))
    proj = r(linear(merged, w["proj_w"], w["proj_b"]))
    x1 = r(residual_ls(x, proj, w["ls1"]))
    normed2 = r(layernorm(x1, w["norm2_w"], w["norm2_b"], eps))
    hidden = r(gelu(r(linear(normed2, w["fc1_w"], w["fc1_b"]))))
    mlp = r(linear(hidden, w["fc2_w"], w["fc2_b"]))
    return r(residual_ls(x1, mlp, w["ls2"]))


def dino_forward(images: np.ndarray, w: dict, cfg, store: str, taps: dict | None = None) -> np.ndarray:
    """Dino::forward: images (N, 3, H, W) -> patch tokens (N*P, C)."""
    n, _, h, wd = images.shape
    hp, wp = h // cfg.patch, wd // cfg.patch
    p, pre = hp * wp, cfg.dino_prefix
    t = p + pre
    cols = round_to(store, im2col_patch(images, cfg.patch, w["mean"], w["std"], cfg.k_patch))
    emb = round_to(store, linear(cols, w["proj_w"], w["proj_b"]))
    x = np.empty((n * t, cfg.dim), np.float32)
    for i in range(n):
        x[i * t] = w["cls_token"][0]
        x[i * t + 1:i * t + pre] = w["storage_tokens"]
        x[i * t + pre:(i + 1) * t] = emb[i * p:(i + 1) * p]
    sin, cos = rope_tables(hp, wp)
    for i, bw in enumerate(w["blocks"]):
        x = block_forward(x, bw, n, t, cfg.heads, cfg.norm_eps, store, (sin, cos, pre))
        if taps is not None:
            taps[f"dino.block.{i:02}"] = x
    normed = round_to(store, layernorm(x, w["norm_w"], w["norm_b"], cfg.norm_eps))
    out = np.concatenate([normed[i * t + pre:(i + 1) * t] for i in range(n)])
    if taps is not None:
        taps["dino.tokens"] = out
    return out


def trunk_forward(tokens: np.ndarray, w: dict, cfg, n: int, hp: int, wp: int, store: str,
                  taps: dict | None = None) -> list:
    """Trunk::forward: (N*P, C) patch tokens -> the f32 caches of cfg.cached_layers."""
    p, pre = hp * wp, cfg.trunk_prefix
    t = p + pre
    reg = pre - 1
    x = np.empty((n * t, cfg.dim), np.float32)
    for i in range(n):
        variant = int(i != 0)
        x[i * t] = w["camera_token"][variant]
        x[i * t + 1:i * t + pre] = w["register_token"][variant * reg:(variant + 1) * reg]
        x[i * t + pre:(i + 1) * t] = tokens[i * p:(i + 1) * p]
    sin, cos = rope_tables(hp, wp)
    caches = []
    for k in range(cfg.trunk_pairs):
        frame_out = block_forward(x, w["frame_blocks"][k], n, t, cfg.heads, cfg.norm_eps, store, (sin, cos, pre))
        if taps is not None:
            taps[f"trunk.frame.{k:02}"] = frame_out
        if k in cfg.register_layers:
            regs = np.concatenate([frame_out[i * t:i * t + pre] for i in range(n)])
            reg_out = block_forward(regs, w["inter_blocks"][k], 1, n * pre, cfg.heads, cfg.norm_eps, store)
            if taps is not None:
                taps[f"trunk.inter.{k:02}"] = reg_out
            frame_out = frame_out.copy()
            for i in range(n):
                frame_out[i * t:i * t + pre] = reg_out[i * pre:(i + 1) * pre]
            x = frame_out
        else:
            inter_out = block_forward(frame_out, w["inter_blocks"][k], 1, n * t, cfg.heads, cfg.norm_eps, store)
            if taps is not None:
                taps[f"trunk.inter.{k:02}"] = inter_out
            if k in cfg.cached_layers:
                caches.append(cache_build(frame_out, inter_out))
            x = inter_out
    return caches
