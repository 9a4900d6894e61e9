"""The aggregator forward on the GPU against the oracle's composition of the
reference's model code (oracle/model.py: Block::forward, Dino::forward,
Trunk::forward, Cache::build), plus the ops it added: the patch-embedding
im2col (im2col_patch.wesl), the model-width LayerNorm path and the
broadcast row copy that assembles the per-frame prefix tokens."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import model as omodel
from headshot_b200.aggregator import Aggregator, AggregatorConfig, Cancelled
from headshot_b200.engine import GpuContext

pytestmark = pytest.mark.gpu
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().to(TORCH[dtype])


def host(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("patch,hw,stride", [(14, (56, 42), 592), (16, (64, 32), 768), (14, (28, 28), 600)])
def test_im2col_patch(gpu_ctx: GpuContext, dtype, patch, hw, stride):
    rng = np.random.default_rng(patch + stride)
    images = rng.random((3, 3, *hw), dtype=np.float32)
    mean, std = (0.485, 0.456, 0.406), (0.229, 0.224, 0.225)
    out = gpu_ctx.im2col_patch(torch.from_numpy(images).cuda(), patch, TORCH[dtype], stride, mean, std)
    ref = omodel.im2col_patch(images, patch, mean, std, stride)
    if dtype != "f32":
        ref = oracle.round_to(dtype, ref)
    gpu_ctx.sync()
    assert out.shape == ref.shape
    assert np.array_equal(host(out), ref)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("dim", [256, 768, 1024, 2048])
def test_layernorm_model_width(gpu_ctx, dtype, dim):
    """Rows of the model width take the register-resident path (dim = 256*C); same
    tolerance as the reference's LayerNorm test (kernels.rs:100-126) for f32."""
    rows = 1031
    x = oracle.rng_uniform(dim, rows * dim).reshape(rows, dim) * 3.0
    if dtype != "f32":
        x = oracle.round_to(dtype, x)
    w = oracle.rng_uniform(dim + 1, dim)
    b = oracle.rng_uniform(dim + 2, dim)
    ref = oracle.layernorm(x, w, b, 1e-6)
    out = gpu_ctx.layernorm(dev(x, dtype), torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda(), 1e-6)
    gpu_ctx.sync()
    tol = 1e-4 if dtype == "f32" else 2e-2 * max(1.0, float(np.abs(ref).max()))
    assert np.abs(host(out) - ref).max() <= tol


def test_broadcast_row_copy(gpu_ctx):
    """src_stride 0: the same source rows land in every group (per-frame prefix tokens)."""
    n, t, c = 5, 21, 64
    tok = torch.randn((4, c), device="cuda").to(torch.bfloat16)
    x = torch.zeros((n * t, c), device="cuda", dtype=torch.bfloat16)
    gpu_ctx.copy_row_blocks(tok, x[1:], n, 0, t, 4)
    exp = oracle.copy_row_blocks(host(tok), np.zeros((n * t, c), np.float32)[1:], n, 0, t, 4)
    gpu_ctx.sync()
    assert np.array_equal(host(x)[1:], exp)
    assert not host(x)[0].any()


def _weights_np(agg: Aggregator) -> tuple[dict, dict]:
    def a(t):
        return t.float().cpu().numpy()

    def blk(b):
        w = b.w
        qn = None if w.qk_norm is None else (a(w.qk_norm.q_w), a(w.qk_norm.q_b), a(w.qk_norm.k_w),
                                             a(w.qk_norm.k_b), w.qk_norm.eps)
        return {"norm1_w": a(w.norm1_w), "norm1_b": a(w.norm1_b), "qkv_w": [a(x) for x in w.qkv_w],
                "qkv_b": [a(x) for x in w.qkv_b], "proj_w": a(w.proj_w), "proj_b": a(w.proj_b), "ls1": a(w.ls1),
                "norm2_w": a(w.norm2_w), "norm2_b": a(w.norm2_b), "fc1_w": a(w.fc1_w), "fc1_b": a(w.fc1_b),
                "fc2_w": a(w.fc2_w), "fc2_b": a(w.fc2_b), "ls2": a(w.ls2), "qk_norm": qn}

    d = agg.dino
    dino = {"proj_w": a(d.proj_w), "proj_b": a(d.proj_b), "cls_token": a(d.cls_token),
            "storage_tokens": a(d.storage_tokens), "blocks": [blk(b) for b in d.blocks], "norm_w": a(d.norm_w),
            "norm_b": a(d.norm_b), "mean": (0.485, 0.456, 0.406), "std": (0.229, 0.224, 0.225)}
    t = agg.trunk
    trunk = {"camera_token": a(t.camera_token), "register_token": a(t.register_token),
             "frame_blocks": [blk(b) for b in t.frame_blocks], "inter_blocks": [blk(b) for b in t.inter_blocks]}
    return dino, trunk


# Small aggregators with every kind of layer: RoPE frame blocks, global blocks, a
# register layer, cached layers.  LayerScale 0.5 so each block moves the residual
# stream (at the model's 1e-5 a bf16 residual would absorb the branches).
SMALL = {
    "baseline_layout": (AggregatorConfig(dim=256, heads=4, mlp_hidden=1024, patch=14, dino_layers=2, dino_prefix=5,
                                         trunk_pairs=3, trunk_prefix=5, register_layers=(1,), cached_layers=(0, 2),
                                         ls_init=0.5), (56, 56), 3),
    "checkpoint_layout": (AggregatorConfig(dim=128, heads=2, mlp_hidden=512, patch=16, dino_layers=1,
                                           dino_prefix=5, trunk_pairs=2, trunk_prefix=17, register_layers=(0,),
                                           cached_layers=(1,), ls_init=0.5), (64, 48), 2),
}


def small_images(n: int, h: int, w: int) -> np.ndarray:
    return np.random.default_rng(11).random((n, 3, h, w), dtype=np.float32)


def _oracle_caches(agg: Aggregator, images: np.ndarray, taps: dict | None = None) -> list:
    cfg = agg.cfg
    n, _, h, w = images.shape
    dino_w, trunk_w = _weights_np(agg)
    tokens = omodel.dino_forward(images, dino_w, cfg, "bf16", taps)
    return omodel.trunk_forward(tokens, trunk_w, cfg, n, h // cfg.patch, w // cfg.patch, "bf16", taps)


def _close(ours: np.ndarray, ref: np.ndarray, what) -> None:
    # bf16 storage after every op and a few layers deep: cosine >= 0.999 and max |diff|
    # within 5 % of the tensor's scale (one ulp of bf16 is 0.4-0.8 %).
    m = oracle.compare(ours, ref)
    assert m["cosine"] >= 0.999 and m["max_abs"] <= 0.05 * max(1.0, m["ref_scale"]), (what, m)


@pytest.mark.parametrize("name", sorted(SMALL))
def test_aggregator_matches_oracle(gpu_ctx, name):
    cfg, (h, w), n = SMALL[name]
    agg = Aggregator(cfg, torch.bfloat16, seed=7, device=0)
    images = small_images(n, h, w)
    taps = {}

    def tap(key, t):
        taps[key] = host(t)

    caches = agg.forward(gpu_ctx, torch.from_numpy(images).cuda(), tap=tap)
    gpu_ctx.sync()
    ref_taps = {}
    ref_caches = _oracle_caches(agg, images, ref_taps)
    assert len(caches) == len(ref_caches) == len(cfg.cached_layers)
    for key in ["dino.tokens"] + [k for k in ref_taps if k.startswith("trunk.")]:
        _close(taps[key], ref_taps[key], key)
    for ours, ref in zip(caches, ref_caches):
        assert ours.dtype == torch.float32 and tuple(ours.shape) == ref.shape
        _close(host(ours), ref, "cache")


@pytest.mark.parametrize("name", sorted(SMALL))
def test_aggregator_frame_sharded_ring(tmp_path, name):
    """Two ranks (one process per GPU): frames sharded unevenly (2 + 1 or 1 + 1), global
    blocks on the ring in whole-frame shards, register layers on the all-gathered prefix
    rows; the rows of both ranks' caches must match the oracle's single-device forward."""
    import os
    import socket
    import subprocess
    import sys
    from pathlib import Path

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    here = Path(__file__).resolve().parent
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(here / "_aggregator_worker.py"), str(r), str(world), str(port),
                               str(tmp_path), name], env=env) for r in range(world)]
    rcs = [p.wait(timeout=600) for p in procs]
    assert rcs == [0] * world, f"worker exit codes {rcs}"
    cfg, (h, w), n = SMALL[name]
    agg = Aggregator(cfg, torch.bfloat16, seed=7, device=0)
    ref_caches = _oracle_caches(agg, small_images(n, h, w))
    for i, ref in enumerate(ref_caches):
        ours = np.concatenate([np.load(tmp_path / f"cache{i}_{r}.npy") for r in range(world)])
        assert ours.shape == ref.shape
        _close(ours, ref, f"cache {i}")


def test_aggregator_cancel(gpu_ctx):
    cfg = SMALL["checkpoint_layout"][0]
    agg = Aggregator(cfg, torch.bfloat16, seed=1, device=0)
    images = torch.rand((1, 3, 32, 32), device="cuda")
    agg.cancel()
    with pytest.raises(Cancelled):
        agg.forward(gpu_ctx, images)
    caches = agg.forward(gpu_ctx, images)  # the request is consumed; the next forward runs
    assert len(caches) == len(cfg.cached_layers)
