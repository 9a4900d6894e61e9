"""Host-side pieces of the aggregator that need no GPU: the oracle's im2col
against the shader's own index decode (im2col_patch.wesl:33-58), the FLOP
count the frames/s roofline uses, and the register-layer all-gather of the
frame-sharded trunk over gloo ranks."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import model as omodel
from headshot_b200.aggregator import AggregatorConfig, _all_gather_frames
from headshot_b200.session import shard_bounds


def test_im2col_matches_shader_decode():
    rng = np.random.default_rng(0)
    n, ps, h, w = 2, 4, 8, 12
    images = rng.random((n, 3, h, w), dtype=np.float32)
    mean, std = np.float32([0.1, 0.2, 0.3]), np.float32([0.5, 0.25, 0.125])
    got = omodel.im2col_patch(images, ps, mean, std)
    row_len = 3 * ps * ps
    wp, hp = w // ps, h // ps
    want = np.empty(n * hp * wp * row_len, np.float32)
    for i in range(want.size):  # im2col_patch.wesl:43-57, one invocation per output element
        col = i % row_len
        kx, ky, c = col % ps, (col // ps) % ps, col // (ps * ps)
        patch = i // row_len
        pc, pr, f = patch % wp, (patch // wp) % hp, patch // (wp * hp)
        value = images[f, c, pr * ps + ky, pc * ps + kx]
        want[i] = (value - mean[c]) * (np.float32(1) / std[c])
    assert np.array_equal(got.ravel(), want)


def test_patch_k_is_padded_to_16_bytes():
    assert AggregatorConfig(patch=14).k_patch == 592
    assert AggregatorConfig(patch=16).k_patch == 768


def test_flops_match_the_config5_figures():
    """A global layer at 100 frames x 1374 tokens is 7.73e13 attention FLOPs, a frame
    layer 7.73e11 (the hot-path scope table's config 5 row)."""
    cfg = AggregatorConfig()
    from headshot_b200.aggregator import Aggregator

    f = Aggregator.flops(type("A", (), {"cfg": cfg})(), 100, 518, 518)
    t = 37 * 37 + 5
    glob = 4 * 16 * (100 * t) ** 2 * 64
    assert abs(glob - 7.73e13) / 7.73e13 < 0.01
    assert cfg.register_layers == () and cfg.trunk_pairs == 24  # config 5: 24 global layers
    assert f["attention"] > 24 * glob
    assert f["total"] == f["gemm"] + f["attention"]
    shared = AggregatorConfig.headshot_shared()
    assert shared.register_layers == (2, 6, 9, 14, 20)
    fs = Aggregator.flops(type("A", (), {"cfg": shared})(), 100, 518, 518)
    assert 19 * glob < fs["attention"] < 20 * glob


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank: int, world: int, port: int, n_total: int, pre: int, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        f0, f1 = shard_bounds(n_total, world, rank)
        # frame f's prefix row j holds f * 100 + j in every column
        rows = torch.tensor([[float(f * 100 + j)] * 8 for f in range(f0, f1) for j in range(pre)])
        out = _all_gather_frames(rows, n_total, None)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_total", [(2, 5), (3, 7)])
def test_register_all_gather_keeps_frame_order(world, n_total):
    pre = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n_total, pre, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.array([[float(f * 100 + j)] * 8 for f in range(n_total) for j in range(pre)], np.float32)
    for r in range(world):
        assert np.array_equal(results[r], want)
