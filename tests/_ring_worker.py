"""One rank of the ring-attention GPU test (spawned by tests/test_ring_gpu.py).

Builds the global seeded inputs, keeps this rank's shard, runs
RingSession.attention_fused (or attention_ulysses, the head-parallel
all-to-all path) over NCCL and saves the local output."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def device_inputs(dev, T: int, H: int, dtype: str, seed: int):
    """q, k, v (1, H, T, 64) drawn on the device (torch generator, N(0,1) f32 rounded to the
    storage type): the same bytes on every GPU of this type, and fast at config 4's size."""
    import torch

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    g = torch.Generator(device=dev).manual_seed(seed)
    return tuple(torch.randn((1, H, T, 64), device=dev, generator=g).to(tdt) for _ in range(3))


def run(rank: int, world: int, port: int, outdir: str, T: int, H: int, dtype: str, seed: int, fused: bool,
        unit: int = 0, gen: str = "np", mode: str = "ring") -> None:
    """unit = 0: head-major (1, H, T_r, 64) shards of hs_shard's token rule (attention_fused);
    unit > 0: the (T_r, H*64) projection layout in shards of whole `unit`-token frames
    (attention_block).  gen = "np": inputs from numpy's generator (small cases); "torch":
    from device_inputs."""
    import torch
    import torch.distributed as dist

    import oracle
    from headshot_b200.engine import GpuContext, QkNorm, Rope
    from headshot_b200.session import RingSession

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        ctx = GpuContext(rank)
        sess = RingSession(ctx, rank, world)
        tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
        if gen == "torch":
            q, k, v = device_inputs(dev, T, H, dtype, seed)
        else:
            rng = np.random.default_rng(seed)
            q, k, v = (oracle.round_to(dtype, rng.standard_normal((1, H, T, 64), np.float32)) for _ in range(3))
        if unit:
            assert gen == "np"
            t0, t1 = sess.unit_shard(T, unit)

            def loc(a):  # (1, H, T, 64) -> this rank's (T_r, H*64) rows
                rows = oracle.attn_merge(a)[t0:t1]
                return torch.from_numpy(np.ascontiguousarray(rows)).to(dev).to(tdt)

            out = torch.empty((t1 - t0, H * 64), dtype=tdt, device=dev)
        else:
            t0, t1 = sess.shard(T)
            if gen == "torch":
                loc = lambda a: a[:, :, t0:t1].contiguous()  # noqa: E731
            else:
                loc = lambda a: torch.from_numpy(np.ascontiguousarray(a[:, :, t0:t1])).to(dev).to(tdt)  # noqa: E731
            out = torch.empty((1, H, t1 - t0, 64), dtype=tdt, device=dev)
        norm = rope = None
        if fused:
            w = torch.ones(64, device=dev)
            b = torch.zeros(64, device=dev)
            norm = QkNorm(w, b, w, b, 1e-6)
            sin, cos = oracle.rope_tables(37, 37)
            rope = Rope(torch.from_numpy(sin).to(dev), torch.from_numpy(cos).to(dev), 5, 1374)
        for _ in range(2):  # the second call reuses the ring's buffers and state
            if unit:
                sess.attention_block(loc(q), loc(k), loc(v), out, T_total=T, heads=H, shard_unit=unit,
                                     qk_norm=norm, rope=rope, check_peers=True)
            else:
                call = sess.attention_ulysses if mode == "ulysses" else sess.attention_fused
                call(loc(q), loc(k), loc(v), out, T_total=T, qk_norm=norm, rope=rope, check_peers=True)
            sess.sync(60_000)
        np.save(Path(outdir) / f"out_{rank}.npy", out.float().cpu().numpy())
        sess.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    a = sys.argv[1:]
    run(int(a[0]), int(a[1]), int(a[2]), a[3], int(a[4]), int(a[5]), a[6], int(a[7]), a[8] == "1",
        int(a[9]) if len(a) > 9 else 0, a[10] if len(a) > 10 else "np", a[11] if len(a) > 11 else "ring")
