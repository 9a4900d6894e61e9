"""One rank of the frame-sharded aggregator GPU test (spawned by
tests/test_aggregator_gpu.py): the rank's frames through DINO and the trunk,
global blocks on the ring, register layers on the all-gathered prefix rows;
saves the rank's caches."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def run(rank: int, world: int, port: int, outdir: str, name: str) -> None:
    import torch
    import torch.distributed as dist

    from headshot_b200.aggregator import Aggregator
    from headshot_b200.engine import GpuContext
    from headshot_b200.session import RingSession, shard_bounds
    from tests.test_aggregator_gpu import SMALL, small_images

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        cfg, (h, w), n = SMALL[name]
        ctx = GpuContext(rank)
        sess = RingSession(ctx, rank, world)
        agg = Aggregator(cfg, torch.bfloat16, seed=7, device=dev)
        f0, f1 = shard_bounds(n, world, rank)
        images = torch.from_numpy(small_images(n, h, w)[f0:f1]).to(dev)
        caches = agg.forward(ctx, images, ring=sess, n_total=n, frame0=f0)
        sess.sync(60_000)
        for i, c in enumerate(caches):
            np.save(Path(outdir) / f"cache{i}_{rank}.npy", c.cpu().numpy())
        sess.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    a = sys.argv[1:]
    run(int(a[0]), int(a[1]), int(a[2]), a[3], a[4])
