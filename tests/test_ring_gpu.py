"""Ring (sequence-parallel) global attention on 2+ GPUs against the oracle.

Each rank is a separate process on its own GPU (tests/_ring_worker.py); the
concatenated shard outputs must match the oracle's single-sequence
attention within the parity gate.  Skipped with fewer than 2 GPUs.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


# unit 0: head-major shards of the token rule; unit > 0: projection-layout rows in shards of
# whole frames (the frame-sharded trunk's global blocks), uneven when frames % world != 0.
@pytest.mark.parametrize("world,T,fused,dtype,unit", [(2, 2748, True, "bf16", 0), (2, 2748, True, "f16", 0),
                                                      (2, 1001, False, "f16", 0), (2, 4122, True, "bf16", 1374),
                                                      (2, 1001, False, "bf16", 143)])
def test_ring_matches_oracle(tmp_path, world, T, fused, dtype, unit):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    H, seed = 2, 17
    port = _free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(HERE / "_ring_worker.py"), str(r), str(world), str(port),
                               str(tmp_path), str(T), str(H), dtype, str(seed), "1" if fused else "0", str(unit)],
                              env=env)
             for r in range(world)]
    rcs = [p.wait(timeout=600) for p in procs]
    assert rcs == [0] * world, f"worker exit codes {rcs}"
    parts = [np.load(tmp_path / f"out_{r}.npy") for r in range(world)]
    if unit:
        out = oracle.split_heads(np.concatenate(parts, axis=0), 1, T, H, 64)
    else:
        out = np.concatenate(parts, axis=2)

    rng = np.random.default_rng(seed)
    q, k, v = (oracle.round_to(dtype, rng.standard_normal((1, H, T, 64), np.float32)) for _ in range(3))
    if fused:
        w, b = np.ones(64, np.float32), np.zeros(64, np.float32)
        sin, cos = oracle.rope_tables(37, 37)
        q = oracle.qk_prep(q, w, b, 1e-6, sin, cos, 5, 1374)
        k = oracle.qk_prep(k, w, b, 1e-6, sin, cos, 5, 1374)
    ref = oracle.attention(q, k, v)
    oracle.gate(oracle.compare(out, ref), 0.9999, 1e-2)
