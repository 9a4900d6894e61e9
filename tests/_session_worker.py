"""One CPU rank of the session-layer tests (gloo), spawned by
tests/test_session_cpu.py.

mode "ring": runs the ring schedule of libheadshot_cuda.so (hs_ring_plan,
hs_ring_shard — host functions) with [K|V] blocks exchanged over gloo, and a
numpy model of the kernel's per-step math (scores in the log2 domain,
carried running max / sum / unnormalised O in f64).  The result must equal
the oracle's attention for this rank's query rows.

mode "preflight": rank 1 leaves right after joining; rank 0's
session.preflight() must raise instead of waiting forever.

mode "drop": the ring's block exchange with one message dropped (the last
rank leaves instead of sending); the other ranks' exchanges must fail.
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

LOG2E = 1.4426950408889634


def step_model(q, kb, vb, state, scale):
    """One ring step for one head: q (Tq, D), kb/vb (Tk, D); state (o, m, l) or None."""
    s = (q.astype(np.float64) @ kb.astype(np.float64).T) * scale * LOG2E
    m_blk = s.max(1)
    if state is None:
        m = m_blk
        o = np.zeros((q.shape[0], vb.shape[1]))
        l = np.zeros(q.shape[0])
    else:
        o, m_old, l = state
        m = np.maximum(m_old, m_blk)
        corr = np.exp2(m_old - m)
        o = o * corr[:, None]
        l = l * corr
    p = np.exp2(s - m[:, None])
    return o + p @ vb.astype(np.float64), m, l + p.sum(1)


def ring(rank: int, world: int) -> int:
    import torch
    import torch.distributed as dist

    import oracle
    from headshot_b200 import session

    H, T, D = 2, 301, 64
    rng = np.random.default_rng(42)
    q, k, v = (rng.standard_normal((1, H, T, D)).astype(np.float32) for _ in range(3))
    t0, t1 = session.ring_shard(T, world, rank)
    ql = q[0, :, t0:t1]
    block = (rank, np.ascontiguousarray(k[0, :, t0:t1]), np.ascontiguousarray(v[0, :, t0:t1]))
    states = [None] * H
    scale = 1.0 / np.sqrt(D)
    for step in range(world):
        plan = session.ring_plan(rank, world, step)
        bid, kb, vb = block
        assert bid == plan["src"], f"rank {rank} step {step}: holds block {bid}, plan says {plan['src']}"
        assert (states[0] is not None) == plan["load"]
        for h in range(H):
            states[h] = step_model(ql[h], kb[h], vb[h], states[h], scale)
        if plan["send_to"] >= 0:
            nsrc = (plan["src"] - 1) % world
            n0, n1 = session.ring_shard(T, world, nsrc)
            send = torch.from_numpy(np.concatenate([kb.ravel(), vb.ravel()]))
            recv = torch.empty(2 * H * (n1 - n0) * D, dtype=torch.float32)
            ops = [dist.P2POp(dist.isend, send, plan["send_to"]), dist.P2POp(dist.irecv, recv, plan["recv_from"])]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            r = recv.numpy()
            half = H * (n1 - n0) * D
            block = (nsrc, r[:half].reshape(H, n1 - n0, D), r[half:].reshape(H, n1 - n0, D))
    out = np.stack([o / l[:, None] for o, _, l in states])  # (H, Tr, D)
    rows = np.array([h * T + t for h in range(H) for t in range(t0, t1)], np.int64)
    want = oracle.attention_rows(q, k, v, rows, nthreads=1).reshape(H, t1 - t0, D)
    err = float(np.abs(out - want).max())
    if err > 1e-4:
        print(f"rank {rank}: max err {err}", flush=True)
        return 1
    return 0


def preflight(rank: int, world: int) -> int:
    import torch.distributed as dist

    from headshot_b200 import session

    if rank == 1:
        os._exit(0)  # leaves the session between steps, nothing in flight
    try:
        session.preflight(timeout_s=10.0)
    except Exception as e:  # noqa: BLE001
        print(f"rank 0: preflight raised {type(e).__name__}", flush=True)
        return 0
    print("rank 0: preflight did not notice the departed rank", flush=True)
    return 1


def drop(rank: int, world: int) -> int:
    """The last rank drops the [K|V] block it owes its successor after step 0
    and leaves; every other rank must see its next exchange fail (an
    exception within the group timeout) instead of waiting forever."""
    import torch
    import torch.distributed as dist

    from headshot_b200 import session

    H, T, D = 2, 64, 64
    t0, t1 = session.ring_shard(T, world, rank)
    block = torch.full((2 * H * (t1 - t0) * D,), float(rank))
    try:
        for step in range(world - 1):
            plan = session.ring_plan(rank, world, step)
            if rank == world - 1 and step == 0:
                os._exit(0)  # the message to send_to is dropped; this rank is gone
            n0, n1 = session.ring_shard(T, world, (plan["src"] - 1) % world)
            recv = torch.empty(2 * H * (n1 - n0) * D)
            ops = [dist.P2POp(dist.isend, block, plan["send_to"]), dist.P2POp(dist.irecv, recv, plan["recv_from"])]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            block = recv
    except Exception as e:  # noqa: BLE001
        print(f"rank {rank}: exchange failed with {type(e).__name__}", flush=True)
        return 0
    print(f"rank {rank}: every exchange completed although a rank dropped its block", flush=True)
    return 1


def main() -> int:
    mode, rank, world, port = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    timeout = timedelta(seconds=10 if mode == "drop" else 20)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    if mode == "ring":
        rc = ring(rank, world)
        dist.destroy_process_group()
        return rc
    rc = preflight(rank, world) if mode == "preflight" else drop(rank, world)
    os._exit(rc)


if __name__ == "__main__":
    sys.exit(main())
