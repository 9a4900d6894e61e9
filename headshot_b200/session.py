"""Multi-GPU session layer for the aggregator's attention (new: the
reference is single-device, src/model/trunk.rs:92-144).

- Frame attention shards by frame: rank r owns frames shard_bounds(N, R, r)
  and needs no communication.
- Global attention shards the sequence: rank r owns tokens
  shard_bounds(T, R, r) of q, k and v and runs the ring implemented in
  libheadshot_cuda.so (hs_ring_attention_fused).
"""
from __future__ import annotations


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of n items; the first n % world ranks get one extra."""
    assert world >= 1 and 0 <= rank < world
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)
