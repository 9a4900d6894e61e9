"""Multi-GPU session layer for the aggregator's attention (new: the
reference is single-device, src/model/trunk.rs:92-144).

- Frame attention shards by frame: rank r owns frames shard_bounds(N, R, r)
  and needs no communication (each frame is an independent sequence).
- Global attention shards the sequence: rank r owns tokens
  shard_bounds(T, R, r) of q, k and v (all heads) and runs the ring in
  libheadshot_cuda.so (hs_ring_attention_fused): [K'|V] blocks rotate over
  NCCL send/recv while the tcgen05 kernel works on the previous block,
  carrying the f32 softmax state in-kernel.  Or by head parallelism
  (hs_ring_ulysses_attention_fused): an all-to-all gives each rank the
  whole sequence of H / world heads, one attention launch, an all-to-all
  back.

Failure detection: before each ring call every rank joins a small host
"preflight" collective on the session's process group; a rank that has
left (exited, raised) makes it fail within the group's timeout, so the
others raise before any NCCL ring traffic is queued.  `sync()` waits with
hs_ring_sync's watchdog, which aborts the NCCL communicator on an async
error or timeout.
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import check

_vp, _u32, _f32, _i = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float, ctypes.c_int

RING_SIGNATURES = {
    "hs_ring_shard": (_i, [_u32, _i, _i, ctypes.POINTER(_u32), ctypes.POINTER(_u32)]),
    "hs_ring_plan": (_i, [_i, _i, _i] + [ctypes.POINTER(_i)] * 5),
    "hs_ring_id_bytes": (ctypes.c_size_t, []),
    "hs_ring_unique_id": (_i, [_vp]),
    "hs_ring_create": (_i, [_vp, _i, _i, _vp, ctypes.POINTER(_vp)]),
    "hs_ring_destroy": (_i, [_vp]),
    "hs_ring_attention_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp, _vp, _f32,
                                     _vp, _vp, _u32, _u32, _u32]),
    "hs_ring_attention_block_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp, _vp,
                                           _f32, _vp, _vp, _u32, _u32, _u32, _u32]),
    "hs_ring_ulysses_attention_fused": (_i, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _i, _f32, _vp, _vp, _vp, _vp,
                                             _f32, _vp, _vp, _u32, _u32, _u32]),
    "hs_ring_sync": (_i, [_vp, _u32]),
    "hs_ring_set_reserved_sms": (_i, [_vp, _u32]),
}


def _L():
    L = _lib.lib()
    for name, (res, args) in RING_SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of n items; the first n % world ranks get one extra."""
    assert world >= 1 and 0 <= rank < world
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def ring_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """hs_ring_shard: the C library's shard rule (same as shard_bounds)."""
    s, ln = _u32(), _u32()
    check(_L().hs_ring_shard(n, world, rank, ctypes.byref(s), ctypes.byref(ln)))
    return s.value, s.value + ln.value


def ring_plan(rank: int, world: int, step: int) -> dict:
    """hs_ring_plan: the block a rank attends to at `step`, its peers and state flags."""
    v = [_i() for _ in range(5)]
    check(_L().hs_ring_plan(rank, world, step, *[ctypes.byref(x) for x in v]))
    src, send_to, recv_from, load, store = (x.value for x in v)
    return {"src": src, "send_to": send_to, "recv_from": recv_from, "load": bool(load), "store": bool(store)}


def preflight(group=None, timeout_s: float | None = None) -> None:
    """Host check that every rank of `group` is still in the session.

    A one-element all_reduce on the session's group: if a peer has left,
    the collective fails (gloo: connection closed; NCCL: group timeout) and
    this raises before the caller queues ring traffic."""
    import torch
    import torch.distributed as dist

    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    flag = torch.ones(1, dtype=torch.int32, device=dev)
    work = dist.all_reduce(flag, group=group, async_op=True)
    if timeout_s is None:
        work.wait()
    else:
        from datetime import timedelta

        work.wait(timeout=timedelta(seconds=timeout_s))
    if int(flag.item()) != dist.get_world_size(group):
        raise RuntimeError("session preflight: a rank did not join")


class RingSession:
    """One rank of a ring over `world` GPUs (one process per GPU)."""

    def __init__(self, ctx, rank: int, world: int, group=None):
        import torch
        import torch.distributed as dist

        self.ctx, self.rank, self.world, self.group = ctx, rank, world, group
        L = _L()
        n = L.hs_ring_id_bytes()
        buf = ctypes.create_string_buffer(n)
        if rank == 0:
            check(L.hs_ring_unique_id(buf))
        backend = dist.get_backend(group)
        dev = ctx.device if backend == "nccl" else torch.device("cpu")
        t = torch.frombuffer(bytearray(buf.raw), dtype=torch.uint8).to(dev)
        dist.broadcast(t, src=0, group=group)
        uid = bytes(t.cpu().numpy().tobytes())
        h = ctypes.c_void_p()
        check(L.hs_ring_create(ctx.handle, rank, world, ctypes.c_char_p(uid), ctypes.byref(h)))
        self._h = h
        self._L = L

    def shard(self, t_total: int) -> tuple[int, int]:
        return ring_shard(t_total, self.world, self.rank)

    def attention_fused(self, q, k, v, out, T_total: int, qk_norm=None, rope=None, scale: float | None = None,
                        check_peers: bool = False):
        """Ring global attention on this rank's shard: q, k, v, out (H, T_r, 64) or (1, H, T_r, 64)."""
        return self._global(self._L.hs_ring_attention_fused, q, k, v, out, T_total, qk_norm, rope, scale,
                            check_peers)

    def _global(self, fn, q, k, v, out, T_total, qk_norm, rope, scale, check_peers):
        import torch

        from .engine import _code, _ptr

        if check_peers:
            preflight(self.group)
        h = q.shape[-3]
        t0, t1 = self.shard(T_total)
        assert q.shape[-2] == t1 - t0, f"rank {self.rank} owns {t1 - t0} tokens, q has {q.shape[-2]}"
        for x in (q, k, v, out):
            assert x.shape == q.shape and x.dtype == q.dtype and x.is_contiguous()
        n_args = [None] * 4
        eps = 1e-5
        if qk_norm is not None:
            n_args = [qk_norm.q_w, qk_norm.q_b, qk_norm.k_w, qk_norm.k_b]
            eps = qk_norm.eps
        r_sin = r_cos = None
        rows = prefix = tpf = 0
        if rope is not None:
            r_sin, r_cos = rope.sin, rope.cos
            rows = rope.sin.numel() // 64
            prefix = rope.prefix
            tpf = rope.tokens_per_frame or T_total
        check(self._L.hs_ctx_set_stream(self.ctx.handle,
                                        ctypes.c_void_p(torch.cuda.current_stream(self.ctx.device).cuda_stream)))
        check(fn(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out), h, T_total, 64, _code(q),
                 0.0 if scale is None else float(scale), *[_ptr(x) for x in n_args], float(eps), _ptr(r_sin),
                 _ptr(r_cos), rows, prefix, tpf))
        return out

    def attention_ulysses(self, q, k, v, out, T_total: int, qk_norm=None, rope=None, scale: float | None = None,
                          check_peers: bool = False):
        """attention_fused's contract by head parallelism (hs_ring_ulysses_attention_fused): an
        all-to-all gathers the whole sequence of H / world heads on each rank, one attention launch,
        an all-to-all back.  H must be a multiple of the world size."""
        return self._global(self._L.hs_ring_ulysses_attention_fused, q, k, v, out, T_total, qk_norm, rope, scale,
                            check_peers)

    def unit_shard(self, t_total: int, unit: int) -> tuple[int, int]:
        """Token range of this rank when shards are whole `unit`s of tokens (whole frames)."""
        assert t_total % unit == 0, "t_total must be a multiple of the shard unit"
        u0, u1 = shard_bounds(t_total // unit, self.world, self.rank)
        return u0 * unit, u1 * unit

    def attention_block(self, q, k, v, out, T_total: int, heads: int, shard_unit: int = 1, qk_norm=None, rope=None,
                        scale: float | None = None, check_peers: bool = False):
        """Ring global attention on Block::forward's layout: q, k, v are this rank's (T_r, H*64) q/k/v
        linear outputs, out its (T_r, H*64) merged output; shards are whole `shard_unit`s of tokens
        (hs_ring_attention_block_fused)."""
        import torch

        from .engine import _code, _ptr

        if check_peers:
            preflight(self.group)
        t0, t1 = self.unit_shard(T_total, shard_unit)
        assert q.shape[-1] == heads * 64 and q.numel() == (t1 - t0) * heads * 64, \
            f"rank {self.rank} owns {t1 - t0} tokens of (T, {heads * 64})"
        for x in (q, k, v, out):
            assert x.shape == q.shape and x.dtype == q.dtype and x.is_contiguous()
        pro = self.ctx._prologue_args(64, T_total, qk_norm, rope)
        check(self._L.hs_ctx_set_stream(self.ctx.handle,
                                        ctypes.c_void_p(torch.cuda.current_stream(self.ctx.device).cuda_stream)))
        check(self._L.hs_ring_attention_block_fused(
            self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(out), heads, T_total, 64, _code(q),
            0.0 if scale is None else float(scale), *pro, shard_unit))
        return out

    def set_reserved_sms(self, sms: int) -> None:
        """SMs the ring's attention launches leave free for the transfer of the next block."""
        check(self._L.hs_ring_set_reserved_sms(self._h, int(sms)))

    def sync(self, timeout_ms: int = 120_000) -> None:
        check(self._L.hs_ring_sync(self._h, int(timeout_ms)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.hs_ring_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
