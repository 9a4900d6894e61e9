#!/usr/bin/env python
"""bench.py — aggregator attention on B200 through libheadshot_cuda.so.

Default workload (the metric's "global attention at 200
frames"): one non-causal sequence of 200 x 1374 = 274,800 tokens, 16 heads
x 64, bf16 q/k/v ~ N(0,1) (seed 3), fused QK-LayerNorm (w=1, b=0, eps 1e-6)
and per-frame 2D RoPE (37x37 grid, 5 special tokens unrotated).  A step is
one hs_attention_fused call over the whole sequence; at N GPUs it is the
ring-parallel session call over N sequence shards (strong scaling).

`--workload frame` runs config 3 (200 frames of 1374 tokens, fp16, frames
sharded across ranks) and `--workload global43k` config 2.

Prints ONE JSON line on rank 0.  `--impl reference` times the CPU
restatement of the reference's f32 attention (oracle/, a port: the Rust/WGSL
reference cannot run here) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "global-attn TFLOP/s (% bf16 peak) at 200 frames, 1/2/4/8 GPU; aggregator frames/s"

WORKLOADS = {
    "global": dict(S=1, H=16, frames=200, T_f=1374, dtype="bf16", seed=3, prefix=5, grid=(37, 37), eps=1e-6,
                   name="global attention, 200 frames x 1374 tokens = 274,800 tokens, 16 heads x 64, bf16, "
                        "fused QK-LayerNorm + per-frame 2D RoPE (37x37, 5 special tokens), non-causal"),
    "global43k": dict(S=1, H=16, frames=32, T_f=1374, dtype="bf16", seed=1, prefix=5, grid=(37, 37), eps=1e-6,
                      name="global attention, 32 frames x 1374 = 43,968 tokens, 16 heads x 64, bf16, "
                           "fused QK-LayerNorm + per-frame 2D RoPE, non-causal"),
    "frame": dict(S=200, H=16, frames=1, T_f=1374, dtype="f16", seed=2, prefix=5, grid=(37, 37), eps=1e-6,
                  name="batched frame attention, 200 frames x 1374 tokens, 16 heads x 64, fp16, "
                       "fused QK-LayerNorm + 2D RoPE (37x37, 5 special tokens)"),
    # The same two workloads with a QK-norm gain that lifts the score bound past the
    # fixed-offset limit (bf16 48, f16 14), so the kernel runs its running-max softmax.
    "global_running_max": dict(S=1, H=16, frames=200, T_f=1374, dtype="bf16", seed=3, prefix=5, grid=(37, 37),
                               eps=1e-6, ln_gain=2.5,
                               name="config 4 with QK-LayerNorm weight 2.5 (score bound ~72 > 48): the "
                                    "running-max softmax, 274,800 tokens, 16 heads x 64, bf16"),
    "frame_running_max": dict(S=200, H=16, frames=1, T_f=1374, dtype="f16", seed=2, prefix=5, grid=(37, 37),
                              eps=1e-6, ln_gain=1.2,
                              name="config 3 with QK-LayerNorm weight 1.2 (score bound ~16.6 > 14): the "
                                   "running-max softmax, 200 frames x 1374 tokens, 16 heads x 64, fp16"),
    # Same work as "frame" on the layout Block::forward hands over: q, k, v are the
    # (S*T, H*D) projection outputs and the output is the merged (S*T, H*D) tensor
    # (split_heads, QK-norm, RoPE, attention and attn_merge in one call).
    # The block MLP of the aggregator (block.rs:167-176 + residual_ls) at BASELINE
    # config 5's global-layer token count: fc1 + GELU, fc2 + LayerScale residual.
    "mlp": dict(kind="mlp", tokens=137400, d=1024, hidden=4096, dtype="bf16", seed=5,
                name="block MLP at 137,400 tokens (100 frames x 1374), d 1024, hidden 4096, bf16: "
                     "fc1 + bias + erf-GELU, fc2 + bias + LayerScale residual (hs_linear)"),
    # Head-input cache build of one cached trunk layer at BASELINE config 5 (100 frames x
    # 1374 tokens, C = 1024, bf16 -> f32 (N*T, 2048)), plus the register-layer gather and
    # scatter of the 17 prefix tokens per frame (trunk.rs:105-140, cache.rs:25-52).
    "trunk_glue": dict(kind="glue", frames=100, t=1374, c=1024, prefix=17, dtype="bf16", seed=6,
                       name="trunk glue at 100 frames x 1374 tokens, C 1024, bf16: f32 head-input cache "
                            "build (concat + cast) and the register gather/scatter"),
    # the full aggregator forward (DINO 24 layers + 24 frame/global block
    # pairs + the 4 head-input caches) over 100 frames of 518x518 RGB, bf16, random weights.
    "aggregator": dict(kind="aggregator", frames=100, size=518, dtype="bf16", seed=4,
                       name="VGGT-1B aggregator forward, 100 frames 518x518 (patch 14, 37x37, 5 prefix tokens), "
                            "DINO 24 layers + 24 frame/global block pairs, bf16, random-init N(0,0.02), "
                            "LayerScale 1e-5"),
    # The reference server's own trunk layout (headshot-shared src/model.rs:25): five of the
    # 24 inter-frame layers attend over the 5 prefix tokens of every frame only.
    "aggregator_shared": dict(kind="aggregator", layout="headshot_shared", frames=100, size=518, dtype="bf16",
                              seed=4,
                              name="VGGT aggregator forward in headshot-server's trunk layout (19 global + 5 "
                                   "register-only inter-frame layers), 100 frames 518x518, bf16, random-init"),
    # BASELINE config 1's shape: one frame block + one global block over 4 frames x 1374 tokens,
    # dim 1024, random weights N(0,0.02), LayerScale 1e-5, QK-LN eps 1e-6, seed 0 (the reference
    # runs it f32 on lavapipe; here bf16 storage, the tensor-core path).
    "block_pair": dict(kind="block_pair", frames=4, t=1374, dtype="bf16", seed=0,
                       name="config 1's shape in bf16 storage (not config 1's f32): VGGT block pair (frame block + "
                            "global block), 4 frames x 1374 tokens, dim 1024, 16 heads x 64, MLP 4096, "
                            "random-init N(0,0.02), LayerScale 1e-5"),
    # Config 1 as BASELINE words it, f32 storage throughout: f32 LayerNorms and linears (f32
    # arithmetic on the CUDA cores), f32 q/k/v into the attention, whose tensor-core products
    # take bf16-rounded operands (f32 softmax statistics, f32 output).
    "block_pair_f32": dict(kind="block_pair", frames=4, t=1374, dtype="f32", seed=0,
                           name="BASELINE config 1: VGGT block pair (frame block + global block), 4 frames x 1374 "
                                "tokens, dim 1024, 16 heads x 64, MLP 4096, f32 storage (attention operands "
                                "rounded to bf16 for the tensor core), random-init N(0,0.02), LayerScale 1e-5"),
    "frame_block": dict(S=200, H=16, frames=1, T_f=1374, dtype="f16", seed=2, prefix=5, grid=(37, 37), eps=1e-6,
                        layout="block",
                        name="batched frame attention on the projection layout (S*T, H*D) in and merged out, "
                             "200 frames x 1374 tokens, 16 heads x 64, fp16, fused QK-LayerNorm + 2D RoPE"),
}


# DRAM bytes (read + write) per attention launch from one-pass ncu captures
# (dram__bytes_read.sum + dram__bytes_write.sum), each stored with the sha256 of
# the attention kernel's sources at capture time: a figure whose hash no longer
# matches the sources is not reported (traffic null, with the reason).
MEASURED_TRAFFIC = {
    "global": {"bytes": 6957943552 + 576583936, "sources_sha256": "845b00488f5fe5b6f2e0542294df6f33b811aae0deccb2ce83b20efa91ef5598"},
    "global43k": {"bytes": 270670336 + 73345536, "sources_sha256": "845b00488f5fe5b6f2e0542294df6f33b811aae0deccb2ce83b20efa91ef5598"},
    "frame": {"bytes": 1688890368 + 542964992, "sources_sha256": "845b00488f5fe5b6f2e0542294df6f33b811aae0deccb2ce83b20efa91ef5598"},
}
TRAFFIC_SOURCES = ("headshot_b200/csrc/attention_sm100.cu", "headshot_b200/csrc/hs_ptx.cuh")


def attention_sources_sha256() -> str:
    import hashlib

    h = hashlib.sha256()
    for rel in TRAFFIC_SOURCES:
        h.update((ROOT / rel).read_bytes())
    return h.hexdigest()


def measured_traffic(workload: str) -> tuple[int | None, str]:
    """(bytes per launch, source note) for `workload`, or (None, why not)."""
    rec = MEASURED_TRAFFIC.get(workload)
    if rec is None:
        return None, "not captured for this workload"
    if rec["sources_sha256"] != attention_sources_sha256():
        return None, "stale: the attention kernel's sources changed since the ncu capture"
    return int(rec["bytes"]), "ncu dram__bytes_read+write of this launch (1 pass), kernel sources unchanged"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": float(d["bf16_tflops"]), "bf16_sustained": float(d["bf16_tflops_sustained"]),
                "source": "measured"}
    return {"bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------- clocks ---

class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.lines: list[str] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._pump, daemon=True)
        self.thread.start()

    def _pump(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        sm, mx, power, reasons = [], 0.0, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "power_w_median": statistics.median(power) if power else None}


# ---------------------------------------------------------- CPU oracle ---

def cpu_attention_sample(q_h, k_h, v_h, T, seconds_target: float, threads: int, prep: dict):
    """Time the oracle's per-query online softmax (attention.wesl restated in C) on
    sampled query rows of head 0 against all T keys: returns (TFLOP/s, rows, seconds)."""
    import numpy as np

    import oracle

    sin, cos = oracle.rope_tables(*prep["grid"])
    w = np.full(64, prep.get("ln_gain", 1.0), np.float32)
    b = np.zeros(64, np.float32)
    qn = oracle.qk_prep(q_h, w, b, prep["eps"], sin, cos, prep["prefix"], prep["T_f"])
    kn = oracle.qk_prep(k_h, w, b, prep["eps"], sin, cos, prep["prefix"], prep["T_f"])
    rng = np.random.default_rng(0)
    probe = rng.integers(0, T, threads)
    t0 = time.perf_counter()
    oracle.attention_rows(qn, kn, v_h, probe, nthreads=threads)
    per_round = max(time.perf_counter() - t0, 1e-3)
    rounds = max(1, int(seconds_target / per_round))
    rows = rng.integers(0, T, rounds * threads)
    t0 = time.perf_counter()
    oracle.attention_rows(qn, kn, v_h, rows, nthreads=threads)
    dt = time.perf_counter() - t0
    flops = 4.0 * rows.size * T * 64
    return flops / dt / 1e12, int(rows.size), dt


# -------------------------------------------------------------- helpers ---

def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gpu_id_for_smi(local: int) -> str:
    import torch

    try:
        u = str(torch.cuda.get_device_properties(local).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[local]
        return str(local)


# ------------------------------------------------------------ our arm ----

def run_ours(args, wl: dict, rank: int, world: int, local: int) -> dict | None:
    import numpy as np
    import torch

    import headshot_b200.rope as rope_mod
    from headshot_b200.engine import GpuContext, QkNorm, Rope
    from headshot_b200.session import shard_bounds

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[wl["dtype"]]
    S, H, T_f, frames = wl["S"], wl["H"], wl["T_f"], wl["frames"]
    T = T_f * frames
    ctx = GpuContext(local)
    dev = torch.device("cuda", local)

    sin, cos = rope_mod.tables(None, *wl["grid"])
    sin_d, cos_d = torch.from_numpy(sin).to(dev), torch.from_numpy(cos).to(dev)
    w = torch.full((64,), float(wl.get("ln_gain", 1.0)), device=dev)
    b = torch.zeros(64, device=dev)
    norm = QkNorm(w, b, w, b, wl["eps"])

    block = wl.get("layout") == "block"
    if S > 1:  # frame attention: frames sharded across ranks, no communication
        s0, s1 = shard_bounds(S, world, rank)
        shape = ((s1 - s0) * T, H * 64) if block else (s1 - s0, H, T, 64)
        flops_rank = 4.0 * (s1 - s0) * H * T * T * 64
        flops_total = 4.0 * S * H * T * T * 64
        session = None
    else:  # global attention: sequence sharded, ring over ranks
        t0, t1 = shard_bounds(T, world, rank)
        shape = (1, H, t1 - t0, 64)
        flops_rank = 4.0 * H * (t1 - t0) * T * 64
        flops_total = 4.0 * H * T * T * 64
        session = None
        if world > 1:
            from headshot_b200.session import RingSession

            session = RingSession(ctx, rank, world)
            if args.ring_reserved_sms is not None:
                session.set_reserved_sms(args.ring_reserved_sms)

    g = torch.Generator(device=dev).manual_seed(wl["seed"] * 1000 + rank)
    q, k, v = (torch.randn(shape, device=dev, dtype=torch.float32, generator=g).to(tdt) for _ in range(3))
    out = torch.empty_like(q)
    rope = Rope(sin_d, cos_d, wl["prefix"], T_f)

    if block:
        def step():
            ctx.attention_block(q, k, v, s1 - s0, T, H, qk_norm=norm, rope=rope, out=out)
    elif session is None:
        def step():
            ctx.attention_fused(q, k, v, qk_norm=norm, rope=rope, out=out)
    else:
        global_call = session.attention_ulysses if args.global_mode == "ulysses" else session.attention_fused

        def step():
            global_call(q, k, v, out, T_total=T, qk_norm=norm, rope=rope)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    ctx.sync()
    torch.cuda.synchronize(dev)

    # ---- device-resident timed region --------------------------------
    sampler = ClockSampler(gpu_id_for_smi(local))
    sampler.start()
    time.sleep(0.3)
    ctx.prof_reset()
    ctx.prof_enable(True)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    ctx.prof_enable(False)
    clocks = sampler.stop()
    ctx.sync()
    ms_local = e0.elapsed_time(e1)
    attn_ms, attn_n = ctx.prof_read("attention")
    xfer_ms, xfer_n = ctx.prof_read("ring_transfer")
    all_ms, all_n = ctx.prof_read("*")
    all_ms -= xfer_ms  # transfers run on the ring's own stream, beside the kernels
    all_n -= xfer_n
    ms = max_over_ranks(ms_local, world)
    ms_per_step = ms / args.steps
    value = flops_total / (ms_per_step / 1e3) / 1e12

    # ---- end to end through the C ABI: pinned host in, host out -------
    # Every step copies its q, k, v from pinned host memory (hs_memcpy_h2d) and
    # its output back (hs_memcpy_d2h).  Serial: copies and compute in one
    # stream.  Pipelined (the reported value): two device buffer sets; step
    # i+1's inputs upload on one copy stream and step i-1's output downloads
    # on another while step i computes, as a serving loop would run it.  All
    # copies of all timed steps lie inside the timed region.
    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    oh = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    e2e_steps = max(2, min(args.steps, 6))

    def run_step(qq, kk, vv, oo):
        if block:
            ctx.attention_block(qq, kk, vv, s1 - s0, T, H, qk_norm=norm, rope=rope, out=oo)
        elif session is None:
            ctx.attention_fused(qq, kk, vv, qk_norm=norm, rope=rope, out=oo)
        else:
            global_call(qq, kk, vv, oo, T_total=T, qk_norm=norm, rope=rope)

    def e2e_serial():
        ctx.upload(q, qh)
        ctx.upload(k, kh)
        ctx.upload(v, vh)
        run_step(q, k, v, out)
        ctx.download(oh[0], out)

    e2e_serial()
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e2e_steps):
        e2e_serial()
    f1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync()
    serial_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)

    sets = [(q, k, v, out), tuple(torch.empty_like(x) for x in (q, k, v, out))]
    up_stream, down_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def upload_set(i):
        b = i % 2
        with torch.cuda.stream(up_stream):
            if i >= 2:
                up_stream.wait_event(ev_done[b])  # step i-2 has finished reading this set
            for dst, src in zip(sets[b][:3], (qh, kh, vh)):
                ctx.upload(dst, src)
            ev_in[b].record(up_stream)

    def pipelined(n):
        upload_set(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                upload_set(i + 1)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # step i-2's output has left this set's out buffer
            run_step(*sets[b])
            ev_done[b].record(stream)
            with torch.cuda.stream(down_stream):
                down_stream.wait_event(ev_done[b])
                ctx.download(oh[b], sets[b][3])
                ev_out[b].record(down_stream)
        stream.wait_stream(down_stream)
        stream.wait_stream(up_stream)

    pipelined(2)
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    f0.record(stream)
    up_stream.wait_event(f0)
    down_stream.wait_event(f0)
    pipelined(e2e_steps)
    f1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)
    e2e_value = flops_total / (e2e_ms / 1e3) / 1e12
    serial_value = flops_total / (serial_ms / 1e3) / 1e12
    h2d = 3 * q.numel() * q.element_size() * world
    d2h = out.numel() * out.element_size() * world
    del sets

    # ---- roofline of the dominant kernel (attention), live events ----
    peaks = measured_peaks()
    attn_per_launch_ms = attn_ms / max(attn_n, 1)
    if session is None:
        flops_per_launch = flops_rank
    elif args.global_mode == "ulysses":  # one launch over the whole sequence of H / world heads
        flops_per_launch = 4.0 * (H // world) * T * T * 64
    else:  # one ring step: this rank's queries against one block of keys
        flops_per_launch = flops_rank / world
    achieved = flops_per_launch / (attn_per_launch_ms / 1e3) / 1e12
    # DRAM bytes per attention launch from one-pass ncu captures of these exact
    # single-GPU launches, reported only while the kernel sources still hash to
    # the captured ones; ring steps and uncaptured workloads report null.
    traffic, traffic_note = measured_traffic(args.workload) if world == 1 else (None, "not captured for ring steps")
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16"], 4), "traffic": traffic,
                "traffic_source": traffic_note,
                "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                # the launches run back to back for seconds under the 1000 W cap, the regime of
                # the sustained figure: both fractions are given, `frac` is the burst one
                "frac_of_sustained_peak": round(achieved / peaks["bf16_sustained"], 4),
                "kernel": "attn_fwd_sm100", "kernel_ms_per_launch": round(attn_per_launch_ms, 3),
                "launches": attn_n,
                # device time of this rank's attention launches over the timed region's device time
                "kernel_share_of_step": round(attn_ms / max(ms_local, 1e-9), 4),
                "other_launches_ms_per_step": round((all_ms - attn_ms) / args.steps, 3)}
    if session is not None:
        # Ring overlap, from events on both streams of this rank: the block transfers
        # (NCCL send/recv on the ring's stream) and the attention launches.  A transfer's
        # span runs from the point its stream reaches it (the previous step's attention
        # launch has been queued) to its completion, so it includes any wait for SMs.
        # What the step spends outside attention launches is what the transfers, the
        # Q'/K' prep and the launches' own tails did not hide.
        roofline["ring"] = {
            "mode": args.global_mode,
            "reserved_sms": args.ring_reserved_sms if args.ring_reserved_sms is not None else "library default (0)",
            "transfers_per_step": round(xfer_n / args.steps, 2),
            "transfer_span_ms_per_step": round(xfer_ms / args.steps, 3),
            "attention_ms_per_step": round(attn_ms / args.steps, 3),
            "outside_attention_frac": round(1.0 - attn_ms / max(ms_local, 1e-9), 4)}

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and S == 1:
            head = lambda x: x[0, 0].float().cpu().numpy()[None, None]  # noqa: E731
            tf, rows, dt = cpu_attention_sample(head(q), head(k), head(v), T, args.cpu_seconds,
                                                args.cpu_threads or _threads(), dict(wl, T_f=T_f))
            cpu = {"value": round(tf, 6), "unit": "TFLOP/s", "cores": args.cpu_threads or _threads(), "kind": "port",
                   "sample": f"{rows} query rows of head 0 x all {T} keys (rows are independent), "
                             f"fused QK-LN + RoPE on the CPU, {dt:.1f} s"}
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": wl["dtype"],
            "data": f"synthetic N(0,1) q/k/v, seed {wl['seed']}",
            "config": {"workload": wl["name"], "S": S, "H": H, "T": T, "D": 64,
                       "tokens": S * T, "tokens_per_s": round(S * T / (ms_per_step / 1e3), 1),
                       "flops_per_step": flops_total,
                       "frac_of_measured_bf16_peak": round(value / peaks["bf16"], 4),
                       "parallelism": (("head-parallel all-to-all" if args.global_mode == "ulysses" and world > 1
                                        else "ring sequence-parallel") if S == 1 else "frame-sharded") + f" x{world}",
                       "l2": "inputs larger than L2 (each of q/k/v > 126 MB); no flush needed"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3), "steps": e2e_steps,
                    "mode": "pipelined: step i+1's uploads and step i-1's download overlap step i's compute",
                    "serial_value": round(serial_value, 2), "serial_ms_per_step": round(serial_ms, 3)},
            "gpu_launches": int(all_n) * world,
            "clocks": clocks,
        }
    if session is not None:
        session.close()
    ctx.close()
    return result


def run_mlp(args, wl: dict, rank: int, world: int, local: int) -> dict | None:
    """Block MLP through hs_linear: rows sharded across ranks, no communication."""
    import torch

    from headshot_b200.engine import GpuContext
    from headshot_b200.session import shard_bounds

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[wl["dtype"]]
    ctx = GpuContext(local)
    dev = torch.device("cuda", local)
    r0, r1 = shard_bounds(wl["tokens"], world, rank)
    m, d, hid = r1 - r0, wl["d"], wl["hidden"]
    g = torch.Generator(device=dev).manual_seed(wl["seed"] * 1000 + rank)
    x = torch.randn((m, d), device=dev, generator=g).to(tdt)  # LayerNorm'd block input
    res = torch.randn((m, d), device=dev, generator=g).to(tdt)  # residual stream
    w1 = (torch.randn((hid, d), device=dev, generator=g) * 0.02).to(tdt)
    w2 = (torch.randn((d, hid), device=dev, generator=g) * 0.02).to(tdt)
    b1 = torch.zeros(hid, device=dev)
    b2 = torch.zeros(d, device=dev)
    ls = torch.full((d,), 1e-5, device=dev)
    hidden = torch.empty((m, hid), device=dev, dtype=tdt)
    out = torch.empty((m, d), device=dev, dtype=tdt)

    def step(xx=x, rr=res, oo=out):
        ctx.linear(xx, w1, b1, epilogue="gelu", out=hidden)
        ctx.linear(hidden, w2, b2, epilogue="residual_ls", residual=rr, gamma=ls, out=oo)

    flops_rank = 2.0 * m * d * hid * 2
    flops_total = 2.0 * wl["tokens"] * d * hid * 2
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    ctx.sync()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id_for_smi(local))
    sampler.start()
    time.sleep(0.3)
    ctx.prof_reset()
    ctx.prof_enable(True)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    ctx.prof_enable(False)
    clocks = sampler.stop()
    ctx.sync()
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    lin_ms, lin_n = ctx.prof_read("linear")
    value = flops_total / (ms / 1e3) / 1e12

    # the same two layers unfused through cuBLAS and torch element-wise ops, for context
    b1h, b2h, lsh = b1.to(tdt), b2.to(tdt), ls.to(tdt)

    def unfused():
        hh = torch.nn.functional.gelu(torch.nn.functional.linear(x, w1, b1h))
        return res + lsh * torch.nn.functional.linear(hh, w2, b2h)

    for _ in range(3):
        unfused()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        unfused()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    unfused_ms = e0.elapsed_time(e1) / args.steps

    # end to end: the step's input rows and residual up, the output down (pinned host memory)
    xh, rh = x.cpu().pin_memory(), res.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        ctx.upload(x, xh)
        ctx.upload(res, rh)
        step()
        ctx.download(oh, out)

    e2e_step()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps

    peaks = measured_peaks()
    achieved = flops_rank / (lin_ms / max(lin_n, 1) * 2 / 1e3) / 1e12  # two launches per step
    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_mlp_sample(x, w1, w2, res, ls, args.cpu_threads or _threads())
        result = {
            "metric": "block MLP TFLOP/s (fc1+GELU, fc2+LayerScale residual) at 137,400 tokens",
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl["dtype"], "data": f"synthetic N(0,1) rows, weights N(0, 0.02), seed {wl['seed']}",
            "config": {"workload": wl["name"], "tokens": wl["tokens"], "d": d, "hidden": hid,
                       "parallelism": f"row-sharded x{world}", "unfused_cublas_torch_ms": round(unfused_ms, 3),
                       "l2": "inputs larger than L2 (x 281 MB, hidden 1.1 GB); no flush needed"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16"], 4), "traffic": None,
                         "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)", "kernel": "gemm_sm100",
                         "kernel_ms_per_launch": round(lin_ms / max(lin_n, 1), 3), "launches": lin_n},
            "cpu_baseline": cpu,
            "e2e": {"value": round(flops_total / (e2e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 2 * x.numel() * x.element_size() * world,
                    "d2h_bytes_per_step": out.numel() * out.element_size() * world, "ms_per_step": round(e2e_ms, 3)},
            "gpu_launches": int(lin_n) * world,
            "clocks": clocks,
        }
    ctx.close()
    return result


def run_glue(args, wl: dict, rank: int, world: int, local: int) -> dict | None:
    """Cache build + register gather/scatter; frames sharded across ranks, no communication."""
    import torch

    from headshot_b200.engine import GpuContext
    from headshot_b200.session import shard_bounds

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[wl["dtype"]]
    ctx = GpuContext(local)
    dev = torch.device("cuda", local)
    f0, f1 = shard_bounds(wl["frames"], world, rank)
    n, t, c, pre = f1 - f0, wl["t"], wl["c"], wl["prefix"]
    g = torch.Generator(device=dev).manual_seed(wl["seed"] * 1000 + rank)
    frame_out = torch.randn((n * t, c), device=dev, generator=g).to(tdt)
    global_out = torch.randn((n * t, c), device=dev, generator=g).to(tdt)
    cache = torch.empty((n * t, 2 * c), device=dev, dtype=torch.float32)
    reg = torch.empty((n * pre, c), device=dev, dtype=tdt)

    def step():
        ctx.copy_row_blocks(frame_out, reg, n, t, pre, pre)
        ctx.copy_row_blocks(reg, frame_out, n, pre, t, pre)
        ctx.cache_build(frame_out, global_out, out=cache)

    esz = frame_out.element_size()
    cache_bytes = n * t * 2 * c * (esz + 4)
    bytes_rank = cache_bytes + 4 * n * pre * c * esz
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    ctx.sync()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id_for_smi(local))
    sampler.start()
    time.sleep(0.3)
    ctx.prof_reset()
    ctx.prof_enable(True)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    ctx.prof_enable(False)
    clocks = sampler.stop()
    ctx.sync()
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    cb_ms, cb_n = ctx.prof_read("cache_build")
    value = bytes_rank * world / (ms / 1e3) / 1e9
    peaks_hbm = None
    mp = ROOT / "MEASURED_PEAKS.json"
    if mp.exists():
        peaks_hbm = float(json.loads(mp.read_text()).get("hbm_gbs", 0) or 0) or None
    peak = peaks_hbm or 6650.0
    achieved = cache_bytes / (cb_ms / max(cb_n, 1) / 1e3) / 1e9
    fh, gh = frame_out.cpu().pin_memory(), global_out.cpu().pin_memory()
    ch = torch.empty(cache.shape, dtype=cache.dtype).pin_memory()

    def e2e_step():
        ctx.upload(frame_out, fh)
        ctx.upload(global_out, gh)
        step()
        ctx.download(ch, cache)

    e2e_step()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    result = None
    if rank == 0:
        result = {
            "metric": "trunk glue GB/s (f32 head-input cache build + register gather/scatter) at 100 frames",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": wl["dtype"], "data": f"synthetic N(0,1), seed {wl['seed']}",
            "config": {"workload": wl["name"], "frames": wl["frames"], "t": t, "c": c,
                       "parallelism": f"frame-sharded x{world}",
                       "l2": "each buffer larger than L2 (cache 1.1 GB); no flush needed"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": "measured copy bandwidth (MEASURED_PEAKS.json)" if peaks_hbm else "fallback",
                         "kernel": "cache_build_kernel", "kernel_ms_per_launch": round(cb_ms / max(cb_n, 1), 3),
                         "launches": cb_n},
            "cpu_baseline": None,
            "e2e": {"value": round(bytes_rank * world / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": 2 * frame_out.numel() * esz * world,
                    "d2h_bytes_per_step": cache.numel() * 4 * world, "ms_per_step": round(e2e_ms, 3)},
            "gpu_launches": 3 * args.steps * world,
            "clocks": clocks,
        }
    ctx.close()
    return result


def run_aggregator(args, wl: dict, rank: int, world: int, local: int) -> dict | None:
    """Config 5: Aggregator.forward, frames sharded across ranks, global blocks on the ring."""
    import torch

    from headshot_b200.aggregator import Aggregator, AggregatorConfig
    from headshot_b200.engine import GpuContext
    from headshot_b200.session import RingSession, shard_bounds

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[wl["dtype"]]
    cfg = _aggregator_config(wl)
    ctx = GpuContext(local)
    dev = torch.device("cuda", local)
    n_total, size = wl["frames"], wl["size"]
    f0, f1 = shard_bounds(n_total, world, rank)
    agg = Aggregator(cfg, tdt, seed=wl["seed"], device=dev)
    g = torch.Generator(device=dev).manual_seed(wl["seed"])
    images_all = torch.rand((n_total, 3, size, size), device=dev, generator=g)
    images = images_all[f0:f1].contiguous()
    del images_all
    ring = RingSession(ctx, rank, world) if world > 1 else None

    def step(imgs=images):
        return agg.forward(ctx, imgs, ring=ring, n_total=n_total, frame0=f0)

    fl = agg.flops(n_total, size, size)
    p = (size // cfg.patch) ** 2
    reg_att = len(cfg.register_layers) * 4 * cfg.heads * (n_total * cfg.trunk_prefix) ** 2 * (cfg.dim // cfg.heads)
    att_rank = (fl["attention"] - reg_att) * (f1 - f0) / n_total + reg_att  # register blocks run on every rank
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        caches = step()
    del caches
    ctx.sync()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id_for_smi(local))
    sampler.start()
    time.sleep(0.3)
    ctx.prof_reset()
    ctx.prof_enable(True)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        caches = step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    ctx.prof_enable(False)
    clocks = sampler.stop()
    ctx.sync()
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    att_ms, att_n = ctx.prof_read("attention")
    lin_ms, lin_n = ctx.prof_read("linear")
    all_ms, all_n = ctx.prof_read("*")
    # device time per kind of launch over this rank's timed region
    local_ms = e0.elapsed_time(e1)
    shares = {}
    for kind in ("attention", "linear", "qk_prep", "layernorm", "cache_build", "copy_rows", "im2col_patch"):
        k_ms, k_n = ctx.prof_read(kind)
        shares[kind] = {"share_of_step": round(k_ms / local_ms, 4), "launches_per_step": round(k_n / args.steps, 1)}
    shares["unbracketed"] = {"share_of_step": round(max(0.0, 1.0 - all_ms / local_ms), 4)}
    value = n_total / (ms / 1e3)

    # end to end: the rank's images up from pinned host memory, its four caches down; each
    # cache's download starts on a copy stream as soon as the cache is built, overlapping the
    # layers after it
    ih = images.cpu().pin_memory()
    ch = [torch.empty(c.shape, dtype=c.dtype).pin_memory() for c in caches]
    copy_stream = torch.cuda.Stream(dev)

    def e2e_step():
        ctx.upload(images, ih)
        built = []

        def tap(name, t):
            if name.startswith("cache."):
                ev = torch.cuda.Event()
                ev.record(stream)
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_event(ev)
                    ctx.download(ch[len(built)], t)
                built.append(t)

        out = agg.forward(ctx, images, tap=tap, ring=ring, n_total=n_total, frame0=f0)
        stream.wait_stream(copy_stream)
        return out

    del caches
    e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    if ring is not None:
        ring.sync()
        ring.close()

    peaks = measured_peaks()
    att_achieved = att_rank * args.steps / (att_ms / 1e3) / 1e12
    lin_achieved = fl["gemm"] * (f1 - f0) / n_total * args.steps / (lin_ms / 1e3) / 1e12
    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_aggregator_estimate(cfg, n_total, size, args.cpu_threads or _threads(), wl["dtype"])
        result = {
            "metric": "aggregator frames/s (BASELINE config 5: VGGT-1B aggregator forward at 100 frames)",
            "value": round(value, 3), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": wl["dtype"],
            "data": f"synthetic images U[0,1], random-init weights N(0,0.02), seed {wl['seed']}",
            "config": {"workload": wl["name"], "frames": n_total, "image": size, "patch": cfg.patch,
                       "tokens_per_frame": p + cfg.trunk_prefix, "dino_layers": cfg.dino_layers,
                       "block_pairs": cfg.trunk_pairs, "register_layers": list(cfg.register_layers),
                       "cached_layers": list(cfg.cached_layers),
                       "parallelism": f"frame-sharded x{world}" + (", global blocks ring" if world > 1 else ""),
                       "tflops_per_step": round(fl["total"] / 1e12, 1),
                       "tflop_s_whole_step": round(fl["total"] / (ms / 1e3) / 1e12, 1),
                       "l2": "activations larger than L2 (281 MB per token tensor); no flush needed"},
            "roofline": {"bound": "tensor", "achieved": round(att_achieved, 1), "peak": peaks["bf16_sustained"],
                         "unit": "TFLOP/s", "frac": round(att_achieved / peaks["bf16_sustained"], 4),
                         "traffic": None,
                         "peak_source": f"{peaks['source']} bf16 sustained (MEASURED_PEAKS.json): kernels inside a "
                                        f"seconds-long step",
                         "kernel": "attn_fwd_sm100 (all attention launches of the step)",
                         "attention_share_of_step": round(att_ms / local_ms, 4),
                         "linear_tflops": round(lin_achieved, 1),
                         "linear_share_of_step": round(lin_ms / local_ms, 4),
                         "shares_by_kind": shares},
            "cpu_baseline": cpu,
            "e2e": {"value": round(n_total / (e2e_ms / 1e3), 3), "unit": "frames/s",
                    "h2d_bytes_per_step": images.numel() * 4 * world,
                    "d2h_bytes_per_step": sum(c.numel() * 4 for c in ch) * world, "ms_per_step": round(e2e_ms, 2)},
            "gpu_launches": int(all_n) * world,
            "clocks": clocks,
        }
    ctx.close()
    return result


def _aggregator_config(wl: dict):
    from headshot_b200.aggregator import AggregatorConfig

    return AggregatorConfig.headshot_shared() if wl.get("layout") == "headshot_shared" else AggregatorConfig()


def _block_pair_setup(wl: dict, dev, tdt):
    import torch

    from headshot_b200 import rope as rope_mod
    from headshot_b200.aggregator import AggregatorConfig, Block, BlockWeights
    from headshot_b200.engine import Rope

    cfg = AggregatorConfig()
    g = torch.Generator(device=dev).manual_seed(wl["seed"])
    frame_blk = Block(BlockWeights.random(cfg, True, tdt, g, dev), cfg.heads, cfg.norm_eps)
    global_blk = Block(BlockWeights.random(cfg, True, tdt, g, dev), cfg.heads, cfg.norm_eps)
    n, t = wl["frames"], wl["t"]
    x = torch.randn((n * t, cfg.dim), generator=g, device=dev).to(tdt)
    sin, cos = rope_mod.tables(None, 37, 37)
    rope = Rope(torch.from_numpy(sin).to(dev), torch.from_numpy(cos).to(dev), t - 37 * 37, t)
    return cfg, frame_blk, global_blk, x, rope


def _block_pair_flops(cfg, n: int, t: int) -> float:
    d, hid = cfg.dim, cfg.mlp_hidden
    gemm = 2.0 * n * t * (4 * d * d + 2 * d * hid)
    return 2 * gemm + 4.0 * n * cfg.heads * t * t * 64 + 4.0 * cfg.heads * (n * t) ** 2 * 64


def run_block_pair(args, wl: dict, rank: int, world: int, local: int) -> dict | None:
    """Config 1's block pair through Block.forward (hs_layernorm, hs_linear, hs_attention_block_fused);
    too small to shard, so at N > 1 every rank runs a replica (weak scaling)."""
    import torch

    from headshot_b200.engine import GpuContext

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[wl["dtype"]]
    ctx = GpuContext(local)
    dev = torch.device("cuda", local)
    cfg, fb, gb, x, rope = _block_pair_setup(wl, dev, tdt)
    n, t = wl["frames"], wl["t"]

    def step(xx=x):
        return gb.forward(ctx, fb.forward(ctx, xx, n, t, rope), 1, n * t)

    fl = _block_pair_flops(cfg, n, t)
    stream = torch.cuda.current_stream(dev)
    # 5.6k tokens of activations fit in L2: a 256 MB write between steps evicts them
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step()
    # The library's launches of one step, counted on an untimed step: the events that
    # bracket each launch would add ~0.1 ms to a 0.8 ms step of 14 launches.
    ctx.prof_reset()
    ctx.prof_enable(True)
    step()
    ctx.prof_enable(False)
    _, launches_per_step = ctx.prof_read("*")
    ctx.sync()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_id_for_smi(local))
    sampler.start()
    time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    launches = launches_per_step * args.steps
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(starts, ends)), world) / args.steps
    value = fl * world / (ms / 1e3) / 1e12

    xh = x.cpu().pin_memory()
    out = step()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        ctx.upload(x, xh)
        o = step()
        ctx.download(oh, o)

    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        starts[i].record(stream)
        e2e_step()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(starts, ends)), world) / args.steps
    peaks = measured_peaks()
    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            fl_s, dt = cpu_block_pair_sample(wl, fb, gb, x, args.cpu_threads or _threads())
            cpu = {"value": round(fl_s / dt / 1e12, 6), "unit": "TFLOP/s", "cores": args.cpu_threads or _threads(),
                   "kind": "port", "sample": f"one frame of the frame block and the global block's rows of that frame "
                                             f"(all 5496 keys), f32 oracle, {dt:.1f} s"}
        result = {
            "metric": ("block pair TFLOP/s (BASELINE config 1: frame block + global block, 4 frames, f32)"
                       if wl["dtype"] == "f32" else
                       "block pair TFLOP/s (BASELINE config 1's shape in bf16: frame block + global block, 4 frames)"),
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": wl["dtype"], "data": f"synthetic x N(0,1), random-init weights N(0,0.02), seed {wl['seed']}",
            "config": {"workload": wl["name"], "tokens": n * t, "tokens_per_s": round(n * t * world / (ms / 1e3)),
                       "flops_per_step": fl, "parallelism": f"replicas x{world}",
                       "l2": "256 MB buffer written between timed steps (activations fit in L2)"},
            "roofline": {"bound": "tensor", "achieved": round(fl / (ms / 1e3) / 1e12, 1), "peak": peaks["bf16"],
                         "unit": "TFLOP/s", "frac": round(fl / (ms / 1e3) / 1e12 / peaks["bf16"], 4),
                         "traffic": None, "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                         "kernel": f"whole step ({launches // args.steps} launches: attention, linears, "
                                   f"LayerNorms, QK prep)"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(fl * world / (e2e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x.numel() * x.element_size() * world,
                    "d2h_bytes_per_step": out.numel() * out.element_size() * world, "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": int(launches) * world,
            "clocks": clocks,
        }
    ctx.close()
    return result


def _np_block(b) -> dict:
    a = lambda t: t.float().cpu().numpy()  # noqa: E731
    w = b.w
    qn = None if w.qk_norm is None else (a(w.qk_norm.q_w), a(w.qk_norm.q_b), a(w.qk_norm.k_w), a(w.qk_norm.k_b),
                                         w.qk_norm.eps)
    return {"norm1_w": a(w.norm1_w), "norm1_b": a(w.norm1_b), "qkv_w": [a(y) for y in w.qkv_w],
            "qkv_b": [a(y) for y in w.qkv_b], "proj_w": a(w.proj_w), "proj_b": a(w.proj_b), "ls1": a(w.ls1),
            "norm2_w": a(w.norm2_w), "norm2_b": a(w.norm2_b), "fc1_w": a(w.fc1_w), "fc1_b": a(w.fc1_b),
            "fc2_w": a(w.fc2_w), "fc2_b": a(w.fc2_b), "ls2": a(w.ls2), "qk_norm": qn}


def cpu_block_pair_sample(wl: dict, fb, gb, x, threads: int, np_blocks: tuple | None = None) -> tuple[float, float]:
    """The reference path (oracle restatements, f32, reference op order) on a bounded,
    exactly counted quarter of config 1: frame 0 through the frame block, then the global
    block for frame 0's rows (LayerNorm, q/proj/MLP linears on those rows; k/v linears on
    all 5496 rows; attention of those rows over every key).  Returns (FLOPs, seconds)."""
    import numpy as np

    import oracle
    from oracle import model as om

    n, t = wl["frames"], wl["t"]
    d, heads = 1024, 16
    fbn, gbn = np_blocks or (_np_block(fb), _np_block(gb))
    xs = x.float().cpu().numpy()
    sin, cos = oracle.rope_tables(37, 37)
    prefix = t - 37 * 37

    def r(a):
        return oracle.round_to(wl["dtype"], a)

    t0 = time.perf_counter()
    frame0 = om.block_forward(xs[:t], fbn, 1, t, heads, 1e-5, wl["dtype"], (sin, cos, prefix))
    # the other frames' frame-block outputs are inputs to the global block: taken as the
    # (untimed) rounded input rows, the sample's cost is frame 0's
    xg = np.concatenate([frame0, r(xs[t:])])
    normed = r(oracle.layernorm(xg, gbn["norm1_w"], gbn["norm1_b"], 1e-5))
    q = r(oracle.linear(normed[:t], gbn["qkv_w"][0], gbn["qkv_b"][0], nthreads=threads))
    k = r(oracle.linear(normed, gbn["qkv_w"][1], gbn["qkv_b"][1], nthreads=threads))
    v = r(oracle.linear(normed, gbn["qkv_w"][2], gbn["qkv_b"][2], nthreads=threads))
    qw, qb, kw, kb, eps = gbn["qk_norm"]
    qh = r(oracle.layernorm(oracle.split_heads(q, 1, t, heads, 64), qw, qb, eps))
    kh = r(oracle.layernorm(oracle.split_heads(k, 1, n * t, heads, 64), kw, kb, eps))
    vh = oracle.split_heads(v, 1, n * t, heads, 64)
    # rows of frame 0 (head-major, per head over every key)
    qpad = np.zeros((1, heads, n * t, 64), np.float32)
    qpad[:, :, :t] = qh
    rows = np.concatenate([np.arange(t) + h * n * t for h in range(heads)])
    att = oracle.attention_rows(qpad, kh, vh, rows, nthreads=threads).reshape(heads, t, 64)
    merged = r(oracle.attn_merge(att[None]))
    x1 = r(oracle.residual_ls(xg[:t], r(oracle.linear(merged, gbn["proj_w"], gbn["proj_b"], nthreads=threads)),
                              gbn["ls1"]))
    h2 = r(oracle.layernorm(x1, gbn["norm2_w"], gbn["norm2_b"], 1e-5))
    hid = r(oracle.gelu(r(oracle.linear(h2, gbn["fc1_w"], gbn["fc1_b"], nthreads=threads))))
    oracle.residual_ls(x1, r(oracle.linear(hid, gbn["fc2_w"], gbn["fc2_b"], nthreads=threads)), gbn["ls2"])
    dt = time.perf_counter() - t0
    gemm_rows = 2.0 * t * (4 * d * d + 2 * d * 4096)  # frame block on frame 0
    gemm_glob = 2.0 * t * d * d * 2 + 2.0 * n * t * d * d * 2 + 2.0 * t * 2 * d * 4096  # q, proj; k, v; fc1, fc2
    flops = gemm_rows + 4.0 * heads * t * t * 64 + gemm_glob + 4.0 * heads * t * n * t * 64
    return flops, dt


def cpu_aggregator_estimate(cfg, frames: int, size: int, threads: int, dtype: str, seconds: float = 12.0) -> dict:
    """CPU frames/s of the reference path for config 5, extrapolated from timed oracle samples:
    a fc1-shaped linear (linear.wesl) for the GEMM rate and query rows of one head of global
    attention (attention.wesl) for the attention rate, each sized to about seconds/2."""
    import numpy as np

    import oracle
    from headshot_b200.aggregator import Aggregator

    rng = np.random.default_rng(5)
    d, hid = cfg.dim, cfg.mlp_hidden
    w = oracle.round_to(dtype, (0.02 * rng.standard_normal((hid, d))).astype(np.float32))

    def gemm(rows):
        x = oracle.round_to(dtype, rng.standard_normal((rows, d)).astype(np.float32))
        t0 = time.perf_counter()
        oracle.linear(x, w, None, nthreads=threads)
        return time.perf_counter() - t0

    probe = max(gemm(8 * threads), 1e-3)
    rows = int(max(8 * threads, 8 * threads * seconds / 2 / probe))
    g_dt = gemm(rows)
    gemm_rate = 2.0 * rows * d * hid / g_dt
    t = ((size // cfg.patch) ** 2 + cfg.trunk_prefix) * frames
    q, k, v = (oracle.round_to(dtype, rng.standard_normal((1, 1, t, 64)).astype(np.float32)) for _ in range(3))

    def att(n):
        t0 = time.perf_counter()
        oracle.attention_rows(q, k, v, rng.integers(0, t, n), nthreads=threads)
        return time.perf_counter() - t0

    probe = max(att(threads), 1e-3)
    n_rows = int(max(threads, threads * seconds / 2 / probe))
    a_dt = att(n_rows)
    att_rate = 4.0 * n_rows * t * 64 / a_dt
    fl = Aggregator.flops(type("A", (), {"cfg": cfg})(), frames, size, size)
    cpu_s = fl["gemm"] / gemm_rate + fl["attention"] / att_rate
    return {"value": round(frames / cpu_s, 8), "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"extrapolated: {rows} rows of a 1024->4096 linear ({g_dt:.1f} s, {gemm_rate / 1e9:.1f} GFLOP/s) "
                      f"and {n_rows} query rows of one head over {t} keys ({a_dt:.1f} s, "
                      f"{att_rate / 1e9:.1f} GFLOP/s), scaled by the forward's GEMM and attention FLOPs; "
                      f"LayerNorm, GELU, RoPE and copies left out (favours the CPU)",
            "cpu_seconds_per_forward": round(cpu_s, 1)}


def cpu_mlp_sample(x, w1, w2, res, ls, threads: int) -> dict:
    """The reference path on the CPU (oracle linear.wesl + gelu.wesl + residual_ls.wesl) on a
    bounded sample of rows (rows are independent)."""
    import numpy as np

    import oracle

    w1h, w2h, lsh = w1.float().cpu().numpy(), w2.float().cpu().numpy(), ls.float().cpu().numpy()

    def run(rows):
        xs = x[:rows].float().cpu().numpy()
        rs = res[:rows].float().cpu().numpy()
        t0 = time.perf_counter()
        hh = oracle.gelu(oracle.linear(xs, w1h, None, nthreads=threads))
        oracle.residual_ls(rs, oracle.linear(hh, w2h, None, nthreads=threads), lsh)
        return time.perf_counter() - t0

    probe = max(run(4 * threads), 1e-3)  # size the sample at about 10 s of CPU work
    rows = int(min(x.shape[0], max(4 * threads, 4 * threads * 10.0 / probe)))
    dt = run(rows)
    fl = 2.0 * rows * w1h.shape[1] * w1h.shape[0] * 2
    return {"value": round(fl / dt / 1e12, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} token rows through fc1+GELU and fc2+residual, f32, {dt:.2f} s"}


def _threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ------------------------------------------------------ reference arm ----

def run_reference(args, wl: dict) -> dict:
    """The reference path's CPU implementation (oracle port of attention.wesl +
    layernorm.wesl + rope_apply.wesl) on all host cores, bounded samples."""
    import numpy as np

    import oracle

    S, H, T_f, frames = wl["S"], wl["H"], wl["T_f"], wl["frames"]
    T = T_f * frames
    threads = args.cpu_threads or _threads()
    rng = np.random.default_rng(wl["seed"])
    q, k, v = (oracle.round_to(wl["dtype"], rng.standard_normal((1, 1, T, 64), np.float32)) for _ in range(3))
    sin, cos = oracle.rope_tables(*wl["grid"])
    w = np.full(64, wl.get("ln_gain", 1.0), np.float32)
    b = np.zeros(64, np.float32)
    # probe to size a step at ~ args.ref_step_seconds of CPU time
    qn = oracle.qk_prep(q, w, b, wl["eps"], sin, cos, wl["prefix"], T_f)
    kn = oracle.qk_prep(k, w, b, wl["eps"], sin, cos, wl["prefix"], T_f)
    t0 = time.perf_counter()
    oracle.attention_rows(qn, kn, v, rng.integers(0, T, threads), nthreads=threads)
    per = max(time.perf_counter() - t0, 1e-3)
    rows_per_step = threads * max(1, int(args.ref_step_seconds / per))

    def step():
        rows = rng.integers(0, T, rows_per_step)
        qs = oracle.qk_prep(q, w, b, wl["eps"], sin, cos, wl["prefix"], T_f)
        ks = oracle.qk_prep(k, w, b, wl["eps"], sin, cos, wl["prefix"], T_f)
        oracle.attention_rows(qs, ks, v, rows, nthreads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    flops = 4.0 * rows_per_step * T * 64 * args.steps
    value = flops / dt / 1e12
    sample = (f"{rows_per_step} query rows x all {T} keys per step of one head (rows are independent), "
              f"QK-LN + RoPE of that head's q/k each step; f32 per-query online softmax")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic N(0,1), seed {wl['seed']}, rounded to {wl['dtype']}",
            "config": {"workload": wl["name"], "S": S, "H": H, "T": T, "D": 64},
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_mlp(args, wl: dict) -> dict:
    """The reference's CPU path for the block MLP (oracle restatements), bounded row samples."""
    import numpy as np

    import oracle

    threads = args.cpu_threads or _threads()
    rng = np.random.default_rng(wl["seed"])
    d, hid = wl["d"], wl["hidden"]
    w1 = oracle.round_to(wl["dtype"], (0.02 * rng.standard_normal((hid, d))).astype(np.float32))
    w2 = oracle.round_to(wl["dtype"], (0.02 * rng.standard_normal((d, hid))).astype(np.float32))
    ls = np.full(d, 1e-5, np.float32)
    rows = 32 * threads
    x = oracle.round_to(wl["dtype"], rng.standard_normal((rows, d)).astype(np.float32))
    r = oracle.round_to(wl["dtype"], rng.standard_normal((rows, d)).astype(np.float32))

    def step():
        hh = oracle.gelu(oracle.linear(x, w1, None, nthreads=threads))
        oracle.residual_ls(r, oracle.linear(hh, w2, None, nthreads=threads), ls)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = 2.0 * rows * d * hid * 2 * args.steps / dt / 1e12
    return {"impl": "reference", "metric": "block MLP TFLOP/s (fc1+GELU, fc2+LayerScale residual) at 137,400 tokens",
            "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": f"synthetic, seed {wl['seed']}, rounded to {wl['dtype']}",
            "config": {"workload": wl["name"], "tokens": wl["tokens"], "d": d, "hidden": hid},
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{rows} token rows per step (rows are independent), f32 linear.wesl order"},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_aggregator(args, wl: dict) -> dict:
    """Config 5 on the CPU: the oracle's linear and attention rates, extrapolated to one
    forward (cpu_aggregator_estimate); each step re-measures the two samples."""
    cfg = _aggregator_config(wl)
    threads = args.cpu_threads or _threads()
    for _ in range(args.warmup):
        cpu_aggregator_estimate(cfg, wl["frames"], wl["size"], threads, wl["dtype"], seconds=2.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        est = cpu_aggregator_estimate(cfg, wl["frames"], wl["size"], threads, wl["dtype"],
                                      seconds=args.ref_step_seconds)
        vals.append(est["value"])
    dt = time.perf_counter() - t0
    value = float(sum(vals) / len(vals))
    return {"impl": "reference", "metric": "aggregator frames/s (BASELINE config 5: VGGT-1B aggregator forward at "
            "100 frames)", "value": round(value, 8), "unit": "frames/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic, rounded to {wl['dtype']}", "config": {"workload": wl["name"]},
            "cpu_baseline": {"value": round(value, 8), "unit": "frames/s", "cores": threads, "kind": "port",
                             "sample": est["sample"]},
            "e2e": {"value": round(value, 8), "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_block_pair(args, wl: dict) -> dict:
    """Config 1 on the CPU: the oracle composition of Block::forward on the bounded quarter
    sample of cpu_block_pair_sample, each step one sample."""
    import torch

    from headshot_b200.aggregator import AggregatorConfig, Block, BlockWeights

    threads = args.cpu_threads or _threads()
    cfg = AggregatorConfig()
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[wl["dtype"]]
    g = torch.Generator().manual_seed(wl["seed"])  # CPU generator: the same shapes and distribution
    fb = Block(BlockWeights.random(cfg, True, tdt, g, torch.device("cpu")), cfg.heads, cfg.norm_eps)
    gb = Block(BlockWeights.random(cfg, True, tdt, g, torch.device("cpu")), cfg.heads, cfg.norm_eps)
    x = torch.randn((wl["frames"] * wl["t"], cfg.dim), generator=g).to(tdt)
    blocks = (_np_block(fb), _np_block(gb))
    for _ in range(min(args.warmup, 1)):
        cpu_block_pair_sample(wl, fb, gb, x, threads, blocks)
    fl = dt = 0.0
    for _ in range(args.steps):
        f, d = cpu_block_pair_sample(wl, fb, gb, x, threads, blocks)
        fl += f
        dt += d
    value = fl / dt / 1e12
    metric = ("block pair TFLOP/s (BASELINE config 1: frame block + global block, 4 frames, f32)"
              if wl["dtype"] == "f32" else
              "block pair TFLOP/s (BASELINE config 1's shape in bf16: frame block + global block, 4 frames)")
    return {"impl": "reference", "metric": metric, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": f"synthetic, rounded to {wl['dtype']}",
            "config": {"workload": wl["name"]},
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": "per step one quarter of the block pair (frame 0's rows; every key)"},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_glue(args, wl: dict) -> dict:
    """The trunk glue on the CPU (the oracle's numpy restatement of copy_rows,
    concat_channels and cast_to_f32) over a bounded sample of frames."""
    import numpy as np

    import oracle

    t, c, pre = wl["t"], wl["c"], wl["prefix"]
    frames = 10
    rng = np.random.default_rng(wl["seed"])
    a = oracle.round_to(wl["dtype"], rng.standard_normal((frames * t, c)).astype(np.float32))
    b = oracle.round_to(wl["dtype"], rng.standard_normal((frames * t, c)).astype(np.float32))
    a, b = a.astype(np.float16), b.astype(np.float16)  # 2-byte storage on the host (numpy has no bf16)
    reg = np.empty((frames * pre, c), a.dtype)

    def step():
        oracle.copy_row_blocks(a, reg, frames, t, pre, pre)
        oracle.copy_row_blocks(reg, a, frames, pre, t, pre)
        oracle.cache_build(a, b)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    nbytes = frames * t * 2 * c * (2 + 4) + 4 * frames * pre * c * 2
    value = nbytes * args.steps / dt / 1e9
    return {"impl": "reference", "metric": "trunk glue GB/s (f32 head-input cache build + register gather/scatter) "
            "at 100 frames", "value": round(value, 3), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": wl["dtype"], "data": "synthetic",
            "config": {"workload": wl["name"]},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"{frames} frames of the 100 (rows are independent), numpy, one thread"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def _json_out():
    """The one JSON line goes to the original stdout; everything else written to
    file descriptor 1 during the run (NCCL prints its version banner there) is
    sent to stderr, so stdout carries exactly one line."""
    saved = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    return os.fdopen(saved, "w")


def main():
    out = _json_out()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="global")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--ref-step-seconds", type=float, default=4.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--global-mode", choices=["ring", "ulysses"], default="ring",
                    help="multi-GPU global attention: the K/V ring, or head parallelism by all-to-all")
    ap.add_argument("--ring-reserved-sms", type=int, default=None,
                    help="SMs the ring's attention launches leave to the block transfers (default: the library's)")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    wl = WORKLOADS[args.workload]

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        if wl.get("kind") == "glue":
            ref = run_reference_glue(args, wl)
        elif wl.get("kind") == "aggregator":
            ref = run_reference_aggregator(args, wl)
        elif wl.get("kind") == "block_pair":
            ref = run_reference_block_pair(args, wl)
        else:
            ref = run_reference_mlp(args, wl) if wl.get("kind") == "mlp" else run_reference(args, wl)
        print(json.dumps(ref), file=out, flush=True)
        return 0

    rank, world, local = dist_setup()
    if world != args.gpus:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE {world}; using {world}")
    try:
        kind = wl.get("kind")
        runner = {"mlp": run_mlp, "glue": run_glue, "aggregator": run_aggregator,
                  "block_pair": run_block_pair}.get(kind, run_ours)
        res = runner(args, wl, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), file=out, flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
