"""bench.py's host-side reporting logic, without a GPU.

- DRAM traffic measured by ncu is reported only while the attention kernel's sources
  still hash to the ones the capture was taken on; otherwise null with the reason.
- The aggregator workloads select BASELINE config 5's layout (24 global layers) and the
  reference server's layout (19 global + 5 register-only layers).
"""
from __future__ import annotations

import bench


def test_traffic_reported_only_for_the_captured_sources(monkeypatch):
    current = bench.attention_sources_sha256()
    monkeypatch.setitem(bench.MEASURED_TRAFFIC, "global", {"bytes": 123.0, "sources_sha256": current})
    traffic, note = bench.measured_traffic("global")
    assert traffic == 123 and "unchanged" in note
    monkeypatch.setitem(bench.MEASURED_TRAFFIC, "global", {"bytes": 123.0, "sources_sha256": "0" * 64})
    traffic, note = bench.measured_traffic("global")
    assert traffic is None and note.startswith("stale")
    assert bench.measured_traffic("block_pair") == (None, "not captured for this workload")


def test_aggregator_layouts():
    cfg = bench._aggregator_config(bench.WORKLOADS["aggregator"])
    assert cfg.register_layers == () and cfg.trunk_pairs == 24
    shared = bench._aggregator_config(bench.WORKLOADS["aggregator_shared"])
    assert shared.register_layers == (2, 6, 9, 14, 20)


def test_running_max_workloads_lift_the_bound_past_the_fixed_offset_limit():
    # |q'|, |k'| <= 8 * gain for unit-direction LayerNorm rows; bound = |q'| |k'| / 8 * log2(e).
    for name, limit in (("global_running_max", 48.0), ("frame_running_max", 14.0)):
        g = bench.WORKLOADS[name]["ln_gain"]
        assert (8 * g) ** 2 / 8 * 1.4426950408889634 > limit
    for name, limit in (("global", 48.0), ("frame", 14.0)):
        assert bench.WORKLOADS[name].get("ln_gain", 1.0) ** 2 * 64 / 8 * 1.4426950408889634 < limit
