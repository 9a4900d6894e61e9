"""Multi-process session-layer tests on CPU (gloo, world size 2 and 3)."""
from __future__ import annotations

import socket
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(mode: str, world: int, timeout: int = 180) -> list[int]:
    from headshot_b200.build import OUT, build

    if not OUT.exists():
        build()
    port = _port()
    procs = [subprocess.Popen([sys.executable, str(HERE / "_session_worker.py"), mode, str(r), str(world), str(port)])
             for r in range(world)]
    return [p.wait(timeout=timeout) for p in procs]


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_and_state_carry_gloo(world):
    """hs_ring_plan/hs_ring_shard driven over gloo with the kernel's state-carry
    math reproduces full attention on every rank."""
    assert _run("ring", world) == [0] * world


def test_preflight_detects_a_departed_rank():
    """A rank that leaves between steps is noticed on the host before ring traffic."""
    rcs = _run("preflight", 2, timeout=120)
    assert rcs[0] == 0


@pytest.mark.parametrize("world", [2, 3])
def test_dropped_ring_block_fails_every_waiting_rank(world):
    """A ring block that is never sent (its owner leaves) ends the other ranks'
    exchanges with an error within the group timeout; none waits forever."""
    rcs = _run("drop", world, timeout=120)
    assert rcs == [0] * world
