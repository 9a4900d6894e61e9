"""The C ABI without a GPU: the library loads, exports every symbol
include/headshot_cuda.h declares, its host helpers agree with the oracle,
and argument errors come back as status codes (never an abort)."""
from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest

import oracle
from headshot_b200 import _lib, session
from headshot_b200.build import OUT as LIB_PATH
from headshot_b200.build import build


@pytest.fixture(scope="module")
def L():
    if not LIB_PATH.exists():
        build()
    return _lib.lib()


def test_library_exports_every_declared_symbol(L):
    declared = _lib.header_symbols()
    assert len(declared) >= 30
    nm = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True, check=True)
    exported = {ln.split()[-1] for ln in nm.stdout.splitlines() if " T " in ln}
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for s in declared:
        getattr(L, s)


def test_python_bindings_cover_the_header(L):
    bound = set(_lib.SIGNATURES) | set(session.RING_SIGNATURES) | {"hs_attention_fused_noalloc"}
    assert set(_lib.header_symbols()) == bound


def test_python_bindings_match_header_arity(L):
    """Every ctypes binding passes as many arguments as the header's prototype declares."""
    import re

    text = re.sub(r"/\*.*?\*/", "", _lib.HEADER.read_text(), flags=re.S)
    arity = {}
    for name, params in re.findall(r"HS_API[^;(]*?\b(hs_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        params = params.strip()
        arity[name] = 0 if params in ("", "void") else params.count(",") + 1
    bound = {**_lib.SIGNATURES, **session.RING_SIGNATURES}
    assert set(bound) <= set(arity), sorted(set(bound) - set(arity))
    wrong = {n: (len(args), arity[n]) for n, (_, args) in bound.items() if len(args) != arity[n]}
    assert not wrong, f"(bound, declared) argument counts differ: {wrong}"


def test_abi_version(L):
    assert L.hs_abi_version() == 2


def test_rope_host_helpers_match_oracle(L):
    from headshot_b200 import rope

    np.testing.assert_array_equal(rope.periods(), oracle.rope_periods())
    for hp, wp in ((2, 3), (37, 37), (4, 7)):
        s1, c1 = rope.tables(None, hp, wp)
        s2, c2 = oracle.rope_tables(hp, wp)
        np.testing.assert_array_equal(s1, s2)
        np.testing.assert_array_equal(c1, c2)


def test_errors_are_status_codes(L):
    # null context: HS_ERR_INVALID with a message, no abort
    rc = L.hs_attention(None, None, None, None, None, 1, 1, 16, 64, _lib.HS_BF16, 0.0)
    assert rc == _lib.HS_ERR_INVALID and "null context" in _lib.last_error()
    rc = L.hs_sync(None)
    assert rc == _lib.HS_ERR_INVALID
    rc = L.hs_rope_tables(None, 2, 2, None, None)
    assert rc == _lib.HS_ERR_INVALID


def test_context_creation_fails_cleanly_without_a_gpu(L):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = L.hs_ctx_create(0, ctypes.byref(h))
    assert rc != _lib.HS_OK and h.value is None and _lib.last_error()


def test_engine_has_no_cpu_fallback():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from headshot_b200.engine import GpuContext

    with pytest.raises(_lib.HsError):
        GpuContext(0)


def test_ring_shard_matches_python(L):
    for n in (1, 7, 1001, 274800):
        for world in (1, 2, 3, 4, 8):
            if n < world:
                continue
            spans = [session.ring_shard(n, world, r) for r in range(world)]
            assert spans == [session.shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            lens = [e - s for s, e in spans]
            assert max(lens) - min(lens) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_ring_plan_visits_every_block_once(L, world):
    for rank in range(world):
        plans = [session.ring_plan(rank, world, s) for s in range(world)]
        assert sorted(p["src"] for p in plans) == list(range(world))
        assert plans[0]["src"] == rank and not plans[0]["load"]
        assert not plans[-1]["store"] and plans[-1]["send_to"] == -1
        assert all(p["load"] for p in plans[1:]) and all(p["store"] for p in plans[:-1])
    # what rank r sends at step s is what rank r+1 attends to at step s+1
    for s in range(world - 1):
        for rank in range(world):
            p = session.ring_plan(rank, world, s)
            nxt = session.ring_plan(p["send_to"], world, s + 1)
            assert nxt["src"] == p["src"] and nxt["recv_from"] in (rank, -1)
    with pytest.raises(_lib.HsError):
        session.ring_plan(0, 2, 2)
