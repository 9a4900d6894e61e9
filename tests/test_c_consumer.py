"""The C ABI as a foreign-language binder sees it (no GPU needed).

- tests/c_abi_consumer.c is compiled as strict C99 against
  include/headshot_cuda.h, linked against libheadshot_cuda.so and run: every
  entry point must resolve, and the host-side calls and the error contract
  must hold (see that file's header);
- the header must also compile as C++;
- the Rust FFI declarations of the `headshot-cuda` crate
  (headshot-cuda/src/ffi.rs, what the headshot-server engine binds) must
  declare every header function with the same parameter and return types,
  so the binding cannot drift from the header.  (No Rust toolchain exists in
  this build's container: the crate is checked here, not compiled.)
"""
from __future__ import annotations

import re
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from headshot_b200 import _lib
from headshot_b200.build import OUT as LIB_PATH
from headshot_b200.build import build

ROOT = _lib.HEADER.parent.parent
CONSUMER = ROOT / "tests" / "c_abi_consumer.c"
FFI_RS = ROOT / "headshot-cuda" / "src" / "ffi.rs"


@pytest.fixture(scope="module")
def lib_path():
    if not LIB_PATH.exists():
        build()
    return LIB_PATH


def _cc(name):
    exe = shutil.which(name)
    if exe is None:
        pytest.skip(f"{name} not installed")
    return exe


def test_header_compiles_as_cxx():
    subprocess.run([_cc("g++"), "-std=c++11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only", "-x", "c++",
                    str(_lib.HEADER)], check=True)


def test_c99_consumer_links_and_runs(lib_path, tmp_path):
    import torch

    exe = tmp_path / "c_abi_consumer"
    subprocess.run([_cc("gcc"), "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", str(_lib.HEADER.parent),
                    str(CONSUMER), "-o", str(exe), "-L", str(lib_path.parent), "-lheadshot_cuda",
                    f"-Wl,-rpath,{lib_path.parent}", "-lm"], check=True)
    tables = tmp_path / "rope_37x37.f32"
    args = [str(exe), str(tables)] + ([] if torch.cuda.is_available() else ["nogpu"])
    run = subprocess.run(args, capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "failures: 0" in run.stdout
    got = np.fromfile(tables, np.float32).reshape(2, 37 * 37, 64)
    sin, cos = oracle.rope_tables(37, 37)
    np.testing.assert_array_equal(got[0], sin)
    np.testing.assert_array_equal(got[1], cos)


def test_consumer_takes_every_entry_point():
    listed = set(re.findall(r"FN\((hs_\w+)\)", CONSUMER.read_text()))
    assert listed == set(_lib.header_symbols())


# ---- the crate's Rust declarations against the header -------------------

_C_TO_RUST = {
    "void": None,
    "hs_status": "hs_status",
    "hs_dtype": "hs_dtype",
    "int": "c_int",
    "float": "f32",
    "uint32_t": "u32",
    "uint64_t": "u64",
    "size_t": "usize",
}


def _rust_type(c: str) -> str | None:
    """C parameter/return type -> the Rust type a binding must use."""
    c = re.sub(r"\s+", " ", c.strip())
    c = re.sub(r"\s*\*", "*", c)
    stars = c.count("*")
    base = c.replace("*", "").strip()
    const = base.startswith("const ")
    base = base.removeprefix("const ").strip()
    inner = {"char": "c_char", "void": "c_void", "double": "f64", "hs_ctx": "hs_ctx", "hs_ring": "hs_ring"}.get(base)
    if stars == 0:
        return _C_TO_RUST[base]
    inner = inner or _C_TO_RUST[base]
    out = inner
    for i in range(stars):
        out = ("*const " if (const and i == 0) else "*mut ") + out
    return out


def _header_decls() -> dict[str, tuple[str | None, list[str | None]]]:
    text = re.sub(r"/\*.*?\*/", "", _lib.HEADER.read_text(), flags=re.S)
    decls = {}
    for ret, name, params in re.findall(r"HS_API\s+([\w\s\*]+?)\s*\b(hs_\w+)\s*\((.*?)\);", text, flags=re.S):
        ps = [] if params.strip() in ("", "void") else [p.strip() for p in params.split(",")]
        types = [_rust_type(re.match(r"(.*?)\w+$", p, flags=re.S).group(1)) for p in ps]
        decls[name] = (_rust_type(ret), types)
    return decls


def _rust_decls() -> dict[str, tuple[str | None, list[str]]]:
    text = FFI_RS.read_text()
    block = re.search(r"#\[link\(name = \"headshot_cuda\"\)\]\s*(?:unsafe )?extern \"C\" \{(.*?)\n\}", text,
                      flags=re.S)
    assert block, "headshot-cuda/src/ffi.rs has no extern \"C\" block for headshot_cuda"
    decls = {}
    for name, params, ret in re.findall(r"pub fn (hs_\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block.group(1), flags=re.S):
        ps = [p.strip() for p in params.split(",") if p.strip()]
        types = [re.sub(r"\s+", " ", p.split(":", 1)[1].strip()) for p in ps]
        decls[name] = (ret.strip() or None, types)
    return decls


def test_rust_binding_matches_header():
    header, rust = _header_decls(), _rust_decls()
    assert set(header) == set(_lib.header_symbols())
    assert set(rust) == set(header), f"missing {set(header) - set(rust)}, extra {set(rust) - set(header)}"
    for name, (ret, params) in header.items():
        r_ret, r_params = rust[name]
        assert r_ret == ret, f"{name}: returns {r_ret}, header says {ret}"
        assert r_params == params, f"{name}: parameters {r_params}, header says {params}"


# ---- the crate's safe layer against its own declarations --------------------

LIB_RS = ROOT / "headshot-cuda" / "src" / "lib.rs"
PATCH_RS = ROOT / "headshot-cuda" / "patches" / "engine_attention.rs"


def _call_args(text: str, start: int) -> list[str]:
    """Top-level comma-separated arguments of the call whose '(' is at text[start]."""
    depth, args, cur = 0, [], []
    for ch in text[start:]:
        if ch in "([{":
            depth += 1
            if depth == 1:
                continue
        elif ch in ")]}":
            depth -= 1
            if depth == 0:
                if "".join(cur).strip():
                    args.append("".join(cur).strip())
                return args
        if depth == 1 and ch == ",":
            args.append("".join(cur).strip())
            cur = []
        elif depth >= 1:
            cur.append(ch)
    raise AssertionError("unbalanced call")


def test_safe_layer_calls_declared_functions_with_their_arity():
    """The crate is not compiled here (no Rust toolchain): every ffi::hs_* call in src/lib.rs
    must name a function src/ffi.rs declares and pass as many arguments as it takes."""
    declared = _rust_decls()
    text = LIB_RS.read_text()
    calls = [(m.group(1), m.end() - 1) for m in re.finditer(r"ffi::(hs_\w+)\(", text)]
    assert len(calls) >= 15
    for name, paren in calls:
        assert name in declared, f"lib.rs calls undeclared {name}"
        n_args = len(_call_args(text, paren))
        assert n_args == len(declared[name][1]), f"{name}: {n_args} arguments, ffi.rs declares {len(declared[name][1])}"


def test_engine_patch_uses_the_safe_layer():
    """patches/engine_attention.rs uses only items src/lib.rs defines."""
    lib = LIB_RS.read_text()
    patch = PATCH_RS.read_text()
    for item in set(re.findall(r"headshot_cuda::(\w+)", patch)):
        assert re.search(rf"pub (struct|fn|enum) {item}\b", lib), f"lib.rs has no pub {item}"
    for method in set(re.findall(r"\.cuda\.(\w+)\(", patch)):
        assert re.search(rf"pub fn {method}\(", lib), f"Context has no method {method}"
