"""CPU checks of the Rust FFI crate (rust/vmlm-ops-cuda), which cannot be
compiled here (no cargo): every C entry point it binds is declared in
include/vmlm_cuda.h with the same number of arguments and is exported by the
built library, and its `kernels` module keeps the reference operators'
names and parameter lists (ops/src/kernels.rs:1200-1204, 1256-1261,
987-995, 407-415)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(ROOT, "rust", "vmlm-ops-cuda")


def _src():
    with open(os.path.join(CRATE, "src", "lib.rs")) as f:
        return f.read()


def _header():
    with open(os.path.join(ROOT, "include", "vmlm_cuda.h")) as f:
        return f.read()


def _args(text):
    return [a for a in (x.strip() for x in text.split(",")) if a and a != "void"]


def test_crate_bindings_match_the_header_and_the_library():
    from sparrow_b200._lib import lib
    h, rs = _header(), _src()
    bound = re.findall(r"pub fn (vmlm_\w+)\(([^)]*)\)", rs, re.S)
    assert len(bound) >= 20
    L = lib()
    for name, args in bound:
        m = re.search(r"VMLM_API [^;]*?\b%s\(([^)]*)\)" % name, h, re.S)
        assert m, f"{name} is not declared in the header"
        assert len(_args(m.group(1))) == len(_args(args)), name
        assert hasattr(L, name), f"{name} is not exported"


def test_crate_kernels_keep_the_reference_signatures():
    rs = _src()
    want = {
        "gemm_nt_int8": "a: *const f32, q: *const i8, scale: *const f32, c: *mut f32, m: usize, n: usize, k: usize",
        "gemm_nt_bf16": "a: *const f32, b: *const u16, c: *mut f32, m: usize, n: usize, k: usize",
        "gemm_nt": "a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize, acc: bool",
        "gemm": "a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize, acc: bool",
    }
    for name, params in want.items():
        m = re.search(r"pub unsafe fn %s\(([^)]*)\)" % name, rs, re.S)
        assert m, name
        assert " ".join(m.group(1).split()) == params, name
    # the misuse convention of the VM: print, then exit 9 (core/src/interp.rs:752-806)
    assert "exit_i(9)" in rs and "vmlm_last_error" in rs


def test_crate_manifest_names_the_library():
    with open(os.path.join(CRATE, "Cargo.toml")) as f:
        toml = f.read()
    assert 'name = "vmlm-ops-cuda"' in toml and "vmlm-sys" in toml
    with open(os.path.join(CRATE, "build.rs")) as f:
        assert "rustc-link-lib=dylib=vmlm_cuda" in f.read()
    assert ctypes.sizeof(ctypes.c_size_t) == 8  # usize <-> size_t on the x86-64 targets
