"""The Rust binding (burn-deltanet_b200/rust/, not compiled here: no Rust
toolchain) against the C ABI it binds.

Every `#[repr(C)]` struct in deltacore-sys must list the header's fields in the
header's order with the matching C type, every constant must carry the
header's value, and every function it declares must be exported by
libdeltacore.so.  A drift between the two would be a silent memory-layout bug
on the Rust side, so it is checked on every CPU run."""
import ctypes
import importlib
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "deltacore.h")
SYS = os.path.join(ROOT, "burn-deltanet_b200", "rust", "deltacore-sys", "src", "lib.rs")

C_TO_RUST = {
    "int64_t": "i64", "int32_t": "i32", "uint32_t": "u32", "uint64_t": "u64", "double": "f64", "float": "f32",
    "const void *": "*const c_void", "void *": "*mut c_void", "const float *": "*const f32", "float *": "*mut f32",
    "dc_chunk_args": "dc_chunk_args",
}


def header_structs():
    text = open(HEADER).read()
    out = {}
    for body, name in re.findall(r"typedef struct \w+ \{(.*?)\} (\w+);", text, re.S):
        fields = []
        for decl in body.split(";"):
            decl = re.sub(r"/\*.*?\*/", "", decl, flags=re.S).strip()
            if not decl:
                continue
            m = re.match(r"((?:const )?\w+)\s*(.*)", decl)
            base, names = m.group(1).strip(), m.group(2)
            for n in names.split(","):
                n = n.strip()
                ty = base
                while n.startswith("*"):
                    ty, n = ty + " *", n[1:].strip()
                fields.append((n, ty))
        out[name] = fields
    return out


def rust_structs():
    text = open(SYS).read()
    out = {}
    for name, body in re.findall(r"pub struct (\w+) \{(.*?)\n\}", text, re.S):
        out[name] = re.findall(r"pub (\w+): ([^,]+),", body)
    return out


def test_every_header_struct_has_a_matching_repr_c_struct():
    hs, rs = header_structs(), rust_structs()
    assert set(hs) == {"dc_chunk_args", "dc_step_args", "dc_chunk_bwd_args", "dc_out_norm_args",
                       "dc_qkv_prologue_args", "dc_gate_args"}
    for name, fields in hs.items():
        assert name in rs, f"{name} missing from deltacore-sys"
        got = [(n, t.strip()) for n, t in rs[name]]
        want = [(n, C_TO_RUST[t]) for n, t in fields]
        assert got == want, f"{name}: rust {got} != header {want}"


def test_constants_carry_the_header_values():
    h = open(HEADER).read()
    r = open(SYS).read()
    consts = dict(re.findall(r"pub const (\w+): \w+ = ([^;]+);", r))
    for name, val in re.findall(r"(DC_\w+) = (\d+)", h):
        assert int(consts[name], 0) == int(val), name
    for name, val in re.findall(r"#define (DC_(?:FLAG|PROLOGUE|GATE)_\w+) (0x[0-9a-f]+|\d+)u?", h):
        assert int(consts[name], 0) == int(val, 0), name
    assert consts["DC_NOALLOC_SCRATCH_BYTES"].replace(" ", "") == "64<<20"
    assert "(64ull << 20)" in h


def test_declared_functions_are_exported_by_the_library():
    abi = importlib.import_module("burn-deltanet_b200._abi")
    path = abi.LIB_PATH
    if not os.path.exists(path):
        pytest.skip("libdeltacore.so not built")
    lib = ctypes.CDLL(path)
    fns = re.findall(r"pub fn (dc_\w+)\(", open(SYS).read())
    assert len(fns) >= 17
    for fn in fns:
        assert hasattr(lib, fn), fn
    hdr = set(re.findall(r"DC_API [^(]*?\b(dc_\w+)\(", open(HEADER).read()))
    assert hdr == set(fns), hdr ^ set(fns)
