"""Rust FFI declarations for include/jaxrs_cuda.h.

`python jax-rs_b200/rust_ffi.py` prints the `extern "C"` block (plus the
opaque handle types and the status/op constants) that a jax-rs
`src/backend/cuda.rs` needs to bind every entry point of the C ABI.
The C types map one to one: `int` -> `c_int`, `int64_t` -> `i64`,
`size_t` -> `usize`, `float` -> `f32`, pointers keep their constness level by
level, `jx_stream_t` -> `JxStream`, and the opaque handles (`jx_tape`,
`jx_graph`, `jx_program`, `jx_mlp`) become zero-sized `#[repr(C)]` structs.
`python jax-rs_b200/rust_ffi.py --update INTEGRATION.md` rewrites the block
between that file's rust-ffi markers.
"""
from __future__ import annotations

import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(HERE, "..", "include", "jaxrs_cuda.h")

SCALARS = {
    "int": "c_int", "unsigned int": "c_uint", "int32_t": "i32", "int64_t": "i64", "uint64_t": "u64",
    "size_t": "usize", "float": "f32", "char": "c_char", "void": "c_void", "jx_stream_t": "JxStream",
    "jx_tape": "JxTape", "jx_graph": "JxGraph", "jx_program": "JxProgram", "jx_mlp": "JxMlp",
}
OPAQUE = ("JxTape", "JxGraph", "JxProgram", "JxMlp")
RUST_KEYWORDS = {"in", "type", "ref", "fn", "loop", "mod", "move", "match", "self", "impl", "use", "where"}


def _strip(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return "\n".join(line for line in text.splitlines() if not line.lstrip().startswith("#"))


def declarations(header: str = HEADER):
    """[(name, return C type, [(param name, C type)])] in header order."""
    with open(header) as f:
        body = _strip(f.read())
    out = []
    for d in re.findall(r"JX_API\s+([^;]*?)\s*;", body, flags=re.S):
        d = " ".join(d.split())
        m = re.match(r"(.*?)\b(jx_\w+)\s*\((.*)\)$", d)
        if not m:
            raise ValueError("cannot parse declaration: " + d)
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        params = []
        if args and args != "void":
            for i, a in enumerate(a.strip() for a in args.split(",")):
                pm = re.match(r"(.*?)([A-Za-z_]\w*)$", a)
                if pm and not pm.group(1).strip().endswith(("const", "unsigned")) and pm.group(1).strip():
                    params.append((pm.group(2), pm.group(1).strip()))
                else:
                    params.append((f"arg{i}", a))
        out.append((name, ret, params))
    return out


def rust_type(ctype: str) -> str:
    """C declaration type (without the name) -> Rust FFI type."""
    t = ctype.replace("*", " * ").split()
    base_const = False
    base = []
    i = 0
    while i < len(t) and t[i] != "*":
        if t[i] == "const":
            base_const = True
        else:
            base.append(t[i])
        i += 1
    base_name = " ".join(base)
    if base_name not in SCALARS:
        raise ValueError("no Rust type for C type " + repr(ctype))
    cur = SCALARS[base_name]
    pointee_const = base_const
    while i < len(t):
        assert t[i] == "*"
        i += 1
        star_const = i < len(t) and t[i] == "const"
        if star_const:
            i += 1
        cur = ("*const " if pointee_const else "*mut ") + cur
        pointee_const = star_const
    return cur


def constants(header: str = HEADER):
    """[(name, value)] of the header's integer #defines (JX_OK, JX_BIN_ADD, ...)."""
    with open(header) as f:
        return re.findall(r"^#define (JX_[A-Z0-9_]+) (-?\d+)\b", f.read(), flags=re.M)


def rust_block(header: str = HEADER) -> str:
    lines = ["use std::os::raw::{c_char, c_int, c_uint, c_void};", "",
             "pub type JxStream = *mut c_void; // a cudaStream_t; null = the legacy default stream"]
    for o in OPAQUE:
        lines.append(f"#[repr(C)] pub struct {o} {{ _private: [u8; 0] }}")
    lines.append("")
    for name, value in constants(header):
        lines.append(f"pub const {name}: c_int = {value};")
    lines += ["", '#[link(name = "jaxrs_cuda")]', 'extern "C" {']
    for name, ret, params in declarations(header):
        args = ", ".join(f"{p + '_' if p in RUST_KEYWORDS else p}: {rust_type(t)}" for p, t in params)
        lines.append(f"    pub fn {name}({args}) -> {rust_type(ret)};")
    lines.append("}")
    return "\n".join(lines) + "\n"


def update_doc(path: str) -> None:
    """Rewrite the block between the rust-ffi markers of a Markdown file."""
    with open(path) as f:
        doc = f.read()
    begin, end = "<!-- rust-ffi:begin -->\n```rust\n", "```\n<!-- rust-ffi:end -->"
    i, j = doc.index(begin) + len(begin), doc.index(end)
    with open(path, "w") as f:
        f.write(doc[:i] + rust_block() + doc[j:])


if __name__ == "__main__":
    if len(sys.argv) == 3 and sys.argv[1] == "--update":
        update_doc(sys.argv[2])
    else:
        sys.stdout.write(rust_block())
