"""The Rust crate skeleton (uncompiled here: no cargo on this machine) against
the C header it binds.

Every `extern "C"` function that rust/src/ffi.rs declares must exist in
include/fa_b200.h with the same number of parameters, so a maintainer who
builds the crate gets link-compatible declarations.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fa_b200.h")
FFI = os.path.join(ROOT, "flash-attention-cpu_b200", "rust", "src", "ffi.rs")


def _params(arglist: str) -> int:
    arglist = arglist.strip()
    if not arglist or arglist == "void":
        return 0
    return arglist.count(",") + 1


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(([^)]*)\)", text):
        out[m.group(1)] = _params(m.group(2))
    return out


def ffi_functions():
    text = open(FFI).read()
    block = text[text.index('extern "C" {'):]
    out = {}
    for m in re.finditer(r"pub fn (fa_\w+)\(([^)]*)\)", block):
        args = re.sub(r"\s+", " ", m.group(2)).strip().rstrip(",")
        out[m.group(1)] = _params(args)
    return out


def test_every_rust_declaration_matches_the_header():
    hdr, ffi = header_functions(), ffi_functions()
    assert len(ffi) >= 10
    for name, n in ffi.items():
        assert name in hdr, f"{name} is not in include/fa_b200.h"
        assert hdr[name] == n, f"{name}: {n} parameters in ffi.rs, {hdr[name]} in the header"


def test_the_crate_entry_points_are_bound():
    ffi = ffi_functions()
    for v in ("v1", "v2", "v3"):
        assert f"fa_flash_attention_{v}" in ffi
        assert f"fa_flash_attention_multihead_{v}" in ffi
    assert "fa_flash_attention_backward" in ffi
