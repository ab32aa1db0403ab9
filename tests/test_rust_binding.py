"""The Rust FFI crate (mlx-gen_b200/rust/qlinear-sys) against include/qlinear.h.

No Rust toolchain is available to compile the crate, so this checks it as text: every
function the header declares is declared in the crate with the same parameter count,
the `ql_epilogue` field order matches the header (and the ctypes mirror), and the
enum constants carry the header's values.
"""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "qlinear.h")
RS = os.path.join(ROOT, "mlx-gen_b200", "rust", "qlinear-sys", "src", "lib.rs")


def _strip_c_comments(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def _header_functions():
    src = _strip_c_comments(open(HDR).read())
    out = {}
    for m in re.finditer(r"\b(ql_[a-z_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


def _rust_functions():
    src = open(RS).read()
    block = src[src.index('extern "C"'):]
    out = {}
    for m in re.finditer(r"pub fn (ql_[a-z_]+)\s*\((.*?)\)\s*(->[^;]*)?;", block, flags=re.S):
        args = m.group(2).strip().rstrip(",")
        out[m.group(1)] = 0 if not args else len(args.split(","))
    return out


def test_every_header_function_is_bound():
    h, r = _header_functions(), _rust_functions()
    assert h, "no functions parsed from the header"
    assert set(h) == set(r), (set(h) ^ set(r))
    for name, n in h.items():
        assert r[name] == n, f"{name}: header {n} parameters, crate {r[name]}"


def _header_epilogue_fields():
    src = _strip_c_comments(open(HDR).read())
    body = re.search(r"typedef struct \{(.*?)\}\s*ql_epilogue;", src, flags=re.S).group(1)
    return [m.group(1) for m in re.finditer(r"\**\s*([a-z_0-9]+)\s*;", body)]


def test_epilogue_layout_matches():
    hdr = _header_epilogue_fields()
    src = open(RS).read()
    body = re.search(r"pub struct ql_epilogue \{(.*?)\}", src, flags=re.S).group(1)
    rs = re.findall(r"pub ([a-z_0-9]+):", body)
    assert hdr == rs
    from qlinear import _lib
    assert [f[0] for f in _lib.Epilogue._fields_] == hdr


@pytest.mark.parametrize("prefix", ["QL_F", "QL_BF", "QL_O", "QL_E", "QL_ACT_", "QL_KERNEL_"])
def test_enum_values_match(prefix):
    hsrc = _strip_c_comments(open(HDR).read())
    hv = dict((k, int(v)) for k, v in re.findall(r"\b(QL_[A-Z0-9_]+)\s*=\s*(\d+)", hsrc) if k.startswith(prefix))
    rv = dict((k, int(v)) for k, v in re.findall(r"pub const (QL_[A-Z0-9_]+): \w+ = (\d+);", open(RS).read())
              if k.startswith(prefix))
    assert hv and hv == rv
