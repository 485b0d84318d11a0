"""The C-ABI library loads without a GPU and exports every symbol that
include/tmg_cuda.h declares; the ctypes table binds each of them."""
import re
from pathlib import Path

from tinyminigo_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "tmg_cuda.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tmg_[a-z0-9_]+)\s*\(", text)) - {"tmg_token_cb"})


def test_header_declares_entry_points():
    names = declared()
    assert "tmg_forward_token" in names and "tmg_generate" in names and len(names) >= 30


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_ctypes_table_covers_header():
    assert sorted(_lib.SIGNATURES) == declared()


def test_version_string():
    assert b"sm_100a" in _lib.lib().tmg_version()


RUST = Path(__file__).resolve().parents[1] / "rust" / "tmg-cuda-sys"


def test_rust_binding_declares_every_entry_point():
    # the Rust crate cannot be compiled here (no Rust toolchain); its extern
    # block must still name exactly the header's entry points, with as many
    # parameters as the C declarations
    src = (RUST / "src" / "lib.rs").read_text()
    block = src[src.index('unsafe extern "C" {'):]
    block = block[:block.index("\n}\n")]
    rust = dict(re.findall(r"pub fn (tmg_[a-z0-9_]+)\(([^)]*)\)", block, flags=re.S))
    assert sorted(rust) == declared()
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, params in rust.items():
        c_params = re.search(rf"\b{name}\s*\(([^)]*)\)", text, flags=re.S).group(1).strip()
        n_c = 0 if c_params in ("", "void") else c_params.count(",") + 1
        n_r = 0 if not params.strip() else params.count(",") + 1 - params.strip().endswith(",")
        assert n_c == n_r, (name, n_c, n_r)
    build = (RUST / "build.rs").read_text()
    assert "rustc-link-lib=dylib=tmg_cuda" in build and "tinyminigo_b200.build" in build
