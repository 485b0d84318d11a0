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
