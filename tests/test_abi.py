"""The C-ABI library builds, loads without a GPU and exports every entry point
declared in include/shrimp_b200.h (no compute calls here)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from hexo_bot_b200 import _lib
from hexo_bot_b200.build import lib_path

HEADER = Path(__file__).resolve().parent.parent / "include" / "shrimp_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^int\s+(sb_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert {"sb_forward_policy_value", "sb_hex_conv", "sb_hex_conv_ln", "sb_attn_pair"} <= syms


def test_library_exports_every_declared_symbol():
    assert lib_path().exists(), "native library not built (python -m hexo_bot_b200.build)"
    h = ctypes.CDLL(str(lib_path()))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(h, s)]
    assert not missing, missing


def test_binding_covers_header():
    assert declared_symbols() <= set(_lib.EXPORTED)


def test_abi_version_and_error_reporting():
    h = _lib.lib()
    assert h.sb_abi_version() == 1
    # host-side argument validation reports through sb_last_error without a GPU
    size = ctypes.c_size_t(0)
    rc = h.sb_forward_workspace_bytes(None, 4, 61, ctypes.byref(size))
    assert rc == 1
    assert "NULL" in _lib.last_error()


def test_struct_layout_matches_header():
    # channels/heads/num_blocks + 33-byte layout, then pointer-aligned fields
    assert _lib.Net.stem_w.offset == 48
    assert ctypes.sizeof(_lib.ConvBlockW) == 9 * 8
    assert ctypes.sizeof(_lib.AttnBlockW) == 15 * 8
    assert ctypes.sizeof(_lib.Inputs) == 4 * 16 + 8
    assert ctypes.sizeof(_lib.Outputs) == 6 * 8
