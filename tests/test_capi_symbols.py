"""CPU checks of the C ABI boundary: the library loads, exports exactly the
entry points include/unicache_b200.h declares, and validates arguments
before touching the GPU."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from unicache_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "unicache_b200.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"^UCB_API\s+[\w\s\*]+?\b(ucb_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_binding_table():
    assert declared_symbols() == set(_capi.SIGNATURES), "ctypes table and header disagree"


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _capi.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (ucb_\w+)", out))
    assert exported == declared_symbols()


def test_version_and_error_reporting():
    lib = _capi.load()
    assert lib.ucb_version() >= 100
    rc = lib.ucb_kivi_pack_key(None, 0, 64, 4, 128, 512, 128, 2, 32, None, None, None, None)
    assert rc == _capi.UCB_ERR_INVALID
    assert "null pointer" in lib.ucb_last_error().decode()
    with pytest.raises(ValueError):
        _capi.check(rc, "ucb_kivi_pack_key")


@pytest.mark.parametrize(
    "bits,group,head_dim,expected",
    [(3, 32, 128, "bits"), (2, 48, 128, "group_size"), (2, 32, 96, "head_dim")],
)
def test_pack_rejects_unsupported_configurations(bits, group, head_dim, expected):
    lib = _capi.load()
    fake = ctypes.c_void_p(16)
    rc = lib.ucb_kivi_pack_key(fake, 0, 64, 4, head_dim, 512, 128, bits, group, fake, fake, fake, None)
    assert rc in (_capi.UCB_ERR_INVALID, _capi.UCB_ERR_UNSUPPORTED)
    assert expected in lib.ucb_last_error().decode()


def test_decode_rejects_bad_shapes_without_a_gpu():
    lib = _capi.load()
    fake = ctypes.c_void_p(256)
    rc = lib.ucb_decode_attention(fake, 28 * 128, 28, 4, 64, fake, 1, fake, 1, fake, fake, 1, 2, 2, 32, 0, 0.1,
                                  fake, fake, fake, 28 * 128, None, None)
    assert rc == _capi.UCB_ERR_UNSUPPORTED and "head_dim" in lib.ucb_last_error().decode()
    rc = lib.ucb_decode_attention(fake, 28 * 128, 28, 5, 128, fake, 1, fake, 1, fake, fake, 1, 2, 2, 32, 0, 0.1,
                                  fake, fake, fake, 28 * 128, None, None)
    assert rc == _capi.UCB_ERR_UNSUPPORTED


def test_struct_layouts_match_the_header():
    assert ctypes.sizeof(_capi.UcbSpan) == 80
    assert ctypes.sizeof(_capi.UcbDecodeCta) == 32
    assert ctypes.sizeof(_capi.UcbDecodePair) == 32
    assert _capi.load().ucb_decode_partial_bytes(128) == (16 + 8 * 128) * 4
