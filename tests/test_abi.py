"""The C-ABI library loads on CPU and exports every symbol the header declares."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "eraserdit_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(erd_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    from eraserdit_b200.csrc.build import LIBRARY, build
    if not LIBRARY.exists():
        build()
    return ctypes.CDLL(str(LIBRARY))


def test_header_declares_entry_points():
    names = _declared()
    for expected in ("erd_abi_version", "erd_error_string", "erd_rope_axis_table",
                     "erd_qk_norm_rope", "erd_attn_fwd_bf16"):
        assert expected in names


def test_every_declared_symbol_is_exported(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_binding_covers_header_and_version(lib):
    from eraserdit_b200 import _native
    assert set(_native.SIGNATURES) == set(_declared())
    lib.erd_abi_version.restype = ctypes.c_int
    assert lib.erd_abi_version() == _native.ABI_VERSION
    lib.erd_error_string.restype = ctypes.c_char_p
    assert lib.erd_error_string(-3).decode().startswith("pointer or stride")
