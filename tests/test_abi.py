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


def test_ring_state_size(lib):
    """Per query tile of 128 rows: 64 fp32 O columns plus the running max and
    sum; tiles = ceil(seg_len / 128) per query segment."""
    lib.erd_ring_state_bytes.restype = ctypes.c_size_t
    assert lib.erd_ring_state_bytes(2, 16, 4080, 2) == 2 * 16 * (32 * 2) * (64 * 128 + 2 * 128) * 4
    assert lib.erd_ring_state_bytes(1, 1, 1, 1) == (64 * 128 + 2 * 128) * 4
    assert lib.erd_ring_state_bytes(0, 16, 4080, 2) == 0
    assert lib.erd_ring_state_bytes(1, 16, 4080, 17) == 0
