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


def test_integration_binding_asserts_current_version():
    """The ctypes stub a maintainer copies from INTEGRATION.md must accept the
    library this repository builds (the version in the header and the binding)."""
    from eraserdit_b200 import _native
    text = (ROOT / "INTEGRATION.md").read_text()
    asserted = [int(v) for v in re.findall(r"assert _lib\.erd_abi_version\(\) == (\d+)", text)]
    assert asserted == [_native.ABI_VERSION]
    header = (ROOT / "include" / "eraserdit_b200.h").read_text()
    assert int(re.search(r"#define ERD_ABI_VERSION (\d+)", header).group(1)) == _native.ABI_VERSION


def test_ring_state_size(lib):
    """Per query tile of 128 rows: 64 fp32 O columns plus the running max and
    sum; tiles = ceil(seg_len / 128) per query segment."""
    lib.erd_ring_state_bytes.restype = ctypes.c_size_t
    assert lib.erd_ring_state_bytes(2, 16, 4080, 2) == 2 * 16 * (32 * 2) * (64 * 128 + 2 * 128) * 4
    assert lib.erd_ring_state_bytes(1, 1, 1, 1) == (64 * 128 + 2 * 128) * 4
    assert lib.erd_ring_state_bytes(0, 16, 4080, 2) == 0
    assert lib.erd_ring_state_bytes(1, 16, 4080, 17) == 0


def test_ring_entry_rejects_bad_arguments_before_any_device_call(lib):
    """Argument errors of erd_attn_fwd_ring_bf16 come back as the documented
    codes (-1 null pointer, -2 bad shape) before the device is touched."""
    from eraserdit_b200 import _native
    fn = lib.erd_attn_fwd_ring_bf16
    fn.argtypes = _native.SIGNATURES["erd_attn_fwd_ring_bf16"]
    fn.restype = ctypes.c_int
    lens = (ctypes.c_int32 * 2)(100, 100)
    big = (ctypes.c_int32 * 2)(100, 300)

    def call(state_mode=0, kv_nseg=2, kv_lens=lens, q_nseg=2, kv_seg_len=128, out=1 << 20):
        return fn(1 << 20, 1 << 20, 1 << 20, *([64] * 12), 1, 1, 128, q_nseg, lens, kv_seg_len,
                  kv_nseg, kv_lens, 64, 0.125, out, 64, 64, 64, 64, None, None, 0, state_mode,
                  None, None)

    assert call(state_mode=4) == -2
    assert call(state_mode=-1) == -2
    assert call(kv_lens=None) == -1
    assert call(kv_nseg=0) == -2
    assert call(kv_nseg=17) == -2
    assert call(q_nseg=0) == -2
    assert call(kv_seg_len=0) == -2
    assert call(kv_lens=big) == -2          # a segment longer than its slot
    assert call(out=None) == -1             # BF16 output requested, no destination


def test_scatter_linear_rejects_bad_layouts_before_any_device_call(lib):
    """Layout errors of erd_linear_bf16_scatter come back as the documented
    codes (-1 null pointer, -2 bad shape, -3 misaligned) before the device is
    touched."""
    from eraserdit_b200 import _native
    fn = lib.erd_linear_bf16_scatter
    fn.argtypes = _native.SIGNATURES["erd_linear_bf16_scatter"]
    fn.restype = ctypes.c_int
    four = (ctypes.c_void_p * 4)(*([1 << 20] * 4))

    def call(col0=4096, dests=four, ndest=4, group=512, rows=64, bs=256, ts=1536, m=128):
        return fn(1 << 20, 2048, 1 << 20, 2048, None, 1 << 20, 6144, m, 6144, 2048, col0,
                  dests, ndest, group, rows, bs, ts, None, None)

    assert call(dests=None) == -1
    assert call(group=384) == -2           # not a power of two
    assert call(group=64, ndest=32) == -2   # narrower than 128 columns, more than 16 groups
    assert call(ndest=3) == -2             # 3 x 512 columns do not cover n - col0
    assert call(col0=4000) == -2           # not a multiple of 256
    assert call(rows=48) == -2             # m not a multiple of the rows per batch entry
    assert call(ts=1537) == -3             # destination stride not 16-byte aligned
    assert call(dests=(ctypes.c_void_p * 4)(1 << 20, 1 << 20, (1 << 20) + 2, 1 << 20)) == -3
