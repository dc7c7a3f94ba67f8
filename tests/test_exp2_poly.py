"""The FMA-pipe exp2 used by the attention softmax: coefficients and error bound.

The kernel's algorithm (eraserdit_b200/csrc/sm100_ptx.cuh, exp2_poly2) is
emulated step by step in fp32 numpy and compared with exact 2^x.  Its bound
(7.5e-5 relative) is far inside the 2^-9 rounding of the BF16 P operand, and
CUDA documents ex2.approx.ftz.f32 at about 2^-22 relative error, so both
paths feed the BF16 P conversion with negligible error.
"""
import re
from pathlib import Path

import numpy as np

HEADER = Path(__file__).resolve().parent.parent / "eraserdit_b200" / "csrc" / "sm100_ptx.cuh"


def _coefficients():
    text = HEADER.read_text()
    vals = dict(re.findall(r"constexpr float (kExp2C\d) = ([0-9a-fx.p+-]+)f;", text))
    return [np.float32(float.fromhex(vals[f"kExp2C{k}"])) for k in range(4)]


def _emulate(x):
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    j = np.floor(x).astype(np.float32)          # add.rm with 1.5 * 2^23, then subtract
    f = (x - j).astype(np.float32)              # exact
    c0, c1, c2, c3 = _coefficients()
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = p.view(np.uint32).astype(np.int64) + (j.astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_coefficients_match_generator():
    from eraserdit_b200.csrc.gen_exp2_poly import minimax_exp2
    coef, err = minimax_exp2(3)
    assert [np.float32(c) for c in coef] == _coefficients()
    assert err < 8e-5


def test_relative_error_over_softmax_range():
    # The softmax feeds x = s*c - m <= 8 (the running max may lag by 2^8).
    x = np.linspace(-125.0, 8.0, 400001, dtype=np.float32)
    y = _emulate(x).astype(np.float64)
    rel = np.abs(y / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() < 8e-5


def test_clamped_inputs_are_finite_and_tiny():
    y = _emulate(np.array([-np.inf, -1e4, -200.0, -126.0, -127.5], np.float32))
    assert np.all(np.isfinite(y)) and np.all(y >= 0) and np.all(y < 1e-37)
