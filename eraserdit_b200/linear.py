"""The self-attention path's linear layers on ``erd_linear_bf16``.

``linear_bf16(x, weight, bias)`` computes ``F.linear(x, weight, bias)`` for
BF16 tensors (FP32 accumulation, bias added in FP32, one rounding to BF16) on
the sm_100a tensor cores.  It serves the Q/K/V projections of
``EraserDiTAttentionProcessor.self_attn``
(``models/dits/eraserdit_attention.py:248-253``; one product over the
concatenated weights) and its output projection ``_project_output``
(``:216-229``).  There is no fallback: an unsupported shape raises.
"""

from __future__ import annotations

import torch

from . import _native

TILE_N = 256  # output columns per tile: n must be a multiple
TILE_K = 64   # reduction depth per pipeline stage: k must be a multiple


def _rows(t: torch.Tensor) -> tuple[int, int] | None:
    """(rows, row stride) of a tensor viewed as [rows, last dim], or None when
    its leading dimensions do not form one strided row axis."""
    lead = t.shape[:-1]
    rows = 1
    for d in lead:
        rows *= d
    stride = t.stride(-2) if t.dim() >= 2 else t.shape[-1]
    expect = stride
    for d, s in zip(reversed(lead), reversed(t.stride()[:-1])):
        if d > 1 and s != expect:
            return None
        expect *= d
    return rows, stride


def _launch(x, weight, bias, out) -> None:
    n, k = weight.shape
    m, ldx = _rows(x)
    _, ldy = _rows(out)
    if m == 0:
        return
    lib = _native.load()
    device = x.device
    with torch.cuda.device(device):
        rc = lib.erd_linear_bf16(x.data_ptr(), ldx, weight.data_ptr(), weight.stride(0),
                                 _native.ptr(bias), out.data_ptr(), ldy, m, n, k,
                                 _native.status_word(device).data_ptr(),
                                 _native.stream_handle(device))
    _native.check(rc, "erd_linear_bf16")


def linear_bf16(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T + bias`` for BF16 CUDA tensors: x [..., k], weight [n, k],
    bias [n] (or None); the result [..., n] (written into ``out`` when given)."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("linear_bf16 needs CUDA bfloat16 tensors")
    if weight.dim() != 2 or weight.shape[1] != x.shape[-1]:
        raise ValueError("weight must be [n, k] with k = x.shape[-1]")
    n, k = weight.shape
    if n % TILE_N or k % TILE_K:
        raise ValueError(f"linear_bf16 needs n % {TILE_N} == 0 and k % {TILE_K} == 0")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.shape != (n,)
                             or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous BF16 [n] tensor")
    if weight.stride(1) != 1:
        raise ValueError("weight must have a contiguous last dimension")
    if out is None:
        out = torch.empty(*x.shape[:-1], n, device=x.device, dtype=torch.bfloat16)
    elif out.shape != (*x.shape[:-1], n) or out.dtype != torch.bfloat16:
        raise ValueError("out must be BF16 [..., n]")
    if x.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("x and out need a contiguous last dimension")
    if _rows(x) is not None and _rows(out) is not None:
        _launch(x, weight, bias, out)
    elif x.dim() >= 3:
        # e.g. [B, L, k] rows of wider [B, L_slot, k] slots: one product per
        # leading index (rows within it are evenly strided)
        for xs, ys in zip(x.unbind(0), out.unbind(0)):
            linear_bf16(xs, weight, bias, out=ys)
    else:
        raise ValueError("x and out must be viewable as [rows, last dim] with one row stride")
    return out


def linear_bf16_scatter(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                        out: torch.Tensor, scatter_col0: int, dest_bases: list[int],
                        group_cols: int, batch_stride: int, token_stride: int) -> None:
    """``linear_bf16`` of ``x`` [B, L, k] with the output columns from
    ``scatter_col0`` on stored into ``dest_bases`` (``erd_linear_bf16_scatter``):
    column j of token (b, t) goes to ``dest_bases[(j - scatter_col0) //
    group_cols]`` at element ``b * batch_stride + t * token_stride +
    (j - scatter_col0) % group_cols``; the columns below go to ``out`` [B, L, n]."""
    import ctypes
    if x.dim() != 3 or x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be a contiguous BF16 [B, L, k] tensor")
    n, k = weight.shape
    if out.shape != (*x.shape[:-1], n) or not out.is_contiguous():
        raise ValueError("out must be a contiguous BF16 [B, L, n] tensor")
    m = x.shape[0] * x.shape[1]
    if m == 0:
        return
    lib = _native.load()
    device = x.device
    bases = (ctypes.c_void_p * len(dest_bases))(*dest_bases)
    with torch.cuda.device(device):
        rc = lib.erd_linear_bf16_scatter(
            x.data_ptr(), k, weight.data_ptr(), weight.stride(0), _native.ptr(bias),
            out.data_ptr(), n, m, n, k, scatter_col0, bases, len(dest_bases), group_cols,
            x.shape[1], batch_stride, token_stride, _native.status_word(device).data_ptr(),
            _native.stream_handle(device))
    _native.check(rc, "erd_linear_bf16_scatter")
