"""Mask-aware block-sparse self-attention on the B200 kernels.

Mirrors ``layers/attention/backends/mask_sta.py``: ``MaskSTA`` (``:134-194``)
built from a latent mask for one window, ``report``/``close``, the
``mask_sta_window`` context and ``current_mask_sta`` (``:197-210``).
Differences from the reference, by design:

- the attention runs in BF16 on ``erd_attn_fwd_sparse_bf16`` (the reference
  quantises Q/K to INT8 and V to E4M3 for its SM89 kernel);
- any batch, and the pattern is a parameter (:class:`StaGeometry`): the
  reference's constants by default, the benchmark's 3 x 9 x 9-cell window
  with ``CONFIG4_GEOMETRY``;
- no library path or SHA: the one in-tree library serves every entry point.

Besides the drop-in operator (inputs and output in raster token order, with
a gather into tile order and the output scattered back by the kernel), the
layer and the sequence-parallel path run the whole attention in tile order
with a :class:`SparsePlan` and no gather at all.
"""

from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar

import torch

from . import _native
from .attention import _check_operand, _segmented_call, validate_bshd_qkv
from .sparse_pattern import (REFERENCE_GEOMETRY, SparseSchedule, StaGeometry, block_mask,
                             build_schedule, protected_query_blocks, tile_order)

_active_window = ContextVar("eraserdit_b200_mask_sta_window", default=None)


class SparsePlan:
    """The kernel's work lists for one block pattern, on one device.

    ``blocks``: bool [query blocks of 128, key blocks of ``kv_block``] over the
    tile-ordered sequence.  ``seg_blocks`` / ``tiles_per_seg`` describe a
    segmented layout (sequence-parallel receive buffers).  ``order`` (optional)
    is the raster index of each tile-order position.
    """

    def __init__(self, blocks: torch.Tensor, kv_block: int, device, *,
                 seg_blocks: list[int] | None = None, tiles_per_seg: int | None = None,
                 order: torch.Tensor | None = None) -> None:
        device = torch.device(device)
        # The work lists are built where the pattern lives (on the device when
        # the mask is there: a handful of launches per window, no host loop).
        built = build_schedule(blocks.to(device), kv_block, seg_blocks=seg_blocks,
                               tiles_per_seg=tiles_per_seg)
        self.host: SparseSchedule = built
        self.schedule = built.schedule.to(device).contiguous()
        self.entries = built.entries.to(device).contiguous()
        self.blocks = blocks.cpu()
        self.kv_block = kv_block
        self.seg_blocks = seg_blocks
        self.tiles_per_seg = tiles_per_seg
        self.order = None if order is None else order.to(device=device, dtype=torch.int32)
        self.device = device

    @classmethod
    def from_mask(cls, mask: torch.Tensor | None, geom: StaGeometry, device, **kw) -> "SparsePlan":
        """Pattern and work lists of one window, computed on ``device``."""
        device = torch.device(device)
        order, _ = tile_order(geom, device)
        blocks = block_mask(None if mask is None else mask.to(device), geom, device)
        return cls(blocks, geom.kv_block, device, order=order, **kw)

    def for_segments(self, seg_blocks: list[int], tiles_per_seg: int) -> "SparsePlan":
        """The same pattern over a segmented layout (one segment per source rank)."""
        return SparsePlan(self.blocks, self.kv_block, self.device, seg_blocks=seg_blocks,
                          tiles_per_seg=tiles_per_seg, order=self.order)

    def launch_args(self) -> tuple:
        return (self.schedule.data_ptr(), int(self.schedule.shape[0]), self.entries.data_ptr(),
                int(self.entries.numel()))

    @property
    def keep_fraction(self) -> float:
        return self.host.keep_fraction


def sparse_attention_into(query, key, value, out, softmax_scale: float, plan: SparsePlan, *,
                          batch, heads, seg_len, nseg, seg_lens, q_strides, k_strides, v_strides,
                          o_strides, out_rows: torch.Tensor | None = None) -> None:
    """Enqueue ``erd_attn_fwd_sparse_bf16`` with segmented strides."""
    _segmented_call("erd_attn_fwd_sparse_bf16", query, key, value, out, softmax_scale,
                    batch=batch, heads=heads, seg_len=seg_len, nseg=nseg, seg_lens=seg_lens,
                    q_strides=q_strides, k_strides=k_strides, v_strides=v_strides,
                    o_strides=o_strides, extra=(*plan.launch_args(), _native.ptr(out_rows)))


def sparse_attention_bshd(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          softmax_scale: float, plan: SparsePlan, out: torch.Tensor | None = None,
                          out_rows: torch.Tensor | None = None) -> torch.Tensor:
    """Block-sparse attention on tile-ordered BSHD tensors (one segment).
    With ``out_rows`` the output row of tile position i is ``out_rows[i]``."""
    validate_bshd_qkv(query, key, value)
    if query.shape != key.shape or query.dtype != torch.bfloat16 or query.shape[-1] != 64:
        raise ValueError("sparse attention needs equal BF16 BSHD shapes with head_dim 64")
    batch, seq, heads, _ = query.shape
    if seq != plan.blocks.shape[0] * 128:
        raise ValueError(f"the plan covers {plan.blocks.shape[0] * 128} tokens, not {seq}")
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    for name, t in (("query", query), ("key", key), ("value", value), ("out", out)):
        _check_operand(name, t)
    st = lambda t: (t.stride(1), t.stride(2), t.stride(0), 0)
    sparse_attention_into(query, key, value, out, softmax_scale, plan, batch=batch, heads=heads,
                          seg_len=seq, nseg=1, seg_lens=None, q_strides=st(query),
                          k_strides=st(key), v_strides=st(value), o_strides=st(out),
                          out_rows=out_rows)
    return out


def gather_tokens(src: torch.Tensor, index: torch.Tensor, out: torch.Tensor | None = None
                  ) -> torch.Tensor:
    """``out[:, i] = src[:, index[i]]`` for BF16 [B, S, ...] on the device."""
    batch, tokens = src.shape[0], index.numel()
    row = src[0, 0].numel()
    if out is None:
        out = torch.empty((batch, tokens, *src.shape[2:]), dtype=src.dtype, device=src.device)
    if src.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("gather_tokens moves BF16 rows")
    if not (src[0, 0].is_contiguous() and out[0, 0].is_contiguous()):
        raise ValueError("rows must be contiguous")
    lib = _native.load()
    with torch.cuda.device(src.device):
        rc = lib.erd_gather_tokens(src.data_ptr(), src.stride(1), src.stride(0), src.shape[1],
                                   out.data_ptr(), out.stride(1), out.stride(0), index.data_ptr(),
                                   batch, tokens, row, _native.stream_handle(src.device))
    _native.check(rc, "erd_gather_tokens")
    return out


class MaskSTA:
    """One window's mask-protected block-sparse attention operator."""

    def __init__(self, mask, grid, library_path=None, library_sha256: str = "",
                 geometry: StaGeometry = REFERENCE_GEOMETRY) -> None:
        del library_path, library_sha256  # one in-tree library serves every entry point
        if tuple(grid) != geometry.grid or tuple(mask.shape[-3:]) != geometry.grid:
            raise ValueError(f"mask STA supports only token grid {geometry.grid}")
        if mask.device.type != "cuda" or torch.cuda.get_device_capability(mask.device) != (10, 0):
            raise ValueError("mask STA requires an sm_100 (B200) CUDA device")
        self.geometry = geometry
        self.device = mask.device
        self.setup_stream = torch.cuda.current_stream(self.device)
        order, coords = tile_order(geometry)
        protected = protected_query_blocks(mask, order, geometry)
        self.plan = SparsePlan(block_mask(mask, geometry), geometry.kv_block, self.device,
                               order=order)
        self.row_order = self.plan.order
        binary = mask.reshape(geometry.grid) > 0
        self._report = dict(
            enabled=True, grid=geometry.grid, background_window=geometry.window,
            protect_kernel=geometry.protect, query_block=geometry.query_block,
            kv_block=geometry.kv_block, calls=0, closed=False,
            keep_fraction=float(self.plan.blocks.double().mean()),
            protected_query_blocks=int(protected.sum()),
            total_query_blocks=geometry.tokens // geometry.query_block,
            mask_tokens=int(binary.sum()))

    def report(self) -> dict:
        return dict(self._report)

    def close(self) -> None:
        self._report["closed"] = True
        self.plan = self.row_order = None

    def __call__(self, q, k, v, scale, peripheral=None):
        del peripheral  # BF16 operands go straight to the kernel
        if self._report["closed"]:
            raise RuntimeError("mask STA window is closed")
        tokens = self.geometry.tokens
        if (q.dim() != 4 or q.shape[1] != tokens or q.dtype != torch.bfloat16
                or q.shape[-1] != 64 or q.device != self.device or torch.is_grad_enabled()):
            raise ValueError(f"mask STA requires eager contiguous BF16 Q/K/V [B,{tokens},H,64]")
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            if stream != self.setup_stream:
                stream.wait_stream(self.setup_stream)
                for t in (self.plan.schedule, self.plan.entries, self.row_order):
                    t.record_stream(stream)
            qt, kt, vt = (gather_tokens(x, self.row_order) for x in (q, k, v))
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
            sparse_attention_bshd(qt, kt, vt, scale, self.plan, out=out, out_rows=self.row_order)
        self._report["calls"] += 1
        return out


def current_mask_sta():
    return _active_window.get()


@contextmanager
def mask_sta_window(mask, grid, library_path=None, library_sha256: str = "",
                    geometry: StaGeometry = REFERENCE_GEOMETRY):
    operator = MaskSTA(mask, grid, library_path, library_sha256, geometry)
    token = _active_window.set(operator)
    try:
        yield operator
    finally:
        _active_window.reset(token)
        operator.close()
