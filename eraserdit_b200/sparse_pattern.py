"""Mask-aware block-sparse self-attention pattern and the sparse kernel's work lists.

The pattern is the reference's mask-STA geometry
(``layers/attention/backends/mask_sta.py:18-24,66-105``), with its constants
made parameters:

- tokens are laid out tile by tile: the latent grid F x H x W is cut into
  tiles of ``tile`` cells; tiles are ordered frame-tile major, then by the
  Morton (Z-order) code of their (row, column) tile coordinates; the cells of
  a tile follow in (frame, row, column) order (``block_geometry`` ``:67-74``);
- queries are grouped in blocks of ``query_block`` consecutive tokens of that
  order, keys and values in blocks of ``kv_block``;
- every query block attends the key blocks that touch a background window of
  ``window`` tiles placed around the block's mean tile coordinate and clamped
  into the tile grid (``:75-83``), plus its own blocks (``:84-86``);
- query blocks holding any token of the mask dilated by ``protect`` cells
  (a centred max-pool, ``protected_blocks`` ``:90-96``) attend every key block.

``REFERENCE_GEOMETRY`` holds the reference's constants.  ``CONFIG4_GEOMETRY``
is the benchmark's sparse configuration: the 3 x 9 x 9-cell background window
rounded out to whole tiles of 4 x 2 x 4 cells (1 x 5 x 3 tiles), key blocks of
128 tokens, and the reference's 3 x 5 x 5 dilation (two cells in the plane).

The sparse attention kernel reads a per-CTA schedule built from a block mask
(:func:`build_schedule`): a pair of 128-row query tiles and the union of
their key-tile lists, each entry flagging which 64-token halves of the key
tile each query tile attends.  Rows of the pair with different lists cost the
union's products; full rows are paired with full rows and background rows
with their Morton neighbours to keep that union small.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

QUERY_TILE = 128  # query rows per kernel tile
KV_TILE = 128     # key rows per kernel tile
_TILE_MASK = (1 << 24) - 1


@dataclass(frozen=True)
class StaGeometry:
    grid: tuple[int, int, int] = (16, 34, 60)
    tile: tuple[int, int, int] = (4, 2, 4)
    window: tuple[int, int, int] = (4, 11, 7)   # background window, in tiles
    protect: tuple[int, int, int] = (3, 5, 5)   # dilation kernel, in cells
    query_block: int = 128
    kv_block: int = 64

    @property
    def tokens(self) -> int:
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def tile_grid(self) -> tuple[int, int, int]:
        return tuple(g // t for g, t in zip(self.grid, self.tile))

    @property
    def tile_tokens(self) -> int:
        return self.tile[0] * self.tile[1] * self.tile[2]

    def validate(self) -> None:
        if any(g % t for g, t in zip(self.grid, self.tile)):
            raise ValueError("the tile must divide the latent grid")
        if self.query_block % self.tile_tokens or self.kv_block % self.tile_tokens:
            raise ValueError("query and key blocks must hold whole tiles")
        if self.tokens % self.query_block or self.tokens % self.kv_block:
            raise ValueError("the blocks must divide the token count")
        if QUERY_TILE % self.query_block or KV_TILE % self.kv_block or self.kv_block % 64:
            raise ValueError("the kernel needs 128-token query blocks and 64 or 128-token key blocks")
        if any(k % 2 == 0 for k in self.protect):
            raise ValueError("the dilation kernel must have odd extents")


REFERENCE_GEOMETRY = StaGeometry()
CONFIG4_GEOMETRY = StaGeometry(window=(1, 5, 3), kv_block=128)


def _morton(row: torch.Tensor, col: torch.Tensor, bits: int) -> torch.Tensor:
    code = torch.zeros_like(row)
    for i in range(bits):
        code |= ((col >> i) & 1) << (2 * i)
        code |= ((row >> i) & 1) << (2 * i + 1)
    return code


def tile_order(geom: StaGeometry, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(order, tile_coords): ``order[i]`` is the raster index f*H*W + h*W + w of
    the token at position i of the tile layout; ``tile_coords`` [tiles, 3] the
    (frame, row, column) tile coordinates in layout order."""
    geom.validate()
    tf, th, tw = geom.tile_grid
    rows = torch.arange(th, device=device).repeat_interleave(tw)
    cols = torch.arange(tw, device=device).repeat(th)
    bits = max(1, math.ceil(math.log2(max(th, tw))))
    spatial = torch.argsort(_morton(rows, cols, bits), stable=True)
    rows, cols = rows[spatial], cols[spatial]
    frames = torch.arange(tf, device=device).repeat_interleave(th * tw)
    coords = torch.stack([frames, rows.repeat(tf), cols.repeat(tf)], dim=1)  # [tiles, 3]
    t0, t1, t2 = geom.tile
    df = torch.arange(t0, device=device).repeat_interleave(t1 * t2)
    dh = torch.arange(t1, device=device).repeat_interleave(t2).repeat(t0)
    dw = torch.arange(t2, device=device).repeat(t0 * t1)
    _, gh, gw = geom.grid
    f = coords[:, 0:1] * t0 + df
    h = coords[:, 1:2] * t1 + dh
    w = coords[:, 2:3] * t2 + dw
    order = ((f * gh + h) * gw + w).flatten()
    return order, coords


def background_blocks(geom: StaGeometry, coords: torch.Tensor | None = None) -> torch.Tensor:
    """Bool [query blocks, key blocks]: the background window plus each query
    block's own key blocks."""
    if coords is None:
        coords = tile_order(geom)[1]
    per_q = geom.query_block // geom.tile_tokens
    per_kv = geom.kv_block // geom.tile_tokens
    nq = geom.tokens // geom.query_block
    nkv = geom.tokens // geom.kv_block
    centre = torch.div(coords.view(nq, per_q, 3).sum(1), per_q, rounding_mode="floor")
    extent = torch.tensor(geom.window, device=coords.device)
    limit = torch.tensor(geom.tile_grid, device=coords.device) - extent
    start = torch.minimum((centre - extent // 2).clamp_min(0), limit)
    inside = ((coords[None] >= start[:, None]) & (coords[None] < (start + extent)[:, None])).all(-1)
    blocks = inside.view(nq, nkv, per_kv).any(-1)
    q = torch.arange(nq, device=coords.device)
    ratio = geom.query_block // geom.kv_block
    for r in range(max(ratio, 1)):
        blocks[q, q * ratio + r] = True
    return blocks


def protected_query_blocks(mask: torch.Tensor, order: torch.Tensor, geom: StaGeometry
                           ) -> torch.Tensor:
    """Bool [query blocks]: blocks holding a token of the dilated mask.
    ``mask`` is [F, H, W] (or [1, 1, F, H, W]); any value > 0 counts."""
    m = (mask.reshape(geom.grid) > 0).float()[None, None]
    pad = tuple(k // 2 for k in geom.protect)
    dilated = F.max_pool3d(m, geom.protect, stride=1, padding=pad) > 0
    return dilated.flatten()[order.to(dilated.device)].view(-1, geom.query_block).any(1).to(order.device)


def block_mask(mask: torch.Tensor | None, geom: StaGeometry, device=None) -> torch.Tensor:
    """The full pattern: background blocks, with protected query rows dense
    (computed on ``device``, the mask's by default)."""
    if device is None:
        device = mask.device if mask is not None else torch.device("cpu")
    order, coords = tile_order(geom, device)
    blocks = background_blocks(geom, coords)
    if mask is not None:
        blocks[protected_query_blocks(mask.to(device), order, geom)] = True
    return blocks


def block_table(blocks: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's LUT form of a block mask (``mask_sta.py:99-105``):
    per row, the kept column indices as successive differences (first one
    from 0), zero-padded after the last; and the per-row counts."""
    nrows, ncols = blocks.shape
    cols = torch.arange(ncols, device=blocks.device)
    kept = torch.where(blocks, cols, ncols).sort(dim=-1).values
    counts = blocks.sum(-1, dtype=torch.int32)
    kept = torch.where(cols < counts[:, None], kept, 0).to(torch.int32)
    prev = torch.cat([torch.zeros_like(kept[:, :1]), kept[:, :-1]], dim=1)
    return (kept - prev).contiguous(), counts.contiguous()


def ellipse_masks(grid: tuple[int, int, int] = (16, 34, 60), seed: int = 3,
                  semi_axes: tuple[int, int] = (6, 12)) -> torch.Tensor:
    """Synthetic inpainting masks: one ellipse per latent frame, semi-axes drawn
    once per video in ``semi_axes`` cells, centre drifting by at most one cell
    per frame (kept inside the frame).  Bool [F, H, W]."""
    frames, height, width = grid
    g = torch.Generator().manual_seed(seed)
    lo, hi = semi_axes
    a = float(torch.randint(lo, hi + 1, (1,), generator=g))  # rows
    b = float(torch.randint(lo, hi + 1, (1,), generator=g))  # columns
    cy = float(torch.randint(0, height, (1,), generator=g))
    cx = float(torch.randint(0, width, (1,), generator=g))
    hh = torch.arange(height, dtype=torch.float64).view(-1, 1)
    ww = torch.arange(width, dtype=torch.float64).view(1, -1)
    out = torch.zeros(grid, dtype=torch.bool)
    for f in range(frames):
        if f:
            step = torch.randint(-1, 2, (2,), generator=g)
            cy = min(max(cy + float(step[0]), 0.0), height - 1.0)
            cx = min(max(cx + float(step[1]), 0.0), width - 1.0)
        out[f] = ((hh - cy) / a) ** 2 + ((ww - cx) / b) ** 2 <= 1.0
    return out


def block_tiles(nblocks: int, seg_blocks: list[int] | None, tiles_per_seg: int
                ) -> torch.Tensor:
    """Kernel tile index of each 128-token block when the blocks are split into
    consecutive segments of ``seg_blocks`` blocks held in slots of
    ``tiles_per_seg`` tiles (one segment: the identity)."""
    if seg_blocks is None:
        return torch.arange(nblocks)
    if sum(seg_blocks) != nblocks:
        raise ValueError("segment blocks must add up to the block count")
    parts = [s * tiles_per_seg + torch.arange(n) for s, n in enumerate(seg_blocks)]
    return torch.cat(parts)


@dataclass
class SparseSchedule:
    """Host copy of the kernel's work lists (int32; moved to a device with ``to``)."""

    schedule: torch.Tensor   # [ctas, 4]: query tile A, query tile B (or -1), first entry, entries
    entries: torch.Tensor    # [total]: key tile | A halves << 24 | B halves << 26
    kept_pairs: int          # (query, key) token pairs of the pattern, per (batch, head)
    issued_pairs: int        # token pairs the kernel computes, per (batch, head)
    dense_pairs: int

    @property
    def ctas(self) -> int:
        return int(self.schedule.shape[0])

    @property
    def keep_fraction(self) -> float:
        return self.kept_pairs / self.dense_pairs

    def to(self, device) -> "SparseSchedule":
        return SparseSchedule(self.schedule.to(device), self.entries.to(device), self.kept_pairs,
                              self.issued_pairs, self.dense_pairs)


def _halves(blocks: torch.Tensor, kv_block: int) -> torch.Tensor:
    """[query tiles, key tiles] 2-bit masks of the 64-token halves kept."""
    nq, nkv = blocks.shape
    if kv_block == 128:
        return blocks.to(torch.int64) * 3
    if kv_block == 64:
        b = blocks.view(nq, nkv // 2, 2).to(torch.int64)
        return b[..., 0] | (b[..., 1] << 1)
    raise ValueError("key blocks of 64 or 128 tokens")


def build_schedule(blocks: torch.Tensor, kv_block: int, seg_blocks: list[int] | None = None,
                   tiles_per_seg: int | None = None) -> SparseSchedule:
    """Pair the 128-row query tiles and list each pair's key tiles.

    ``blocks`` is a bool [query blocks of 128, key blocks of ``kv_block``] mask
    over the tile-ordered sequence, on any device (the lists are built there,
    without host loops).  With ``seg_blocks`` the sequence is held as segments
    (one per source rank of the sequence-parallel exchange) of that many
    128-token blocks each, in slots of ``tiles_per_seg`` tiles; tile indices
    are then those of the segmented layout.

    Full rows are paired with full rows, the others with their neighbours in
    tile order; rows with the longest lists come first (the hardware
    dispatches CTAs in grid order).
    """
    device = blocks.device
    halves = _halves(blocks, kv_block)  # [nq, nt]
    nq, nt = halves.shape
    if nq != nt:
        raise ValueError("self-attention: as many key tiles as query tiles")
    tps = tiles_per_seg if tiles_per_seg is not None else nq
    tile_of = block_tiles(nq, seg_blocks, tps).to(device)
    counts = (halves != 0).sum(1)
    if bool((counts == 0).any()):
        raise ValueError("every query block needs at least one key block")
    full = counts == nt
    idx = torch.arange(nq, device=device)
    order = torch.cat([idx[full], idx[~full]])
    npairs = (nq + 1) // 2
    slots = torch.full((2 * npairs,), -1, dtype=torch.int64, device=device)
    slots[:nq] = order
    pa, pb = slots[0::2], slots[1::2]  # pb is -1 for a lone last tile
    ha = halves[pa]
    hb = torch.where((pb >= 0)[:, None], halves[pb.clamp_min(0)], torch.zeros_like(ha))
    union = (ha | hb) != 0
    n = union.sum(1)
    rank = torch.argsort(-n, stable=True)
    union, ha, hb, pa, pb, n = union[rank], ha[rank], hb[rank], pa[rank], pb[rank], n[rank]
    row, col = torch.nonzero(union, as_tuple=True)  # grouped by row, columns ascending
    entries = tile_of[col] | (ha[row, col] << 24) | (hb[row, col] << 26)
    first = torch.cumsum(n, 0) - n
    qb = torch.where(pb >= 0, tile_of[pb.clamp_min(0)], torch.full_like(pb, -1))
    sched = torch.stack([tile_of[pa], qb, first, n], dim=1)
    # every CTA computes both of its tiles' products (a lone tile's partner
    # repeats it), so the issued work counts two tiles per list entry
    issued = int(n.sum()) * KV_TILE * QUERY_TILE * 2
    kept = int(((halves & 1) + ((halves >> 1) & 1)).sum()) * 64 * QUERY_TILE
    return SparseSchedule(sched.to(torch.int32), entries.to(torch.int32), kept, issued,
                          nq * QUERY_TILE * nt * KV_TILE)


def attention_mask(blocks: torch.Tensor, kv_block: int, query_block: int = 128) -> torch.Tensor:
    """Token-level bool [S, S] mask of a block pattern over the tile-ordered sequence."""
    return blocks.repeat_interleave(query_block, 0).repeat_interleave(kv_block, 1)
