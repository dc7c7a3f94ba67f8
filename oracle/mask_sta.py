"""CPU restatement of the reference's mask-STA sparse pattern, and masked attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``layers/attention/backends/mask_sta.py`` step by step with plain
Python loops (no vectorised shortcuts), its constants passed in:

- ``tile_layout``      :67-74  token order: tiles frame-major, Morton order of
                               the (row, column) tile coordinates, cells
                               (frame, row, column) inside a tile;
- ``background``       :75-86  window around each query block's mean tile
                               coordinate, clamped into the tile grid, plus the
                               block's own key blocks;
- ``protected``        :90-96  query blocks touching the max-pool-dilated mask;
- ``lut``              :99-105 per-row deltas of kept columns and counts.

``masked_attention`` is fp32 SDPA (scale, softmax over the kept keys only) on
the tile-ordered sequence, the semantics both the reference's kernel and the
B200 kernel implement at block granularity.
"""

from __future__ import annotations

import torch


def _morton(row: int, col: int) -> int:
    code = 0
    for i in range(16):
        code |= ((col >> i) & 1) << (2 * i)
        code |= ((row >> i) & 1) << (2 * i + 1)
    return code


def tile_layout(grid, tile):
    """(order, tiles): raster index of each token in tile order; tile coordinates."""
    tg = [g // t for g, t in zip(grid, tile)]
    spatial = sorted(((h, w) for h in range(tg[1]) for w in range(tg[2])),
                     key=lambda hw: _morton(hw[0], hw[1]))
    tiles = [(f, h, w) for f in range(tg[0]) for h, w in spatial]
    order = []
    for f, h, w in tiles:
        for df in range(tile[0]):
            for dh in range(tile[1]):
                for dw in range(tile[2]):
                    ff, hh, ww = f * tile[0] + df, h * tile[1] + dh, w * tile[2] + dw
                    order.append((ff * grid[1] + hh) * grid[2] + ww)
    return order, tiles


def background(grid, tile, window, query_block, kv_block):
    """Bool [query blocks][key blocks] as nested lists."""
    tg = [g // t for g, t in zip(grid, tile)]
    _, tiles = tile_layout(grid, tile)
    tile_tokens = tile[0] * tile[1] * tile[2]
    per_q = query_block // tile_tokens
    per_kv = kv_block // tile_tokens
    nq = len(tiles) // per_q
    nkv = len(tiles) // per_kv
    out = []
    for q in range(nq):
        mine = tiles[q * per_q:(q + 1) * per_q]
        centre = [sum(t[a] for t in mine) // per_q for a in range(3)]
        start = [min(max(centre[a] - window[a] // 2, 0), tg[a] - window[a]) for a in range(3)]
        row = []
        for kv in range(nkv):
            hit = False
            for t in tiles[kv * per_kv:(kv + 1) * per_kv]:
                if all(start[a] <= t[a] < start[a] + window[a] for a in range(3)):
                    hit = True
            first_token, last_token = kv * kv_block, (kv + 1) * kv_block
            if q * query_block <= first_token and last_token <= (q + 1) * query_block:
                hit = True
            row.append(hit)
        out.append(row)
    return out


def protected(mask, order, grid, kernel, query_block):
    """Bool per query block; ``mask`` is an [F][H][W] nested list or tensor."""
    m = torch.as_tensor(mask).reshape(grid)
    rf, rh, rw = (k // 2 for k in kernel)
    dilated = {}
    for f in range(grid[0]):
        for h in range(grid[1]):
            for w in range(grid[2]):
                hit = False
                for df in range(-rf, rf + 1):
                    for dh in range(-rh, rh + 1):
                        for dw in range(-rw, rw + 1):
                            ff, hh, ww = f + df, h + dh, w + dw
                            if (0 <= ff < grid[0] and 0 <= hh < grid[1] and 0 <= ww < grid[2]
                                    and float(m[ff, hh, ww]) > 0):
                                hit = True
                dilated[(f * grid[1] + h) * grid[2] + w] = hit
    nq = len(order) // query_block
    return [any(dilated[order[q * query_block + i]] for i in range(query_block)) for q in range(nq)]


def lut(rows):
    """Per-row (deltas, count) in the reference's padded form."""
    deltas, counts = [], []
    for row in rows:
        kept = [c for c, keep in enumerate(row) if keep]
        d, prev = [], 0
        for c in kept:
            d.append(c - prev)
            prev = c
        if len(kept) < len(row):
            d.append(0 - prev)
        d += [0] * (len(row) - len(d))
        deltas.append(d)
        counts.append(len(kept))
    return deltas, counts


def masked_attention(q, k, v, scale, token_mask):
    """fp32 softmax(Q K^T * scale) V over the keys ``token_mask`` [S, S] keeps.
    q, k, v: [B, S, H, D] (any float dtype); returns fp32 [B, S, H, D]."""
    qh, kh, vh = (t.float().transpose(1, 2) for t in (q, k, v))
    s = (qh @ kh.transpose(-1, -2)) * scale
    s = s.masked_fill(~token_mask, float("-inf"))
    return torch.softmax(s, dim=-1).matmul(vh).transpose(1, 2)
