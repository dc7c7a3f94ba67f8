"""Mask-aware sparse pattern: the product geometry and the oracle restatement
against the reference's own outputs (golden fixtures), and the kernel work
lists against the block mask they encode.  CPU only."""
from pathlib import Path

import numpy as np
import pytest
import torch

from eraserdit_b200 import sparse_pattern as sp
from oracle import mask_sta as oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "mask_sta_golden.npz"
MASKS = ("ellipse", "one_cell", "empty")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _bits(g, name, shape):
    n = int(np.prod(shape))
    return torch.from_numpy(np.unpackbits(g[name])[:n].astype(bool).reshape(shape))


def _golden_mask(g, name):
    return _bits(g, f"{name}_mask", sp.REFERENCE_GEOMETRY.grid)


def test_product_geometry_matches_reference(golden):
    geom = sp.REFERENCE_GEOMETRY
    order, coords = sp.tile_order(geom)
    assert torch.equal(order.to(torch.int32), torch.from_numpy(golden["permutation"]))
    shape = tuple(golden["background_shape"])
    bg = _bits(golden, "background", shape)
    assert torch.equal(sp.background_blocks(geom, coords), bg)
    assert int(bg.sum()) == 46096  # the reference's own regression value
    for name in MASKS:
        mask = _golden_mask(golden, name)
        prot = sp.protected_query_blocks(mask, order, geom)
        assert torch.equal(prot, torch.from_numpy(golden[f"{name}_protected"]))
        lut, counts = sp.block_table(sp.block_mask(mask, geom))
        assert torch.equal(lut, torch.from_numpy(golden[f"{name}_lut"].astype(np.int32)))
        assert torch.equal(counts, torch.from_numpy(golden[f"{name}_counts"]))


def test_oracle_restatement_matches_reference(golden):
    geom = sp.REFERENCE_GEOMETRY
    order, _ = oracle.tile_layout(geom.grid, geom.tile)
    assert order == golden["permutation"].tolist()
    bg = oracle.background(geom.grid, geom.tile, geom.window, geom.query_block, geom.kv_block)
    want = _bits(golden, "background", tuple(golden["background_shape"]))
    assert torch.equal(torch.tensor(bg), want)
    mask = _golden_mask(golden, "ellipse")
    prot = oracle.protected(mask.tolist(), order, geom.grid, geom.protect, geom.query_block)
    assert prot == golden["ellipse_protected"].tolist()
    rows = [[b or p for b in row] for row, p in zip(bg, prot)]
    deltas, counts = oracle.lut(rows)
    assert deltas == golden["ellipse_lut"].astype(np.int32).tolist()
    assert counts == golden["ellipse_counts"].tolist()


def test_synthetic_mask_statistics():
    mask = sp.ellipse_masks(sp.CONFIG4_GEOMETRY.grid, seed=3)
    dil = torch.nn.functional.max_pool3d(mask.float()[None, None], (1, 5, 5), stride=1,
                                         padding=(0, 2, 2)) > 0
    frac = float(dil.float().mean())
    assert 0.10 <= frac <= 0.30, frac  # the configuration's ~15-25 % of tokens
    # centre drifts by at most one cell per frame
    cy = [float(torch.nonzero(mask[f])[:, 0].float().mean()) for f in range(mask.shape[0])]
    assert max(abs(a - b) for a, b in zip(cy, cy[1:])) <= 1.5


def _decode(s: sp.SparseSchedule, nq: int, tile_of: torch.Tensor) -> torch.Tensor:
    """Per query tile, the 2-bit halves it attends per key tile, from the lists."""
    block_of = {int(t): i for i, t in enumerate(tile_of)}
    got = torch.zeros(nq, nq, dtype=torch.int64)
    seen = torch.zeros(nq, dtype=torch.int64)
    for qa, qb, first, n in s.schedule.tolist():
        for e in s.entries[first:first + n].tolist():
            kv = block_of[e & 0xFFFFFF]
            for q, shift in ((qa, 24), (qb, 26)):
                if q >= 0:
                    got[block_of[q], kv] |= (e >> shift) & 3
        for q in (qa, qb):
            if q >= 0:
                seen[block_of[q]] += 1
    assert bool((seen == 1).all()), "each query tile is scheduled exactly once"
    return got


@pytest.mark.parametrize("geom", [sp.REFERENCE_GEOMETRY, sp.CONFIG4_GEOMETRY])
@pytest.mark.parametrize("segments", [None, [32] * 7 + [31]])
def test_schedule_encodes_block_mask(geom, segments):
    blocks = sp.block_mask(sp.ellipse_masks(geom.grid, seed=3), geom)
    tps = 32 if segments else None
    s = sp.build_schedule(blocks, geom.kv_block, seg_blocks=segments, tiles_per_seg=tps)
    nq = blocks.shape[0]
    tile_of = sp.block_tiles(nq, segments, tps or nq)
    got = _decode(s, nq, tile_of)
    assert torch.equal(got, sp._halves(blocks, geom.kv_block))
    counts = s.schedule[:, 3]
    assert bool((counts[:-1] >= counts[1:]).all())  # longest first
    assert s.kept_pairs == int(sp.attention_mask(blocks, geom.kv_block).sum())
    assert s.kept_pairs <= s.issued_pairs


def test_config4_pattern_is_sparse():
    geom = sp.CONFIG4_GEOMETRY
    blocks = sp.block_mask(sp.ellipse_masks(geom.grid, seed=3), geom)
    s = sp.build_schedule(blocks, geom.kv_block)
    assert 0.15 < s.keep_fraction < 0.7, s.keep_fraction
    assert s.issued_pairs < 1.15 * s.kept_pairs + 2 * 128 * 128 * 255
