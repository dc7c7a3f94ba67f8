"""Shard plans and rank topology reproduce the reference's (golden JSON)."""
import pytest

from eraserdit_b200.sequence_sharding import floor_lengths, plan_sequence_shards
from eraserdit_b200.topology import DiTTopology


def test_shard_plans_match_reference(golden_host):
    for key, rows in golden_host["plans"].items():
        length, degree = map(int, key.split("_"))
        got = [[p.global_length, p.padded_length, p.local_start, p.local_end,
                p.valid_local_length, p.pad_right] for p in plan_sequence_shards(length, degree, 0)]
        assert got == rows, key


def test_floor_lengths_match_reference(golden_host):
    for key, lengths in golden_host["floor_lengths"].items():
        length, degree = map(int, key.split("_"))
        assert floor_lengths(length, degree) == lengths


def test_topologies_match_reference(golden_host):
    topos = {"sp8": DiTTopology(ulysses=8), "cfg2_sp4": DiTTopology(ulysses=4, cfg=2),
             "cfg2_sp2": DiTTopology(ulysses=2, cfg=2)}
    for name, topo in topos.items():
        ref = golden_host["topology"][name]
        for axis in ("ulysses", "sp", "cfg"):
            assert [list(g) for g in topo.groups(axis)] == ref[axis], (name, axis)
        assert [list(topo.coordinates(r)) for r in range(topo.world_size)] == ref["coordinates"]


def test_plan_validation_errors():
    with pytest.raises(ValueError):
        plan_sequence_shards(10, 0, 0)
    with pytest.raises(ValueError):
        plan_sequence_shards(10, 2, 2)
    with pytest.raises(TypeError):
        plan_sequence_shards(10.0, 2, 0)
    with pytest.raises(ValueError):
        DiTTopology(cfg=3)


def test_block_partition():
    from eraserdit_b200.sequence_sharding import block_bounds, block_lengths
    assert block_lengths(32640, 8) == [3968] + [4096] * 7
    bounds = [block_bounds(32640, 8, r) for r in range(8)]
    assert bounds[0][0] == 0 and bounds[-1][1] == 32640
    assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
    assert all((e - s) % 128 == 0 for s, e in bounds)
    with pytest.raises(ValueError):
        block_bounds(1000, 2, 0)


def test_sequence_parallel_metadata():
    from eraserdit_b200.attention import AttentionBackendEnum
    from eraserdit_b200.sequence_sharding import SequenceParallelMetadata
    plans = plan_sequence_shards(10, 4, 0)
    meta = SequenceParallelMetadata.from_shard_plan(plans[3], backend=AttentionBackendEnum.B200_NATIVE)
    assert (meta.local_start, meta.local_end, meta.valid_local_length, meta.pad_right) == (9, 12, 1, 2)
    assert meta.local_length == 3
    with pytest.raises(TypeError):
        SequenceParallelMetadata.from_shard_plan(plans[0], backend="b200_native")
    with pytest.raises(ValueError):  # the plan's own contract
        SequenceParallelMetadata(10, 12, 3, 6, 2, 1, 0, 4, 1, AttentionBackendEnum.TORCH_SDPA)
    with pytest.raises(TypeError):
        SequenceParallelMetadata.from_shard_plan(object(), backend=AttentionBackendEnum.SAGE_FP8)


def test_cfg_branches():
    from eraserdit_b200.topology import cfg_branches
    assert cfg_branches(DiTTopology(ulysses=8), 0) == ("positive", "negative")
    assert cfg_branches(DiTTopology(ulysses=4, cfg=2), 0) == ("positive",)
    assert cfg_branches(DiTTopology(ulysses=4, cfg=2), 1) == ("negative",)
