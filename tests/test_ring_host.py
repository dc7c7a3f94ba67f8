"""Ring-axis host logic against the reference's own values.

``tests/golden/ring_host.json`` comes from running the reference's
``DiTTopology`` (``config/dit_parallel.py:36-88``) and ``DistributedSequenceRank``
(``models/adapters/eraserdit/nccl_sequence.py:11-40,218-233``) with the
rotation's point-to-point calls recorded (``tests/golden/make_golden_ring.py``).
The Ulysses x Ring object must give the same sequence-parallel rank, token
slice, Ulysses lengths of its ring index, and for every rotation the same
owner, received length and peers."""
import json
from pathlib import Path
from types import SimpleNamespace

import pytest

from eraserdit_b200 import ring as ring_module
from eraserdit_b200.ring import UspSelfAttention, ring_rotate
from eraserdit_b200.topology import DiTTopology

GOLDEN = json.loads((Path(__file__).parent / "golden" / "ring_host.json").read_text())
SIZES = {"u2_r2": dict(ulysses=2, ring=2), "r4": dict(ring=4), "u4_r2": dict(ulysses=4, ring=2),
         "u2_r2_cfg2": dict(ulysses=2, ring=2, cfg=2), "u1_r2": dict(ring=2)}


class Layer:
    heads, softmax_scale, eps, precision = 8, 0.125, 1e-6, "bf16"


def _peers(ring_ranks, index, monkeypatch):
    """(send_to, recv_from) of one ring_rotate call, its P2P ops recorded."""
    seen = []
    fake = SimpleNamespace(isend="isend", irecv="irecv",
                           P2POp=lambda op, tensor, peer, group: (op, peer),
                           batch_isend_irecv=lambda ops: seen.extend(ops) or [])
    monkeypatch.setattr(ring_module, "dist", fake)
    ring_rotate(None, ring_ranks, index)([object()], [object()])
    sends = [p for op, p in seen if op == "isend"]
    recvs = [p for op, p in seen if op == "irecv"]
    return sends[0], recvs[0]


@pytest.mark.parametrize("name", sorted(SIZES))
def test_ring_axis_matches_reference(name, monkeypatch):
    ref = GOLDEN[name]
    topo = DiTTopology(**SIZES[name])
    for axis in ("ulysses", "ring", "sp", "cfg"):
        assert [list(g) for g in topo.groups(axis)] == ref[axis], axis
    assert [list(topo.coordinates(r)) for r in range(topo.world_size)] == ref["coordinates"]
    for rank_key, want in ref["ranks"].items():
        rank = int(rank_key)
        coords = topo.coordinates(rank)
        usp = UspSelfAttention(Layer(), topo.ulysses, coords[1], None, topo.ring, coords[2], None)
        assert (usp.sp_rank, usp.sp_degree) == (want["sp_rank"], want["degree"])
        ring_ranks = next(g for g in topo.groups("ring") if rank in g)
        send_to, recv_from = _peers(ring_ranks, ring_ranks.index(rank), monkeypatch)
        for length_key, v in want["lengths"].items():
            length = int(length_key)
            sl = usp.partition(length)
            assert [sl.start, sl.stop] == v["slice"]
            assert usp._lengths(length) == v["ulysses_lengths"]
            for hop, h in enumerate(v["hops"]):
                owner = usp.owner(hop + 1)
                assert owner == h["owner"]
                assert sum(usp.piece_lengths(length, owner)) == h["length"]
                assert (send_to, recv_from) == (h["send_to"], h["recv_from"])
