"""Golden host values of the reference's ring axis, made by running its own code.

Run where the reference checkout is available (path as the first argument):

    python tests/golden/make_golden_ring.py /path/to/reference

It runs ``config/dit_parallel.py`` ``DiTTopology`` (groups and coordinates of
Ulysses x Ring layouts) and ``models/adapters/eraserdit/nccl_sequence.py``
``DistributedSequenceRank``: the sequence-parallel rank of ``__init__``,
``partition``, the Ulysses lengths of a ring index (``_length`` as
``_ulysses_input`` uses it) and ``_rotate``.  ``_rotate``'s point-to-point
calls are recorded instead of sent, giving the owner, the peers and the length
received at every rotation.  Output: ``ring_host.json`` beside this script.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from make_golden import install_diffusers_stub  # noqa: E402

TOPOLOGIES = {"u2_r2": dict(ulysses=2, ring=2), "r4": dict(ring=4), "u4_r2": dict(ulysses=4, ring=2),
              "u2_r2_cfg2": dict(ulysses=2, ring=2, cfg=2), "u1_r2": dict(ring=2)}
LENGTHS = (101, 32640, 13)


class _Groups:
    """The parts of ``DiTGroups`` that ``DistributedSequenceRank`` reads."""

    def __init__(self, topology, rank):
        self.topology = topology
        self.coordinates = topology.coordinates(rank)
        self._rank = rank

    def get(self, axis):
        for ranks in self.topology.groups(axis):
            if self._rank in ranks:
                return None, ranks, ranks.index(self._rank)
        raise KeyError(axis)


def main(reference: Path) -> None:
    install_diffusers_stub()
    sys.path.insert(0, str(reference))
    from config.dit_parallel import DiTTopology
    import models.adapters.eraserdit.nccl_sequence as nccl_sequence

    recorded = []
    fake_dist = SimpleNamespace(
        isend="isend", irecv="irecv",
        P2POp=lambda op, tensor, peer, group: (op, tuple(tensor.shape), peer),
        batch_isend_irecv=lambda ops: recorded.append(list(ops)) or [])
    real_dist, nccl_sequence.dist = nccl_sequence.dist, fake_dist
    out = {}
    try:
        for name, sizes in TOPOLOGIES.items():
            topo = DiTTopology(**sizes)
            entry = {axis: [list(g) for g in topo.groups(axis)]
                     for axis in ("ulysses", "ring", "sp", "cfg")}
            entry["coordinates"] = [list(topo.coordinates(r)) for r in range(topo.world_size)]
            entry["ranks"] = {}
            for rank in range(topo.world_size):
                seq = nccl_sequence.DistributedSequenceRank(_Groups(topo, rank))
                per_length = {}
                for length in LENGTHS:
                    sl = seq.partition(length)
                    rrank = seq.groups.coordinates[2]
                    ulysses_lengths = [seq._length(rrank * topo.ulysses + u)
                                       for u in range(topo.ulysses)]
                    _, ring_ranks, owner = seq.groups.get("ring")
                    key = value = torch.empty(1, sl.stop - sl.start, 1, 1)
                    hops = []
                    for _ in range(len(ring_ranks) - 1):
                        recorded.clear()
                        key, value, owner = seq._rotate(key, value, owner)
                        ops = recorded[0]
                        hops.append({"owner": owner, "length": key.shape[1],
                                     "send_to": ops[0][2], "recv_from": ops[1][2]})
                    per_length[str(length)] = {"slice": [sl.start, sl.stop],
                                               "ulysses_lengths": ulysses_lengths,
                                               "hops": hops}
                entry["ranks"][str(rank)] = {"sp_rank": seq.rank, "degree": seq.degree,
                                             "lengths": per_length}
            out[name] = entry
    finally:
        nccl_sequence.dist = real_dist
    (HERE / "ring_host.json").write_text(json.dumps(out, indent=1, sort_keys=True))
    print("wrote", HERE / "ring_host.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(Path(sys.argv[1]))
