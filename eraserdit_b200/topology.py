"""DiT rank topology and process groups (Ulysses x CFG).

Mirrors ``config/dit_parallel.py`` (``DiTTopology`` ``:36-88``: axis order
tp -> ulysses -> ring -> cfg -> replicas, coordinates, orthogonal groups) and
``distributed/dit_groups.py`` (``DiTGroups`` ``:10-46``: one communicator per
distinct rank set, a gloo control group, eager communicator warm-up).  With
CFG2 x SP4 on 8 GPUs, ranks {0..3} hold the cond branch and {4..7} the uncond
branch (``models/adapters/eraserdit/nccl_runner.py:92``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

AXES = {"tp": (0,), "ulysses": (1,), "ring": (2,), "sp": (1, 2), "cfg": (3,)}


@dataclass(frozen=True)
class DiTTopology:
    tp: int = 1
    ulysses: int = 1
    ring: int = 1
    cfg: int = 1
    replicas: int = 1

    def __post_init__(self) -> None:
        if any(type(n) is not int or n < 1 for n in self.sizes):
            raise ValueError("parallel degrees must be positive integers")
        if self.cfg not in (1, 2):
            raise ValueError("CFG degree must be 1 or 2")

    @property
    def sizes(self) -> tuple[int, ...]:
        return (self.tp, self.ulysses, self.ring, self.cfg, self.replicas)

    @property
    def world_size(self) -> int:
        return math.prod(self.sizes)

    @property
    def sp(self) -> int:
        return self.ulysses * self.ring

    def coordinates(self, rank: int) -> tuple[int, ...]:
        if not 0 <= rank < self.world_size:
            raise ValueError("rank outside topology")
        out = []
        for size in self.sizes:
            out.append(rank % size)
            rank //= size
        return tuple(out)

    def rank(self, coordinates) -> int:
        value, stride = 0, 1
        for index, size in zip(coordinates, self.sizes):
            if not 0 <= index < size:
                raise ValueError("coordinate outside topology")
            value += index * stride
            stride *= size
        return value

    def groups(self, axis: str) -> tuple[tuple[int, ...], ...]:
        axes = AXES[axis]
        found: dict[tuple[int, ...], list[int]] = {}
        for r in range(self.world_size):
            coords = self.coordinates(r)
            key = tuple(c for i, c in enumerate(coords) if i not in axes)
            found.setdefault(key, []).append(r)
        return tuple(tuple(v) for v in found.values())


class DiTGroups:
    """Process groups of this rank along every axis of a topology.

    ``get(axis)`` returns ``(group, ranks, index_in_group)``; ``group`` is None
    for a singleton axis.  Identical rank sets share one communicator.
    """

    def __init__(self, topology: DiTTopology, *, warm_up: bool = True) -> None:
        if dist.get_world_size() != topology.world_size:
            raise ValueError("process group world size must equal the topology's")
        self.topology = topology
        self.rank = dist.get_rank()
        self.coordinates = topology.coordinates(self.rank)
        self.groups: dict[str, tuple] = {}
        self.owned = []
        cache = {tuple(range(topology.world_size)): dist.group.WORLD}
        # Every rank creates every group in the same order (new_group is collective).
        for axis in ("tp", "ulysses", "ring", "sp", "cfg"):
            for ranks in topology.groups(axis):
                if len(ranks) == 1:
                    group = None
                else:
                    if ranks not in cache:
                        cache[ranks] = dist.new_group(list(ranks))
                    group = cache[ranks]
                if self.rank in ranks:
                    self.groups[axis] = (group, ranks, ranks.index(self.rank))
                    if group is not None and group is not dist.group.WORLD and group not in self.owned:
                        self.owned.append(group)
        if warm_up and dist.get_backend() == "nccl":
            # Communicator buffers are created before activations are allocated.
            scratch = torch.zeros(1, device=torch.device("cuda", torch.cuda.current_device()))
            dist.all_reduce(scratch)
            for group in self.owned:
                dist.all_reduce(scratch, group=group)
            torch.cuda.synchronize()

    def get(self, axis: str):
        return self.groups[axis]


def cfg_branches(topology: DiTTopology, cfg_rank: int) -> tuple[str, ...]:
    """The guidance branches this rank computes (``nccl_runner.py:92``): both on
    one CFG group, otherwise the positive branch on CFG rank 0 and the negative
    one on rank 1."""
    if topology.cfg == 1:
        return ("positive", "negative")
    return ("positive",) if cfg_rank == 0 else ("negative",)


def gather_cfg_pair(local: torch.Tensor, groups: DiTGroups, owner_only: bool = False):
    """Assemble the two CFG branches' outputs (``nccl_runner.py:127-137``).

    Returns ``(negative, positive)`` on every rank of the CFG group, or only on
    its first rank with ``owner_only`` (the others get ``None``).  With one CFG
    group there is nothing to gather: ``local`` must then be a mapping
    ``{"positive": ..., "negative": ...}``.
    """
    if groups.topology.cfg == 1:
        return local["negative"], local["positive"]
    group, ranks, _ = groups.get("cfg")
    local = local.contiguous()
    if owner_only:
        pair = [torch.empty_like(local) for _ in ranks] if groups.rank == ranks[0] else None
        dist.gather(local, gather_list=pair, dst=ranks[0], group=group)
        if pair is None:
            return None
    else:
        pair = [torch.empty_like(local) for _ in ranks]
        dist.all_gather(pair, local, group=group)
    return pair[1], pair[0]
