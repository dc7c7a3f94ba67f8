"""Sequence shard plans for Ulysses sequence parallelism.

Mirrors ``parallel/sequence_sharding.py`` (``SequenceShardPlan`` ``:12-71``,
``plan_sequence_shards`` ``:74-119``: equal, right-padded shards) and the floor
partition the NCCL Ulysses path uses (``models/adapters/eraserdit/mesh.py:163-169``,
``models/adapters/eraserdit/nccl_sequence.py:37-38``): rank r of N owns tokens
[S * r // N, S * (r + 1) // N).
"""

from __future__ import annotations

from dataclasses import dataclass


def floor_bounds(length: int, degree: int, rank: int) -> tuple[int, int]:
    """Token range [start, end) of ``rank`` under the floor partition."""
    if degree < 1 or not 0 <= rank < degree:
        raise ValueError("rank must be inside the sequence-parallel degree")
    return length * rank // degree, length * (rank + 1) // degree


def floor_lengths(length: int, degree: int) -> list[int]:
    return [length * (r + 1) // degree - length * r // degree for r in range(degree)]


def block_bounds(length: int, degree: int, rank: int, block: int = 128) -> tuple[int, int]:
    """Token range of ``rank`` when whole ``block``-token blocks are floor
    partitioned (the block-sparse attention needs every source segment to hold
    whole query / key tiles)."""
    if length % block:
        raise ValueError(f"block partition needs a multiple of {block} tokens")
    b0, b1 = floor_bounds(length // block, degree, rank)
    return b0 * block, b1 * block


def block_lengths(length: int, degree: int, block: int = 128) -> list[int]:
    return [n * block for n in floor_lengths(length // block, degree)]


@dataclass(frozen=True)
class SequenceShardPlan:
    """One rank's equal-size slice of a right-padded sequence."""

    global_length: int
    padded_length: int
    local_start: int
    local_end: int
    valid_local_length: int
    pad_right: int
    owner_rank: int
    sp_degree: int
    rank: int

    def __post_init__(self) -> None:
        for name in ("global_length", "padded_length", "local_start", "local_end",
                     "valid_local_length", "pad_right", "owner_rank", "sp_degree", "rank"):
            if type(getattr(self, name)) is not int:
                raise TypeError(f"{name} must be an int")
        if self.global_length < 0:
            raise ValueError("global_length must be non-negative")
        if self.sp_degree < 1:
            raise ValueError("sp_degree must be positive")
        if not 0 <= self.rank < self.sp_degree:
            raise ValueError("rank must be inside sp_degree")
        if not 0 <= self.owner_rank < self.sp_degree:
            raise ValueError("owner_rank must be inside sp_degree")
        if self.padded_length < self.global_length:
            raise ValueError("padded_length must cover global_length")
        if self.padded_length % self.sp_degree != 0:
            raise ValueError("padded_length must be divisible by sp_degree")
        if not 0 <= self.local_start <= self.local_end <= self.padded_length:
            raise ValueError("local range must fit padded_length")
        if self.local_start != self.rank * self.local_length:
            raise ValueError("local_start must match rank order")
        if self.local_length != self.padded_length // self.sp_degree:
            raise ValueError("all ranks must use an equal local_length")
        if not 0 <= self.valid_local_length <= self.local_length:
            raise ValueError("valid_local_length must fit local_length")
        if self.pad_right != self.local_length - self.valid_local_length:
            raise ValueError("pad_right must cover the invalid local suffix")
        if self.valid_local_length != max(0, min(self.local_length,
                                                 self.global_length - self.local_start)):
            raise ValueError("valid_local_length must match the global range")

    @property
    def local_length(self) -> int:
        return self.local_end - self.local_start


def plan_sequence_shards(global_length: int, sp_degree: int,
                         owner_rank: int) -> tuple[SequenceShardPlan, ...]:
    """Immutable, rank-ordered metadata for equal (right-padded) sequence shards."""
    for name, value in (("global_length", global_length), ("sp_degree", sp_degree),
                        ("owner_rank", owner_rank)):
        if type(value) is not int:
            raise TypeError(f"{name} must be an int")
    if global_length < 0:
        raise ValueError("global_length must be non-negative")
    if sp_degree < 1:
        raise ValueError("sp_degree must be positive")
    if not 0 <= owner_rank < sp_degree:
        raise ValueError("owner_rank must be inside sp_degree")
    local = (global_length + sp_degree - 1) // sp_degree
    padded = local * sp_degree
    plans = []
    for rank in range(sp_degree):
        start = rank * local
        valid = max(0, min(local, global_length - start))
        plans.append(SequenceShardPlan(global_length, padded, start, start + local, valid,
                                       local - valid, owner_rank, sp_degree, rank))
    return tuple(plans)


# Attention backends that may run under sequence parallelism (the reference's
# set, sequence_parallel.py:88-99, plus the two B200 backends).
SP_BACKENDS = frozenset({"torch_sdpa", "flash_attn", "sage_attn", "sage_fp8", "b200_native",
                         "b200_fp8"})


@dataclass(frozen=True)
class SequenceParallelMetadata:
    """One SP rank's shard and backend contract (``layers/attention/sequence_parallel.py:57-154``).

    The fields and checks are those of a :class:`SequenceShardPlan` plus the
    attention backend, which must be one that runs under sequence parallelism.
    """

    global_length: int
    padded_length: int
    local_start: int
    local_end: int
    valid_local_length: int
    pad_right: int
    owner_rank: int
    sp_degree: int
    rank: int
    backend: object  # an AttentionBackendEnum member

    def __post_init__(self) -> None:
        # The shard fields obey exactly the plan's contract.
        SequenceShardPlan(self.global_length, self.padded_length, self.local_start,
                          self.local_end, self.valid_local_length, self.pad_right,
                          self.owner_rank, self.sp_degree, self.rank)
        from .attention import AttentionBackendEnum
        if not isinstance(self.backend, AttentionBackendEnum):
            raise TypeError("backend must be an AttentionBackendEnum")
        if self.backend.value not in SP_BACKENDS:
            raise ValueError("backend must be one of " + ", ".join(sorted(SP_BACKENDS))
                             + " for sequence parallel")

    @property
    def local_length(self) -> int:
        return self.local_end - self.local_start

    @classmethod
    def from_shard_plan(cls, plan: SequenceShardPlan, *, backend) -> "SequenceParallelMetadata":
        if not isinstance(plan, SequenceShardPlan):
            raise TypeError("plan must be a SequenceShardPlan")
        return cls(plan.global_length, plan.padded_length, plan.local_start, plan.local_end,
                   plan.valid_local_length, plan.pad_right, plan.owner_rank, plan.sp_degree,
                   plan.rank, backend)
