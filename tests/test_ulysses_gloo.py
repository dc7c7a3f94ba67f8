"""Ulysses exchange protocol on 2 CPU ranks (gloo): chunk routing, uneven shards,
head chunks, and peer-failure propagation with every collective always entered
(the reference's tests/test_ulysses_overlap.py:47-60 injects a failing impl the
same way).

The CUDA phases are replaced by CPU stand-ins that move the same buffers, so
only the host protocol is under test here; the GPU tests cover the kernels."""
import os
import socket
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from eraserdit_b200.sequence_sharding import floor_lengths


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from eraserdit_b200.ulysses import (FLAG, SequenceParallelPeerError, UlyssesSelfAttention,
                                            peer_exchange)

        class Layer:
            heads, softmax_scale, eps = 4, 0.125, 1e-6

        class CpuUlysses(UlyssesSelfAttention):
            """Stand-in phases: send block (d, chunk c) carries (c, rank, d, token) tags."""
            broken = False

            def pre(self, x_local, rope, length):
                lengths = floor_lengths(length, self.degree)
                lme = lengths[self.rank]
                n, b, chunks = self.degree, x_local.shape[0], self.head_chunks
                send1 = torch.empty(n, chunks, lme, 1)
                for d in range(n):
                    for c in range(chunks):
                        send1[d, c, :, 0] = (10000 * c + 1000 * self.rank + 100 * d
                                             + torch.arange(lme))
                recv1 = torch.zeros(chunks, n, max(lengths), 1)
                send2 = torch.zeros(chunks, n, FLAG + max(lengths))
                recv2 = torch.empty(chunks, n, FLAG + lme)
                from eraserdit_b200.ulysses import _Step
                return _Step(b, length, lengths, 0, send1, recv1, send2, recv2, chunks=chunks)

            def send_recv_2(self, step, chunk=0):
                outputs = [step.recv2[chunk, s] for s in range(self.degree)]
                inputs = [step.send2[chunk, d, :FLAG + step.lengths[d]]
                          for d in range(self.degree)]
                return outputs, inputs

            def _attend(self, step, chunk=0):
                if self.broken and chunk == step.chunks - 1:
                    raise RuntimeError("injected attention failure")
                for s in range(self.degree):
                    got = step.recv1[chunk, s, :step.lengths[s], 0]
                    expect = (10000 * chunk + 1000 * s + 100 * self.rank
                              + torch.arange(step.lengths[s]))
                    assert torch.equal(got, expect.float())
                    step.send2[chunk, s, FLAG:FLAG + step.lengths[s]] = got + 0.5

            def post(self, step):
                flags = step.recv2[:, :, 0].amax(dim=0)
                if step.failed:
                    raise RuntimeError("local sequence-parallel attention failed")
                bad = torch.nonzero(flags != 0).flatten().tolist()
                if bad:
                    raise SequenceParallelPeerError(tuple(bad))
                return step.recv2[:, :, FLAG:].clone()

        outcomes = []
        for chunks in (1, 2):
            sp = CpuUlysses(Layer(), world, rank, peer_exchange(None, tuple(range(world)), rank),
                            head_chunks=chunks)
            for length in (8, 7, 11):
                out = sp(torch.zeros(2, floor_lengths(length, world)[rank], 1), None, length)
                lme = floor_lengths(length, world)[rank]
                for c in range(chunks):
                    for s in range(world):
                        expect = 10000 * c + 1000 * rank + 100 * s + torch.arange(lme) + 0.5
                        assert torch.equal(out[c, s], expect.float())
            outcomes.append("ok")
        sp.broken = rank == 1
        try:
            sp(torch.zeros(2, 4, 1), None, 8)
            outcomes.append("no error")
        except SequenceParallelPeerError as e:
            outcomes.append(f"peer {e.peer_ranks}")
        except RuntimeError as e:
            outcomes.append(str(e))
        sp.broken = False
        sp(torch.zeros(2, 4, 1), None, 8)  # the group is still usable
        outcomes.append("ok")
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write("|".join(outcomes))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_and_peer_failure():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(2, _free_port(), d), nprocs=2, join=True,
                           start_method="spawn")
        r0 = open(os.path.join(d, "r0")).read().split("|")
        r1 = open(os.path.join(d, "r1")).read().split("|")
    assert r0 == ["ok", "ok", "peer (1,)", "ok"]
    assert r1 == ["ok", "ok", "injected attention failure", "ok"]



def _cfg_rank(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from eraserdit_b200.topology import DiTGroups, DiTTopology, cfg_branches, gather_cfg_pair
        groups = DiTGroups(DiTTopology(cfg=2), warm_up=False)
        branch = cfg_branches(groups.topology, groups.coordinates[3])[0]
        local = torch.full((2, 3), 1.0 if branch == "positive" else -1.0) * (rank + 1)
        negative, positive = gather_cfg_pair(local, groups)
        owner = gather_cfg_pair(local, groups, owner_only=True)
        ok = (float(negative[0, 0]) == -2.0 and float(positive[0, 0]) == 1.0
              and ((owner is None) == (rank != 0)))
        with open(os.path.join(result_dir, f"c{rank}"), "w") as f:
            f.write(f"{branch}|{ok}")
    finally:
        dist.destroy_process_group()


def test_cfg_pair_gather_two_ranks():
    """CFG2: rank 0 computes the positive branch, rank 1 the negative one; the
    pair gather returns (negative, positive) (nccl_runner.py:92,127-137)."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cfg_rank, args=(2, _free_port(), d), nprocs=2, join=True,
                           start_method="spawn")
        got = [open(os.path.join(d, f"c{r}")).read() for r in range(2)]
    assert got == ["positive|True", "negative|True"]
