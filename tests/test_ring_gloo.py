"""Ulysses x Ring (USP) protocol on CPU ranks (gloo): the reference's attention-
level SP hook (``nccl_sequence.py:235-332``) with ring degree 2, uneven shards,
both ring modes, and a failure that every collective survives.

The two kernel launches are replaced by CPU stand-ins on the same buffers
(full fp32 attention over the gathered segments for the reference mode, the
oracle's ring pieces for the streaming mode), so the exchanges, rotations,
piece owners and lengths are what is under test; the GPU tests cover the
kernels."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, ulysses, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from eraserdit_b200.ring import UspSelfAttention, ring_rotate
        from eraserdit_b200.sequence_sharding import floor_lengths
        from eraserdit_b200.topology import DiTGroups, DiTTopology
        from eraserdit_b200.ulysses import FLAG, SequenceParallelPeerError, peer_exchange
        from oracle import ring as oracle_ring
        from oracle.reference_path import sdpa_bshd

        class Layer:
            heads, softmax_scale, eps, precision = 4, 0.125, 1e-6, "bf16"

        class CpuUsp(UspSelfAttention):
            broken = False

            def _ring_attend(self, step, hop):
                if self.broken:
                    raise RuntimeError("injected attention failure")
                n, b, hl = self.degree, step.batch, self.local_heads
                split = lambda buf, lens: torch.cat(
                    [buf[u, :lens[u]].view(lens[u], b, hl, 64) for u in range(len(lens))]
                ).permute(1, 0, 2, 3)
                q = split(step.recv1, step.lengths)
                if hop is None:
                    lens = floor_lengths(step.length, self.sp_degree)
                    k = split(step.kbuf.flatten(0, 1), lens)
                    v = split(step.vbuf.flatten(0, 1), lens)
                    out = sdpa_bshd(q, k, v, self.layer.softmax_scale)
                else:
                    lens = self.piece_lengths(step.length, self.owner(hop))
                    k, v = split(step.kbuf[hop % 2], lens), split(step.vbuf[hop % 2], lens)
                    last = hop == self.ring_degree - 1
                    result = oracle_ring.piece(q, k, v, getattr(step, "cpu_state", None)
                                               if hop else None, final=last,
                                               scale=self.layer.softmax_scale)
                    if not last:
                        step.cpu_state = result
                        return
                    out = result
                row, t0 = b * hl * 64, 0
                for u in range(n):
                    rows = out[:, t0:t0 + step.lengths[u]].permute(1, 0, 2, 3).reshape(-1)
                    step.send2[0, u, FLAG:FLAG + rows.numel()] = rows
                    t0 += step.lengths[u]

        topo = DiTTopology(ulysses=ulysses, ring=world // ulysses)
        groups = DiTGroups(topo, warm_up=False)
        ug, uranks, uindex = groups.get("ulysses")
        rg, rranks, rindex = groups.get("ring")
        outcomes = []
        for mode in ("reference", "streaming"):
            usp = CpuUsp(Layer(), ulysses, uindex, peer_exchange(ug, uranks, uindex),
                         topo.ring, rindex, ring_rotate(rg, rranks, rindex), group_ranks=uranks,
                         mode=mode)
            for length in (16, 13, 29):
                g = torch.Generator().manual_seed(length)
                q, k, v = (torch.randn(2, length, 4, 64, generator=g) for _ in range(3))
                sl = usp.partition(length)
                got = usp.attention(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                    v[:, sl].contiguous())
                want = sdpa_bshd(q, k, v, 0.125)[:, sl]
                err = float((got - want).abs().max())
                outcomes.append("ok" if err <= 1e-5 else f"{mode} {length} err {err}")
        usp.broken = rank == 0
        try:
            sl = usp.partition(16)
            x = torch.zeros(2, sl.stop - sl.start, 4, 64)
            usp.attention(x, x, x)
            outcomes.append("no error")
        except SequenceParallelPeerError as e:
            outcomes.append(f"peer {e.peer_ranks}")
        except RuntimeError as e:
            outcomes.append(str(e))
        usp.broken = False
        usp.attention(x, x, x)  # the groups are still usable
        outcomes.append("ok")
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write("|".join(outcomes))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,ulysses", [(4, 2), (2, 1)])
def test_usp_hook_matches_full_attention_and_survives_failure(world, ulysses):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, ulysses, _free_port(), d), nprocs=world,
                           join=True, start_method="spawn")
        got = [open(os.path.join(d, f"r{r}")).read().split("|") for r in range(world)]
    for r in range(world):
        assert got[r][:6] == ["ok"] * 6, got[r]
        assert got[r][7] == "ok"
    # rank 0 fails its attention: it raises its own error, the other ranks of
    # its Ulysses group report it, the rest finish normally
    assert got[0][6] == "injected attention failure"
    for r in range(1, world):
        expect = "peer (0,)" if (ulysses > 1 and r < ulysses) else "no error"
        assert got[r][6] == expect, (r, got[r])
