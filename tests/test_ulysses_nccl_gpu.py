"""Ulysses SP over real NCCL on every visible GPU (skipped with fewer than 2):
each rank's output equals the single-GPU layer's rows for its tokens, dense,
head-chunked, over peer memory (CUDA IPC) and block-sparse."""
import os
import socket
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=device)
    try:
        from eraserdit_b200.layer import EraserDiTSelfAttention
        from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
        from eraserdit_b200.topology import DiTGroups, DiTTopology
        from eraserdit_b200.ulysses import UlyssesSelfAttention, peer_exchange
        from eraserdit_b200.synthetic import make_params
        groups = DiTGroups(DiTTopology(ulysses=world))
        group, ranks, index = groups.get("ulysses")
        p = make_params(3, 1e-6, random_norm_weight=True, device=device)
        layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device=device)
        for frames, height, width in ((2, 8, 12), (1, 7, 11)):
            rope = LTXVideoRotaryPosEmbed()(frames, height, width, device=device)
            g = torch.Generator(device=device).manual_seed(frames)
            x = torch.randn(2, frames * height * width, 2048, generator=g, device=device).bfloat16()
            want = layer(x, rope)
            sp = UlyssesSelfAttention(layer, world, index, peer_exchange(group, ranks, index), ranks)
            sl = sp.partition(x.shape[1])
            got = sp(x[:, sl].contiguous(), rope, x.shape[1])
            err = float((got.float() - want[:, sl].float()).abs().max())
            cos = float(torch.nn.functional.cosine_similarity(
                got.float().flatten(), want[:, sl].float().flatten(), dim=0))
            assert err <= 1e-2 and cos >= 0.99999, (err, cos)
            # head chunks: exchanges on a second stream overlap the chunks' attention
            chunked = UlyssesSelfAttention(layer, world, index, peer_exchange(group, ranks, index),
                                           ranks, head_chunks=2)
            again = chunked(x[:, sl].contiguous(), rope, x.shape[1])
            assert torch.equal(again, got), "head chunks changed the result"
        # peer-memory exchange (CUDA IPC mappings, stores over NVLink)
        rope = LTXVideoRotaryPosEmbed()(2, 8, 12, device=device)
        g = torch.Generator(device=device).manual_seed(2)
        x = torch.randn(2, 192, 2048, generator=g, device=device).bfloat16()
        want = layer(x, rope)
        sp = UlyssesSelfAttention(layer, world, index, peer_exchange(group, ranks, index), ranks,
                                  transport="peer", group=group)
        sl = sp.partition(x.shape[1])
        for _ in range(3):  # several epochs through the same buffers
            got = sp(x[:, sl].contiguous(), rope, x.shape[1])
        err = float((got.float() - want[:, sl].float()).abs().max())
        cos = float(torch.nn.functional.cosine_similarity(
            got.float().flatten(), want[:, sl].float().flatten(), dim=0))
        assert err <= 1e-2 and cos >= 0.99999, ("peer", err, cos)
        torch.cuda.synchronize()
        dist.barrier()
        sp.close()  # raises if any call of this object saw a peer error
        # block-sparse attention over the exchange (whole 128-token blocks per rank)
        from eraserdit_b200 import sparse_pattern as sp_pattern
        from eraserdit_b200.mask_sta import SparsePlan
        geom = sp_pattern.StaGeometry(grid=(8, 16, 32), window=(1, 3, 2), kv_block=128)
        plan = SparsePlan.from_mask(
            sp_pattern.ellipse_masks(geom.grid, seed=4, semi_axes=(2, 4)), geom, device)
        rope = LTXVideoRotaryPosEmbed()(*geom.grid, device=device)
        g = torch.Generator(device=device).manual_seed(5)
        x = torch.randn(2, geom.tokens, 2048, generator=g, device=device).bfloat16()
        want = layer(x, rope, sparse=plan)
        sp = UlyssesSelfAttention(layer, world, index, peer_exchange(group, ranks, index), ranks,
                                  sparse=plan)
        sl = sp.partition(x.shape[1])
        got = sp(x[:, sl].contiguous(), rope, x.shape[1])
        err = float((got.float() - want[:, sl].float()).abs().max())
        cos = float(torch.nn.functional.cosine_similarity(
            got.float().flatten(), want[:, sl].float().flatten(), dim=0))
        assert err <= 1e-2 and cos >= 0.99999, ("sparse", err, cos)
        torch.cuda.synchronize()
        open(os.path.join(out_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


def test_nccl_ulysses_matches_single_gpu():
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least two GPUs")
    world = 8 if world >= 8 else (4 if world >= 4 else 2)
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        assert sorted(os.listdir(d)) == sorted(f"ok{r}" for r in range(world))
