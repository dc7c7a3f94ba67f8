"""Multi-GPU leg of ``bench.py``: Ulysses SP (optionally CFG x SP, or
Ulysses x Ring with ``--ring``) with peer-memory or NCCL exchanges.

Launched by torchrun with one process per GPU.  Every rank builds the same
seeded layer and input, keeps its floor-partitioned tokens (CFG: its branch's
batch entry) and runs the sequence-parallel layer; per-rank times come from
CUDA events and the reported time is the maximum over ranks (an all-reduce
MAX)."""

from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def _alternate(objects, counter, xd, rope, length):
    """Call the Ulysses objects in turn (step i uses objects[i % 2])."""
    sp = objects[counter[0] % len(objects)]
    counter[0] += 1
    return sp(xd, rope, length)


def run_sequence_parallel(args) -> None:
    import bench as B
    from eraserdit_b200 import _native
    from eraserdit_b200.topology import DiTGroups, DiTTopology
    from eraserdit_b200.ring import UspSelfAttention, ring_rotate
    from eraserdit_b200.ulysses import UlyssesSelfAttention, peer_exchange

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    try:
        cfg, ring = args.cfg, getattr(args, "ring", 1)
        if world % (cfg * ring) or B.BATCH % cfg:
            raise SystemExit("CFG x ring degree must divide the GPU count, CFG the batch")
        topo = DiTTopology(ulysses=world // (cfg * ring), ring=ring, cfg=cfg)
        groups = DiTGroups(topo)
        group, ranks, index = (groups.get("ulysses") if topo.ulysses > 1
                               else (None, (rank,), 0))
        cfg_index = topo.coordinates(rank)[3]
        layer, rope = B.build_problem(device, "fp8" if args.fp8 else "bf16")
        plan, kept, issued = B.build_sparse_plan(device) if args.sparse else (None, 1.0, 1.0)
        g = torch.Generator(device=device).manual_seed(1)
        x_full = torch.randn(B.BATCH, B.SEQ, B.HIDDEN, generator=g, device=device).bfloat16()
        per_branch = B.BATCH // cfg
        x_branch = x_full[cfg_index * per_branch:(cfg_index + 1) * per_branch]
        transport = args.transport

        def make_layer():
            if ring > 1:
                rgroup, rranks, rindex = groups.get("ring")
                return UspSelfAttention(layer, len(ranks), index,
                                        peer_exchange(group, ranks, index), ring, rindex,
                                        ring_rotate(rgroup, rranks, rindex), group_ranks=ranks,
                                        mode=args.ring_mode, transport=transport, group=group)
            return UlyssesSelfAttention(layer, len(ranks), index,
                                        peer_exchange(group, ranks, index), group_ranks=ranks,
                                        sparse=plan, head_chunks=args.head_chunks,
                                        transport=transport, group=group)

        sp = make_layer()
        x_local = x_branch[:, sp.partition(B.SEQ)].contiguous()
        del x_full
        stream = torch.cuda.current_stream(device)
        attn_events = []

        def step(record: bool):
            # The public layer call; the Ulysses object records events around
            # each attention launch (one per head chunk) on the compute stream.
            sp.attention_events = attn_events if record else None
            try:
                return sp(x_local, rope, B.SEQ)
            finally:
                sp.attention_events = None

        for _ in range(args.warmup):
            step(False)
        torch.cuda.synchronize()
        dist.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with B.ClockSampler(local) as clocks:
            start.record(stream)
            for _ in range(args.steps):
                step(True)
            stop.record(stream)
            torch.cuda.synchronize()
        dist.barrier()
        ms = start.elapsed_time(stop) / args.steps
        kernel_ms = sum(a.elapsed_time(b) for a, b in attn_events) / args.steps
        status = _native.read_status(device)

        # End to end through the public API with host buffers (pinned).  Steps
        # alternate between two streams, each with its own Ulysses object (their
        # exchange buffers are per object); every rank issues the exchanges of
        # both in the same order.
        host_x = x_local.cpu().pin_memory()
        host_y = [torch.empty_like(host_x).pin_memory() for _ in range(2)]
        sp2 = make_layer()
        objects = [sp, sp2]
        dist.barrier()
        e2e_ms = B.run_e2e(lambda xd, i=[0]: _alternate(objects, i, xd, rope, B.SEQ), host_x,
                           host_y, device, args.warmup, args.steps)

        stats = torch.tensor([ms, kernel_ms, e2e_ms, float(status)], device=device)
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        ms, kernel_ms, e2e_ms, status = stats.tolist()
        # every rank's exchanges are done: release the peer buffers
        torch.cuda.synchronize()
        dist.barrier()
        sp.close()
        sp2.close()
        clock = clocks.summary()
        if rank == 0:
            if status:
                raise RuntimeError(f"kernel wait timed out on some rank (status {int(status)})")
            peaks, src = B.measured_peaks()
            peak_key = "bf16_tflops_sustained" if ms * args.steps >= 1000 else "bf16_tflops"
            peak = peaks[peak_key]
            if args.fp8:
                peak, peak_key = 2 * peak, f"2 x {peak_key} (dense fp8 = 2x bf16)"
            local_attn_flop = B.ATTN_FLOP * issued / world
            achieved = local_attn_flop / (kernel_ms / 1e3) / 1e12
            layer_flop = B.LINEAR_FLOP + B.ATTN_FLOP * kept
            parallelism = f"cfg{cfg}xsp{world // cfg}" if cfg > 1 else f"sp{world}"
            if ring > 1:
                parallelism += f" (ulysses{topo.ulysses} x ring{ring}, {args.ring_mode} ring)"
            parallelism += f", {transport} exchange"
            chunks = sp.chunks_for(B.SEQ)
            if chunks > 1:
                parallelism += f", {chunks} head chunks"
            attn_launches = chunks
            if ring > 1 and args.ring_mode != "reference":
                attn_launches = ring
            if plan is not None:
                workload = B.SPARSE_WORKLOAD + ", Ulysses SP (whole 128-token blocks per rank)"
                kernel = "attn_fwd_bf16 (block-sparse instantiation)"
            else:
                workload = B.WORKLOAD.replace(
                    "config 1", "config 2 (Ulysses x Ring SP)" if ring > 1
                    else "config 2 (Ulysses SP)")
                kernel = "attn_fwd_fp8" if args.fp8 else "attn_fwd_bf16"
            line = {
                "metric": B.METRIC, "value": layer_flop / (ms / 1e3) / 1e12, "unit": B.UNIT,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "e4m3/bf16" if args.fp8 else "bf16", "data": "synthetic",
                "config": {"workload": workload,
                           "global_batch": B.BATCH, "seq_len": B.SEQ, "parallelism": parallelism,
                           "l2": "inputs larger than L2"},
                "layer_tflop": layer_flop / 1e12,
                "roofline": {"kernel": kernel + " (per rank, max over ranks)",
                             "bound": "tensor", "achieved": achieved, "peak": peak,
                             "unit": B.UNIT, "frac": achieved / peak,
                             "peak_source": f"{src} {peak_key}",
                             "traffic": None, "kernel_ms": kernel_ms},
                "e2e": {"value": layer_flop / (e2e_ms / 1e3) / 1e12, "unit": B.UNIT,
                        "ms_per_step": e2e_ms,
                        "h2d_bytes_per_step": host_x.numel() * host_x.element_size() * world,
                        "d2h_bytes_per_step": host_y[0].numel() * host_y[0].element_size() * world,
                        "streams": 2},
                "gpu_launches": (1 + (3 if args.fp8 else 1) * attn_launches) * args.steps,
                "clocks": clock,
            }
            if plan is not None:
                line["sparsity"] = {"kept_pair_fraction": kept, "issued_pair_fraction": issued,
                                    "dense_equivalent": B.LAYER_FLOP / (ms / 1e3) / 1e12}
            print(json.dumps(line), flush=True)
    finally:
        dist.destroy_process_group()
