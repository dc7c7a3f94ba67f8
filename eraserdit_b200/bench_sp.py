"""Multi-GPU leg of ``bench.py``: Ulysses SP (optionally CFG x SP, or
Ulysses x Ring with ``--ring``) with peer-memory or NCCL exchanges.

Launched by torchrun with one process per GPU.  Every rank builds the same
seeded layer and input, keeps its floor-partitioned tokens (CFG: its branch's
batch entry) and runs the sequence-parallel layer; per-rank times come from
CUDA events and the reported time is the maximum over ranks (an all-reduce
MAX).

Before the timed loop every rank's layer output is gathered and rank 0
compares the assembled output with the single-GPU layer on the same seeded
input (the check of the reference's ``tests/test_nccl_dit.py:17-140``: the
sequence-parallel DiT equals the single-process one).  The result is printed
in the JSON line; a failed check makes the run exit non-zero.  With the
default dense BF16 configuration the line also carries the block-sparse
layer (configuration 4) under the same SP degree and, from 4 GPUs, the FP8
layer under CFG2 x SP (configuration 3), each timed and checked the same way.
"""

from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

BF16_BARS = {"min_cosine": 0.99999, "max_abs": 1e-2}
FP8_MIN_COSINE = 0.995


def gather_output(y_local: torch.Tensor, batch_range: tuple[int, int], tokens: slice,
                  batch: int, seq: int) -> torch.Tensor:
    """Every rank's [b, L_rank, H] output placed into the full [batch, seq, H]
    (returned on every rank; rows no rank owns stay zero)."""
    device = y_local.device
    world = dist.get_world_size()
    n = torch.tensor([y_local.shape[1]], device=device)
    dist.all_reduce(n, op=dist.ReduceOp.MAX)
    lmax = int(n.item())
    pad = torch.zeros(y_local.shape[0], lmax, y_local.shape[2], device=device,
                      dtype=y_local.dtype)
    pad[:, :y_local.shape[1]] = y_local
    meta = torch.tensor([batch_range[0], batch_range[1], tokens.start, tokens.stop],
                        device=device, dtype=torch.int64)
    pads = [torch.empty_like(pad) for _ in range(world)]
    metas = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(pads, pad)
    dist.all_gather(metas, meta)
    full = torch.zeros(batch, seq, y_local.shape[2], device=device, dtype=y_local.dtype)
    for part, m in zip(pads, metas):
        b0, b1, t0, t1 = m.tolist()
        full[b0:b1, t0:t1] = part[:, :t1 - t0]
    return full


def _check_against_single(B, y_local, batch_range, tokens, references, rank) -> dict | None:
    """Gathered output vs each (name, single-GPU output, bars) on rank 0."""
    full = gather_output(y_local, batch_range, tokens, B.BATCH, B.SEQ)
    if rank != 0:
        return None
    checks = {}
    for name, want, bars in references:
        checks[name] = B.parity(full, want, name, bars["min_cosine"], bars.get("max_abs"))
    return {"checks": checks, "ok": all(c["ok"] for c in checks.values())}


def _timed(sp, x_local, rope, seq, steps, warmup, clocks=None):
    """Device ms per call and attention-kernel ms (events the Ulysses object
    records around its attention launches), max over ranks with the caller."""
    stream = torch.cuda.current_stream(x_local.device)
    events = []

    def step(record: bool):
        sp.attention_events = events if record else None
        try:
            return sp(x_local, rope, seq)
        finally:
            sp.attention_events = None

    for _ in range(warmup):
        step(False)
    torch.cuda.synchronize()
    dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks is not None:
        clocks.__enter__()
    try:
        start.record(stream)
        for _ in range(steps):
            step(True)
        stop.record(stream)
        torch.cuda.synchronize()
    finally:
        if clocks is not None:
            clocks.__exit__(None, None, None)
    dist.barrier()
    ms = start.elapsed_time(stop) / steps
    kernel_ms = sum(a.elapsed_time(b) for a, b in events) / steps
    return ms, kernel_ms


def _max_over_ranks(device, *values):
    t = torch.tensor([float(v) for v in values], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


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
    failed = False
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
        branch = (cfg_index * per_branch, (cfg_index + 1) * per_branch)
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
        tokens = sp.partition(B.SEQ)
        x_local = x_full[branch[0]:branch[1], tokens].contiguous()

        # Output check before timing: the assembled SP output against the
        # single-GPU layer (rank 0 runs it on the same seeded input).
        y_local = sp(x_local, rope, B.SEQ)
        references = []
        if rank == 0:
            want = layer(x_full, rope, sparse=plan)
            if args.fp8:
                bf16_layer, _ = B.build_problem(device, "bf16")
                references = [("single-GPU FP8 layer", want, {"min_cosine": FP8_MIN_COSINE}),
                              ("single-GPU BF16 layer", bf16_layer(x_full, rope),
                               {"min_cosine": FP8_MIN_COSINE})]
                del bf16_layer
            else:
                references = [("single-GPU layer", want, BF16_BARS)]
        check = _check_against_single(B, y_local, branch, tokens, references, rank)
        del y_local, references

        clocks = B.ClockSampler(local, interval=0.02)
        ms, kernel_ms = _timed(sp, x_local, rope, B.SEQ, args.steps, args.warmup, clocks)
        status = _native.read_status(device)

        # End to end through the public API with host buffers (pinned): the
        # same Ulysses object, copies on their own streams.
        host_x = x_local.cpu().pin_memory()
        host_y = [torch.empty_like(host_x).pin_memory() for _ in range(2)]
        dist.barrier()
        e2e_ms = B.run_e2e(lambda xd: sp(xd, rope, B.SEQ), host_x, host_y, device,
                           args.warmup, args.steps)
        ms, kernel_ms, e2e_ms, status = _max_over_ranks(device, ms, kernel_ms, e2e_ms,
                                                        status or _native.read_status(device))
        torch.cuda.synchronize()
        dist.barrier()
        chunks = sp.chunks_for(B.SEQ)
        sp.close()
        del host_x, host_y

        extra = {}
        if not (args.fp8 or args.sparse or ring > 1 or cfg > 1 or args.no_extra):
            extra = _extra_legs(B, args, device, rank, world, groups, x_full, layer, rope)
        clock = clocks.summary()
        if rank == 0:
            if status:
                raise RuntimeError(f"kernel wait timed out on some rank (status {int(status)})")
            peaks, src = B.measured_peaks()
            peak_key = "bf16_tflops_sustained" if ms * args.steps >= 1000 else "bf16_tflops"
            peak = peaks[peak_key]
            bf16_peak, bf16_src = peak, f"{src} {peak_key}"
            if args.fp8:
                peak, peak_key = 2 * peak, f"2 x {peak_key} (dense fp8 = 2x bf16)"
            local_attn_flop = B.ATTN_FLOP * issued / world
            achieved = local_attn_flop / (kernel_ms / 1e3) / 1e12
            layer_flop = B.LINEAR_FLOP + B.ATTN_FLOP * kept
            parallelism = f"cfg{cfg}xsp{world // cfg}" if cfg > 1 else f"sp{world}"
            if ring > 1:
                parallelism += f" (ulysses{topo.ulysses} x ring{ring}, {args.ring_mode} ring)"
            parallelism += f", {transport} exchange"
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
                        "h2d_bytes_per_step": x_local.numel() * x_local.element_size() * world,
                        "d2h_bytes_per_step": x_local.numel() * x_local.element_size() * world,
                        "copy_streams": 2},
                # per step: QKV GEMM, prologue, the attention launches (FP8: three
                # kernels each), output GEMM; the peer transport adds a signal and a
                # bounded wait kernel around each of its two exchanges
                "gpu_launches": ((7 if transport == "peer" else 3)
                                 + (3 if args.fp8 else 1) * attn_launches) * args.steps,
                "clocks": clock,
                "parity": check,
            }
            if plan is not None:
                line["sparsity"] = {"kept_pair_fraction": kept, "issued_pair_fraction": issued,
                                    "dense_equivalent": B.LAYER_FLOP / (ms / 1e3) / 1e12}
            for leg in extra.values():
                leg["roofline"]["peak"] = (2 if leg.pop("fp8") else 1) * bf16_peak
                leg["roofline"]["frac"] = leg["roofline"]["achieved"] / leg["roofline"]["peak"]
                leg["roofline"]["peak_source"] = bf16_src
            if extra:
                line["extra"] = extra
            failed = not check["ok"] or any(not v["parity"]["ok"] for v in extra.values())
            print(json.dumps(line), flush=True)
        flag = _max_over_ranks(device, 1.0 if failed else 0.0)[0]
        failed = flag > 0
    finally:
        dist.destroy_process_group()
    if failed:
        raise SystemExit("sequence-parallel output check failed")


def _extra_legs(B, args, device, rank, world, groups, x_full, layer, rope) -> dict:
    """Configuration 4 (block-sparse) under the same SP degree and, from 4 GPUs,
    configuration 3 (FP8 attention, CFG2 x SP) -- timed (max over ranks) and
    checked against the single-GPU layer like the main leg."""
    from eraserdit_b200.topology import DiTGroups, DiTTopology
    from eraserdit_b200.ulysses import UlyssesSelfAttention, peer_exchange
    steps = min(args.steps, 10)
    extra = {}

    # ---- configuration 4: block-sparse, Ulysses SP over all ranks
    plan, kept, issued = B.build_sparse_plan(device)
    group, ranks, index = groups.get("ulysses")
    sp = UlyssesSelfAttention(layer, len(ranks), index, peer_exchange(group, ranks, index),
                              group_ranks=ranks, sparse=plan, transport=args.transport,
                              group=group)
    tokens = sp.partition(B.SEQ)
    x_local = x_full[:, tokens].contiguous()
    y_local = sp(x_local, rope, B.SEQ)
    refs = [("single-GPU block-sparse layer", layer(x_full, rope, sparse=plan), BF16_BARS)] \
        if rank == 0 else []
    check = _check_against_single(B, y_local, (0, B.BATCH), tokens, refs, rank)
    del y_local, refs
    ms, kms = _timed(sp, x_local, rope, B.SEQ, steps, args.warmup)
    ms, kms = _max_over_ranks(device, ms, kms)
    torch.cuda.synchronize()
    dist.barrier()
    sp.close()
    achieved = B.ATTN_FLOP * issued / world / (kms / 1e3) / 1e12
    extra["sparse"] = {
        "workload": B.SPARSE_WORKLOAD + f", Ulysses SP{world}, {args.transport} exchange",
        "ms_per_step": ms, "value": (B.LINEAR_FLOP + B.ATTN_FLOP * kept) / (ms / 1e3) / 1e12,
        "unit": B.UNIT, "dense_equivalent": B.LAYER_FLOP / (ms / 1e3) / 1e12,
        "kept_pair_fraction": kept, "issued_pair_fraction": issued,
        "roofline": {"kernel": "attn_fwd_bf16 (block-sparse instantiation, per rank)",
                     "bound": "tensor", "achieved": achieved, "unit": B.UNIT, "kernel_ms": kms},
        "parity": check, "fp8": False,
    }

    # ---- configuration 3: FP8 attention, CFG2 x SP(world / 2)
    if world >= 4:
        topo = DiTTopology(ulysses=world // 2, cfg=2)
        groups2 = DiTGroups(topo)
        group, ranks, index = groups2.get("ulysses")
        cfg_index = topo.coordinates(rank)[3]
        layer8, _ = B.build_problem(device, "fp8")
        sp = UlyssesSelfAttention(layer8, len(ranks), index, peer_exchange(group, ranks, index),
                                  group_ranks=ranks, transport=args.transport, group=group)
        tokens = sp.partition(B.SEQ)
        x_local = x_full[cfg_index:cfg_index + 1, tokens].contiguous()
        y_local = sp(x_local, rope, B.SEQ)
        refs = []
        if rank == 0:
            refs = [("single-GPU FP8 layer", layer8(x_full, rope), {"min_cosine": FP8_MIN_COSINE}),
                    ("single-GPU BF16 layer", layer(x_full, rope), {"min_cosine": FP8_MIN_COSINE})]
        check = _check_against_single(B, y_local, (cfg_index, cfg_index + 1), tokens, refs, rank)
        del y_local, refs
        ms, kms = _timed(sp, x_local, rope, B.SEQ, steps, args.warmup)
        ms, kms = _max_over_ranks(device, ms, kms)
        torch.cuda.synchronize()
        dist.barrier()
        sp.close()
        achieved = B.ATTN_FLOP / world / (kms / 1e3) / 1e12
        extra["cfg2_fp8"] = {
            "workload": ("config 3: CFG2 x SP{} (cond / uncond branches on separate rank groups, "
                         "B=1 x 32640 each), FP8 attention (E4M3, per-128-token Q/K scales, "
                         "smoothed K, per-channel V scales), {} exchange").format(
                             world // 2, args.transport),
            "ms_per_step": ms, "value": B.LAYER_FLOP / (ms / 1e3) / 1e12, "unit": B.UNIT,
            "roofline": {"kernel": "attn_fwd_fp8 (+ fp8 quantize, per rank)", "bound": "tensor",
                         "achieved": achieved, "unit": B.UNIT, "kernel_ms": kms},
            "parity": check, "fp8": True,
        }
    return extra
