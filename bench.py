"""Benchmark: one EraserDiT self-attention layer at 2 x 32640 tokens on B200.

Metric: "DiT self-attn layer ms & TFLOP/s @2x32640 tok,
1/2/4/8 B200 (% of peak)".  One step = one full layer (QKV projection, fused
QK RMSNorm + RoPE, attention, output projection; at N > 1 the Ulysses
all-to-all exchanges as well) over B=2 x 32640 synthetic tokens (N(0, 1)
hidden states, N(0, 0.02) weights, seed 1).  ``value`` is whole-job TFLOP/s
(19.645 TFLOP per layer / max-over-ranks step time).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--fp8 | --sparse] [--cfg C]

``--fp8`` times the Sage-style FP8 attention (configuration 3's numerics);
``--sparse`` the mask-aware block-sparse attention of configuration 4 (tokens
in tile order, a seeded ellipse mask per latent frame): its ``value`` counts
the FLOPs of the kept (query, key) pairs, ``dense_equivalent`` the full
layer's FLOPs over the same time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, FRAMES, HEIGHT, WIDTH = 2, 16, 34, 60
SEQ = FRAMES * HEIGHT * WIDTH
HIDDEN, HEADS, HEAD_DIM = 2048, 32, 64
EPS = 1e-6
LINEAR_FLOP = 4 * 2 * BATCH * SEQ * HIDDEN * HIDDEN
ATTN_FLOP = 4 * BATCH * HEADS * SEQ * SEQ * HEAD_DIM
LAYER_FLOP = LINEAR_FLOP + ATTN_FLOP
METRIC = "DiT self-attn layer ms & TFLOP/s @2x32640 tok, 1/2/4/8 B200 (% of peak)"
UNIT = "TFLOP/s"
WORKLOAD = ("config 1: one DiT self-attention layer (QKV proj, QK RMSNorm, 3D RoPE, "
            "SDPA, out proj), B=2 (CFG stacked) x 32640 tokens (16x34x60), "
            "hidden 2048, 32x64 heads, BF16")


def log(msg: str) -> None:
    print(msg, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ helpers
def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profiled_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = ROOT / "profiles" / f"{kernel}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region.

    Reads NVML from a thread every ``interval`` seconds (read-only queries:
    5 ms on one GPU, 20 ms per rank on several, where eight processes polling
    the driver would otherwise share it with the short layer steps); falls back to
    ``nvidia-smi -lms 50`` when NVML is unavailable.  Nothing is changed on the
    device."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, interval: float = 0.005) -> None:
        self.index = index
        self.interval = interval
        self.proc = None
        self.file = None
        self.thread = None
        self.samples: list[tuple[float, int]] = []
        self.max_sm = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:  # the CUDA ordinal and the NVML index differ under CUDA_VISIBLE_DEVICES
            prop = torch.cuda.get_device_properties(self.index)
            bus = f"{prop.pci_domain_id:08X}:{prop.pci_bus_id:02X}:{prop.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            nvml, handle = self._nvml_handle()
            self.max_sm = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                        bits = nvml.nvmlDeviceGetCurrentClocksThrottleReasons(handle)
                        self.samples.append((float(sm), int(bits)))
                    except Exception:
                        pass
                    self._stop.wait(self.interval)
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.thread is not None:
            sm = [c for c, _ in self.samples]
            reasons = sorted({name for _, bits in self.samples
                              for bit, name in self.REASONS.items() if bits & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": float(self.max_sm) if self.max_sm else None,
                    "reasons": reasons, "samples": len(sm),
                    "source": f"nvml {self.interval * 1e3:.0f} ms"}
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, value in zip(names, r[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi 50 ms"}


# ------------------------------------------------------------- CPU sample
def cpu_sample_step(threads: int):
    """1/64 of the config-1 layer through the oracle (the reference's CPU path):
    the four projections for 1020 of the 65280 tokens, their QK RMSNorm + RoPE,
    and one (batch, head) of attention over the full 32640-token sequence."""
    from oracle import reference_path as ref
    torch.set_num_threads(threads)
    rows = BATCH * SEQ // 64
    g = torch.Generator().manual_seed(7)
    x = torch.randn(1, rows, HIDDEN, generator=g)
    w = [torch.randn(HIDDEN, HIDDEN, generator=g) * 0.02 for _ in range(4)]
    b = torch.zeros(HIDDEN)
    ones = torch.ones(HIDDEN)
    cos, sin = ref.rope_table(1, FRAMES, HEIGHT, WIDTH)
    cos, sin = cos[:, :rows], sin[:, :rows]
    qh, kh, vh = (torch.randn(1, SEQ, 1, HEAD_DIM, generator=g) for _ in range(3))
    flop = 4 * 2 * rows * HIDDEN * HIDDEN + 4 * SEQ * SEQ * HEAD_DIM

    def step():
        with torch.no_grad():
            q = ref.rms_norm(torch.nn.functional.linear(x, w[0], b), ones, EPS)
            k = ref.rms_norm(torch.nn.functional.linear(x, w[1], b), ones, EPS)
            v = torch.nn.functional.linear(x, w[2], b)
            q, k = ref.apply_rotary_emb(q, cos, sin), ref.apply_rotary_emb(k, cos, sin)
            core = ref.sdpa_bshd(qh, kh, vh, 0.125)
            torch.nn.functional.linear(v, w[3], b)
        return core
    return step, flop, (f"1/64 of the layer: projections + QK norm/RoPE for {rows} tokens and one "
                        f"(batch, head) of fp32 SDPA over {SEQ} tokens")


def cpu_model() -> str:
    """The host CPU's model name (as lscpu reports it)."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(steps: int = 12) -> dict:
    threads = os.cpu_count() or 1
    step, flop, sample = cpu_sample_step(threads)
    step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    return {"value": flop / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": sample + f"; {steps} timed steps of {dt:.2f} s"}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    step, flop, sample = cpu_sample_step(threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = flop / dt / 1e12
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": BATCH, "seq_len": SEQ,
                   "parallelism": "cpu", "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------ GPU arm
def build_problem(device, precision: str = "bf16"):
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.synthetic import make_params  # seeded synthetic weights
    params = make_params(1, EPS, device=device)
    layer = EraserDiTSelfAttention.from_params(params.to(torch.bfloat16), device=device,
                                               precision=precision)
    rope = LTXVideoRotaryPosEmbed()(FRAMES, HEIGHT, WIDTH, device=device)
    return layer, rope


SPARSE_WORKLOAD = ("config 4: mask-aware block-sparse self-attention layer, B=2 x 32640 tokens "
                   "(16x34x60) in 4x2x4-cell tile order, one seeded ellipse per latent frame "
                   "(semi-axes 6-12 cells, drift <= 1 cell/frame, seed 3) dilated by 2 cells; "
                   "masked-neighbourhood query blocks attend all keys, the others a 3x9x9-cell "
                   "window rounded out to tiles; BF16")


def enable_qkv_fp8(layer, x) -> None:
    """FP8 shared QKV with the activation scale calibrated on the input (amax / 448)."""
    from eraserdit_b200.synthetic import make_params
    p = make_params(1, EPS, device=x.device).to(torch.bfloat16)
    layer.enable_qkv_fp8(float(x.float().abs().amax()) / 448, p.wq, p.bq, p.wk, p.bk, p.wv, p.bv)


def build_sparse_plan(device):
    """Configuration 4's pattern; returns (plan, kept fraction, issued fraction)."""
    from eraserdit_b200 import sparse_pattern as sp
    from eraserdit_b200.mask_sta import SparsePlan
    geom = sp.CONFIG4_GEOMETRY
    plan = SparsePlan.from_mask(sp.ellipse_masks(geom.grid, seed=3), geom, device)
    issued = plan.host.issued_pairs / plan.host.dense_pairs
    return plan, plan.keep_fraction, issued


def run_e2e(call, host_x, host_y, device, warmup: int, steps: int) -> float:
    """ms per step of: pinned host -> device copy of the step's input, ``call``
    on the current stream, device -> pinned host copy of its output (timed on
    the device).  The copies run on two copy streams with double-buffered
    device inputs, so step i+1's upload and step i's download overlap the
    kernels of the neighbouring steps; the layer itself runs on one stream."""
    compute = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    xd = [torch.empty(host_x.shape, dtype=host_x.dtype, device=device) for _ in range(2)]
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def one(i):
        k = i % 2
        up.wait_event(consumed[k])  # step i - 2 has finished with xd[k]
        with torch.cuda.stream(up):
            xd[k].copy_(host_x, non_blocking=True)
            uploaded[k].record(up)
        compute.wait_event(uploaded[k])
        y = call(xd[k])
        consumed[k].record(compute)
        down.wait_event(consumed[k])
        with torch.cuda.stream(down):
            host_y[k].copy_(y, non_blocking=True)
        y.record_stream(down)

    for i in range(max(warmup, 1)):
        one(i)
    compute.wait_stream(down)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    up.wait_event(start)
    for i in range(steps):
        one(i)
    compute.wait_stream(down)
    stop.record(compute)
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / steps


def parity(got: torch.Tensor, want: torch.Tensor, vs: str, min_cosine: float,
           max_abs: float | None = None) -> dict:
    """Max-abs difference and cosine of two outputs, against the stated bars."""
    g, w = got.float().flatten(), want.float().flatten()
    err = float((g - w).abs().max()) if g.numel() else 0.0
    cos = float(torch.nn.functional.cosine_similarity(g.double(), w.double(), dim=0))
    ok = cos >= min_cosine and (max_abs is None or err <= max_abs)
    bars = {"min_cosine": min_cosine}
    if max_abs is not None:
        bars["max_abs"] = max_abs
    return {"vs": vs, "max_abs": err, "cosine": cos, "bars": bars, "ok": ok}


def time_layer(layer, rope, x, plan, precision: str, steps: int, warmup: int, clocks=None):
    """Device ms per layer step (the calls of ``EraserDiTSelfAttention.forward``)
    and the attention kernel's mean ms from CUDA events around its launch on the
    stream it is enqueued on.  Returns (ms, kernel_ms, last output)."""
    from eraserdit_b200.attention import attention_bshd
    from eraserdit_b200.mask_sta import sparse_attention_bshd
    from eraserdit_b200.operator_fusion import qk_norm_rope_into
    device = x.device
    stream = torch.cuda.current_stream(device)
    attn_out = torch.empty(x.shape[0], x.shape[1], HIDDEN, device=device, dtype=torch.bfloat16)
    if plan is not None:
        rope = rope.in_order(plan.order)  # the sequence is laid out in tile order
    events = []

    def step(record: bool):
        qkv = layer.project_qkv(x)
        q, k, v = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN], qkv[..., 2 * HIDDEN:]
        qk_norm_rope_into(q, k, layer.norm_q, layer.norm_k, layer.eps, rope, q, k)
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        heads4 = lambda t: t.unflatten(2, (HEADS, HEAD_DIM))
        if plan is not None:
            sparse_attention_bshd(heads4(q), heads4(k), heads4(v), layer.softmax_scale, plan,
                                  out=heads4(attn_out))
        else:
            attention_bshd(heads4(q), heads4(k), heads4(v), layer.softmax_scale,
                           out=heads4(attn_out), precision=precision)
        if record:
            e1.record(stream)
            events.append((e0, e1))
        return layer.project_out(attn_out)

    for _ in range(warmup):
        step(False)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks is not None:
        clocks.__enter__()
    try:
        start.record(stream)
        for _ in range(steps):
            y = step(True)
        stop.record(stream)
        torch.cuda.synchronize()
    finally:
        if clocks is not None:
            clocks.__exit__(None, None, None)
    ms = start.elapsed_time(stop) / steps
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in events)
    return ms, kernel_ms, y


def protected_rows(plan, seq: int) -> torch.Tensor:
    """Token positions (tile order) of the query blocks that attend every key."""
    full = plan.blocks.all(dim=1).nonzero().flatten()
    rows = (full[:, None] * 128 + torch.arange(128)[None, :]).flatten()
    return rows[rows < seq]


def extra_legs(device, x, rope, y_bf16, steps: int, warmup: int, peak_bf16: float,
               peak_src: str) -> dict:
    """Configurations 3 (FP8 attention numerics) and 4 (block-sparse) on one GPU,
    each with its own device time, roofline and an output check."""
    extra = {}
    # FP8 attention (configuration 3's numerics) on the configuration-1 layer.
    layer8, _ = build_problem(device, "fp8")
    ms, kms, y = time_layer(layer8, rope, x, None, "fp8", steps, warmup)
    achieved = ATTN_FLOP / (kms / 1e3) / 1e12
    extra["fp8"] = {
        "workload": "config 3 numerics on one GPU: FP8 (E4M3, per-128-token Q/K scales, "
                    "smoothed K, per-channel V scales) attention in the config-1 layer, "
                    "B=2 x 32640",
        "ms_per_step": ms, "value": LAYER_FLOP / (ms / 1e3) / 1e12, "unit": UNIT,
        "roofline": {"kernel": "attn_fwd_fp8 (+ fp8 quantize)", "bound": "tensor",
                     "achieved": achieved, "peak": 2 * peak_bf16, "unit": UNIT,
                     "frac": achieved / (2 * peak_bf16),
                     "peak_source": f"{peak_src}: dense fp8 = 2 x bf16", "kernel_ms": kms},
        "parity": parity(y, y_bf16, "the BF16 layer on the same input (north-star FP8 bar)",
                         0.995),
    }
    del layer8, y
    # Block-sparse attention (configuration 4); its protected query blocks
    # attend every key, so their rows equal the dense layer's.
    layer, rope1 = build_problem(device, "bf16")
    plan, kept, issued = build_sparse_plan(device)
    ms, kms, y = time_layer(layer, rope1, x, plan, "bf16", steps, warmup)
    dense = layer(x, rope1.in_order(plan.order))
    rows = protected_rows(plan, SEQ).to(device)
    achieved = ATTN_FLOP * issued / (kms / 1e3) / 1e12
    layer_flop = LINEAR_FLOP + ATTN_FLOP * kept
    extra["sparse"] = {
        "workload": SPARSE_WORKLOAD,
        "ms_per_step": ms, "value": layer_flop / (ms / 1e3) / 1e12, "unit": UNIT,
        "dense_equivalent": LAYER_FLOP / (ms / 1e3) / 1e12,
        "kept_pair_fraction": kept, "issued_pair_fraction": issued,
        "roofline": {"kernel": "attn_fwd_bf16 (block-sparse instantiation)", "bound": "tensor",
                     "achieved": achieved, "peak": peak_bf16, "unit": UNIT,
                     "frac": achieved / peak_bf16, "peak_source": peak_src, "kernel_ms": kms},
        "parity": parity(y[:, rows], dense[:, rows],
                         f"the dense BF16 layer on the {rows.numel()} rows of query blocks "
                         "that attend every key", 0.99999, 1e-2),
    }
    return extra


def run_single(args) -> None:
    from eraserdit_b200 import _native
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    precision = "fp8" if args.fp8 else "bf16"
    layer, rope = build_problem(device, precision)
    plan, kept, issued = build_sparse_plan(device) if args.sparse else (None, 1.0, 1.0)
    g = torch.Generator(device=device).manual_seed(1)
    x = torch.randn(BATCH, SEQ, HIDDEN, generator=g, device=device).bfloat16()
    if args.qkv_fp8:
        enable_qkv_fp8(layer, x)
    clocks = ClockSampler(device.index)
    ms, core_ms, y = time_layer(layer, rope, x, plan, precision, args.steps, args.warmup,
                                clocks=clocks)
    status = _native.read_status(device)
    if status:
        raise RuntimeError(f"kernel wait timed out (status {status})")

    # End to end through the public API: pinned host input -> layer -> pinned host
    # output, every step (copies on their own streams, overlapping the kernels).
    host_x = x.cpu().pin_memory()
    host_y = [torch.empty(BATCH, SEQ, HIDDEN, dtype=torch.bfloat16).pin_memory()
              for _ in range(2)]
    e2e_ms = run_e2e(lambda xd: layer(xd, rope, sparse=plan), host_x, host_y, device,
                     args.warmup, args.steps)

    peaks, peak_src = measured_peaks()
    timed_s = ms * args.steps / 1e3
    peak_key = "bf16_tflops_sustained" if timed_s >= 1.0 else "bf16_tflops"
    peak = peaks[peak_key]
    bf16_peak, bf16_src = peak, f"{peak_src} {peak_key}"
    if args.fp8:  # dense FP8 runs at twice the BF16 rate on this part
        peak, peak_key = 2 * peak, f"2 x {peak_key} (dense fp8 = 2x bf16)"
    # Sparse: algorithmic FLOPs are those of the kept pairs; the kernel's
    # roofline counts the products it issues (the union of a CTA's two lists).
    layer_flop = LINEAR_FLOP + ATTN_FLOP * kept
    achieved = ATTN_FLOP * issued / (core_ms / 1e3) / 1e12
    clock = clocks.summary()
    if plan is not None:
        workload, kernel = SPARSE_WORKLOAD, "attn_fwd_bf16 (block-sparse instantiation)"
    elif args.fp8:
        workload = WORKLOAD + ", FP8 attention (configuration 3 numerics)"
        kernel = "attn_fwd_fp8 (+ fp8 quantize)"
    else:
        workload, kernel = WORKLOAD, "attn_fwd_bf16"
    if args.qkv_fp8:
        workload += ", FP8 shared QKV projection (E4M3, static activation scale)"
    line = {
        "metric": METRIC, "value": layer_flop / (ms / 1e3) / 1e12, "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3/bf16" if (args.fp8 or args.qkv_fp8) else "bf16", "data": "synthetic",
        "config": {"workload": workload,
                   "global_batch": BATCH, "seq_len": SEQ, "parallelism": "sp1",
                   "l2": "inputs larger than L2 (x 267 MB, QKV 802 MB per step)"},
        "layer_tflop": layer_flop / 1e12,
        "roofline": {"kernel": kernel,
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak,
                     "peak_source": f"{peak_src} {peak_key}",
                     "traffic": None if (args.fp8 or plan is not None)
                     else profiled_traffic("attn_fwd_bf16_config1"),
                     "kernel_ms": core_ms},
        "e2e": {"value": layer_flop / (e2e_ms / 1e3) / 1e12, "unit": UNIT,
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": host_x.numel() * host_x.element_size(),
                "d2h_bytes_per_step": host_y[0].numel() * host_y[0].element_size(),
                "copy_streams": 2},
        # per layer step: QKV GEMM, prologue, attention (FP8: + statistics and
        # quantisation passes), output GEMM; the FP8 QKV projection adds its
        # activation quantiser
        "gpu_launches": ((6 if args.fp8 else 4) + (1 if args.qkv_fp8 else 0)) * args.steps,
        "clocks": clock,
    }
    if plan is not None:
        line["sparsity"] = {"kept_pair_fraction": kept, "issued_pair_fraction": issued,
                            "dense_equivalent": LAYER_FLOP / (ms / 1e3) / 1e12,
                            "dense_equivalent_e2e": LAYER_FLOP / (e2e_ms / 1e3) / 1e12}
    failed = []
    if not (args.fp8 or args.sparse or args.qkv_fp8 or args.no_extra):
        del host_x, host_y
        line["extra"] = extra_legs(device, x, rope, y, min(args.steps, 10), args.warmup,
                                   bf16_peak, bf16_src)
        failed = [k for k, v in line["extra"].items() if not v["parity"]["ok"]]
        if _native.read_status(device):
            raise RuntimeError("kernel wait timed out in an extra leg")
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    print(json.dumps(line), flush=True)
    if failed:
        raise SystemExit(f"output check failed: {failed}")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="native", choices=["native", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extra", action="store_true",
                        help="skip the configuration-3/4 legs and the output checks")
    parser.add_argument("--cfg", type=int, default=1, help="CFG branches on separate rank groups")
    parser.add_argument("--fp8", action="store_true",
                        help="Sage-style FP8 attention (configuration 3) instead of BF16")
    parser.add_argument("--sparse", action="store_true",
                        help="mask-aware block-sparse attention (configuration 4)")
    parser.add_argument("--qkv-fp8", action="store_true",
                        help="FP8 shared QKV projection (static activation scale)")
    parser.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                        help="Ulysses exchange: peer-memory stores over NVLink or NCCL all-to-all")
    parser.add_argument("--head-chunks", type=int, default=None,
                        help="Ulysses head chunks (exchange/attention overlap); default: policy")
    parser.add_argument("--ring", type=int, default=1,
                        help="ring degree of Ulysses x Ring (USP) sequence parallelism")
    parser.add_argument("--ring-mode", default="streaming", choices=["reference", "streaming"],
                        help="ring mode: gather every K/V piece, or pieces with a carried state")
    args = parser.parse_args()
    if args.fp8 and args.sparse:
        parser.error("--fp8 and --sparse are separate configurations")
    if args.ring > 1 and (args.fp8 or args.sparse or args.qkv_fp8):
        parser.error("the ring path computes dense BF16 attention")
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.gpus == 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        run_single(args)
        return
    from eraserdit_b200.bench_sp import run_sequence_parallel
    run_sequence_parallel(args)


if __name__ == "__main__":
    main()
