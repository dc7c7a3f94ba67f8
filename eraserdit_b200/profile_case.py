"""Small, self-contained workloads for ncu captures of the path's kernels.

    python -m eraserdit_b200.profile_case attention --batch 1 --seq 16320 --iters 3
    python -m eraserdit_b200.profile_case prologue --batch 2 --seq 32640 --iters 3
    python -m eraserdit_b200.profile_case fp8 --batch 1 --seq 16320 --iters 3
    python -m eraserdit_b200.profile_case sparse --batch 1 --heads 16 --iters 3
    python -m eraserdit_b200.profile_case ring --batch 1 --seq 16320 --iters 2
    python -m eraserdit_b200.profile_case linear --batch 1 --seq 16320 --iters 3
    python -m eraserdit_b200.profile_case cudnn --batch 1 --seq 16320 --iters 3

``sparse`` runs the configuration-4 pattern (32640 tokens in tile order, the
seeded ellipse mask) whatever ``--seq`` says.  ``ring`` attends ``--seq``
queries to two ring pieces of ``--seq`` keys each with the carried state (the
per-rank work of ring degree 2): per iteration, one launch writing the state
and one reading it and writing the output.  ``linear`` runs the QKV
projection (``--batch`` x ``--seq`` rows of 2048 into ``--n`` columns, 6144 by
default, with bias)
through ``erd_linear_bf16``.  ``cudnn`` runs torch's SDPA with the cuDNN backend
on the same [B, H, S, 64] BF16 shape: a library yardstick for the attention
kernel, not part of the path.

Each runs the named kernel ``iters`` times on seeded inputs (sized above L2 by
default) and exits 0, so that an ncu capture (``-k``/``-c``) of one to three
launches ends by itself.
"""

from __future__ import annotations

import argparse

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["attention", "prologue", "fp8", "sparse", "ring",
                                       "linear", "cudnn"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=16320)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--n", type=int, default=6144, help="linear: output columns")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(0)
    from eraserdit_b200 import _native
    if args.kernel == "cudnn":
        from torch.nn.attention import SDPBackend, sdpa_kernel
        q, k, v = (torch.randn(args.batch, args.heads, args.seq, 64, generator=g,
                               device=device).bfloat16() for _ in range(3))
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            for _ in range(args.iters):
                torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=0.125)
        torch.cuda.synchronize()
        return
    if args.kernel == "linear":
        from eraserdit_b200.linear import linear_bf16
        x = torch.randn(args.batch * args.seq, 2048, generator=g, device=device).bfloat16()
        w = (torch.randn(args.n, 2048, generator=g, device=device) * 0.02).bfloat16()
        b = torch.zeros(args.n, device=device, dtype=torch.bfloat16)
        y = torch.empty(args.batch * args.seq, args.n, device=device, dtype=torch.bfloat16)
        for _ in range(args.iters):
            linear_bf16(x, w, b, out=y)
    elif args.kernel == "ring":
        from eraserdit_b200.ring import piece
        mk = lambda: torch.randn(args.batch, args.seq, args.heads, 64, generator=g,
                                 device=device).bfloat16()
        q, k0, v0, k1, v1 = mk(), mk(), mk(), mk(), mk()
        for _ in range(args.iters):
            state = piece(q, k0, v0, scale=0.125)
            piece(q, k1, v1, state, final=True, scale=0.125)
    elif args.kernel in ("attention", "fp8", "sparse"):
        from eraserdit_b200.attention import attention_bshd
        plan = None
        if args.kernel == "sparse":
            from eraserdit_b200 import sparse_pattern as sp
            from eraserdit_b200.mask_sta import SparsePlan, sparse_attention_bshd
            geom = sp.CONFIG4_GEOMETRY
            plan = SparsePlan.from_mask(sp.ellipse_masks(geom.grid, seed=3), geom, device)
            args.seq = geom.tokens
        qkv = torch.randn(args.batch, args.seq, 3, args.heads, 64, generator=g,
                          device=device).bfloat16()
        out = torch.empty(args.batch, args.seq, args.heads, 64, device=device,
                          dtype=torch.bfloat16)
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        for _ in range(args.iters):
            if plan is not None:
                sparse_attention_bshd(q, k, v, 0.125, plan, out=out)
            else:
                attention_bshd(q, k, v, 0.125, out=out,
                               precision="fp8" if args.kernel == "fp8" else "bf16")
    else:
        from eraserdit_b200.operator_fusion import qk_norm_rope_into
        from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
        frames = max(1, args.seq // (34 * 60))
        rope = LTXVideoRotaryPosEmbed()(frames, 34, 60, device=device)
        seq = rope.tokens
        qkv = torch.randn(args.batch, seq, 6144, generator=g, device=device).bfloat16()
        w = torch.ones(2048, device=device, dtype=torch.bfloat16)
        q, k = qkv[..., :2048], qkv[..., 2048:4096]
        for _ in range(args.iters):
            qk_norm_rope_into(q, k, w, w, 1e-6, rope, q, k)
    torch.cuda.synchronize()
    if _native.read_status(device):
        raise SystemExit("a kernel wait timed out")


if __name__ == "__main__":
    main()
