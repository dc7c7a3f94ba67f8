"""One EraserDiT self-attention layer (``attn1``) on a B200.

Follows ``EraserDiTAttentionProcessor.self_attn``
(``models/dits/eraserdit_attention.py:242-290``): QKV projection, QK RMSNorm
across heads, 3D RoPE, attention with scale head_dim ** -0.5, flatten heads,
output projection.  Data movement in HBM:

1. one GEMM (``erd_linear_bf16``, tcgen05) with the concatenated
   [Wq; Wk; Wv] writes Q|K|V interleaved per token ([B, S, 6144] BF16);
2. ``erd_qk_norm_rope`` normalises and rotates Q and K in place in that
   buffer (one read + one write of Q and K);
3. ``erd_attn_fwd_bf16`` reads Q/K/V straight from the interleaved buffer via
   TMA (token stride 6144) and writes O in [B, S, H*D] order (or, with
   ``precision="fp8"``, ``erd_attn_fwd_fp8`` quantises them into its
   workspace first);
4. one GEMM (``erd_linear_bf16``) applies ``to_out[0]``.

With a block-sparse plan (``sparse=``, see ``mask_sta.SparsePlan``) the layer
runs on a sequence in the plan's tile order: the prologue takes each token's
RoPE coordinates from the plan's order, ``erd_attn_fwd_sparse_bf16`` replaces
step 3, and the output stays in tile order (every other step is per token).
"""

from __future__ import annotations

import torch

from .attention import attention_bshd
from .linear import linear_bf16
from .mask_sta import sparse_attention_bshd
from .operator_fusion import qk_norm_rope_into
from .rotary import RopeAxisTable

HIDDEN = 2048
HEADS = 32
HEAD_DIM = 64


class EraserDiTSelfAttention:
    def __init__(self, wq, bq, wk, bk, wv, bv, wo, bo, norm_q, norm_k, eps: float,
                 heads: int = HEADS, device: torch.device | str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, precision: str = "bf16") -> None:
        device = torch.device(device)
        kw = dict(device=device, dtype=dtype)
        if heads * HEAD_DIM != HIDDEN:
            raise ValueError("the native path is built for 32 heads x 64")
        self.heads = heads
        self.eps = float(eps)
        self.w_qkv = torch.cat([wq, wk, wv], dim=0).to(**kw).contiguous()
        zero = torch.zeros(HIDDEN)
        self.b_qkv = torch.cat([zero if b is None else b.float().cpu() for b in (bq, bk, bv)]
                               ).to(**kw).contiguous()
        self.w_out = wo.to(**kw).contiguous()
        self.b_out = None if bo is None else bo.to(**kw).contiguous()
        self.norm_q = None if norm_q is None else norm_q.to(**kw).contiguous()
        self.norm_k = None if norm_k is None else norm_k.to(**kw).contiguous()
        self.softmax_scale = HEAD_DIM ** -0.5
        self.device = device
        if precision not in ("bf16", "fp8"):
            raise ValueError("precision must be bf16 or fp8")
        self.precision = precision
        self.qkv_fp8 = None  # optional SharedQKV (FP8 projection, static activation scale)

    def enable_qkv_fp8(self, activation_scale: float, wq, bq, wk, bk, wv, bv) -> None:
        """Project Q|K|V with the FP8 shared QKV GEMM (``qkv_fp8.SharedQKV``)."""
        from .qkv_fp8 import SharedQKV
        self.qkv_fp8 = SharedQKV(wq, bq, wk, bk, wv, bv, activation_scale, self.device)

    @classmethod
    def from_params(cls, p, device="cuda", precision: str = "bf16") -> "EraserDiTSelfAttention":
        """From an object with wq, bq, ..., norm_q, norm_k, eps attributes."""
        return cls(p.wq, p.bq, p.wk, p.bk, p.wv, p.bv, p.wo, p.bo, p.norm_q, p.norm_k, p.eps,
                   device=device, precision=precision)

    @classmethod
    def from_attention_module(cls, attn, device="cuda") -> "EraserDiTSelfAttention":
        """From a diffusers-style ``Attention`` (``to_q/k/v``, ``to_out[0]``, ``norm_q/k``)."""
        return cls(attn.to_q.weight, attn.to_q.bias, attn.to_k.weight, attn.to_k.bias,
                   attn.to_v.weight, attn.to_v.bias, attn.to_out[0].weight, attn.to_out[0].bias,
                   getattr(attn.norm_q, "weight", None), getattr(attn.norm_k, "weight", None),
                   attn.norm_q.eps, heads=attn.heads, device=device)

    def project_qkv(self, hidden_states: torch.Tensor) -> torch.Tensor:
        if self.qkv_fp8 is not None:
            return self.qkv_fp8.project(hidden_states)
        return linear_bf16(hidden_states, self.w_qkv, self.b_qkv)

    def core(self, qkv: torch.Tensor, rope, out: torch.Tensor | None = None,
             sparse=None) -> torch.Tensor:
        """Prologue + attention on a [B, S, 3*2048] QKV buffer (modified in place)."""
        batch, seq, _ = qkv.shape
        q, k, v = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN], qkv[..., 2 * HIDDEN:]
        if sparse is not None:
            if self.precision != "bf16":
                raise ValueError("the block-sparse path computes in BF16")
            if isinstance(rope, RopeAxisTable) and rope.grid_index is None:
                if sparse.order is None:
                    raise ValueError("the sparse plan has no token order for the RoPE table")
                rope = rope.in_order(sparse.order)
        qk_norm_rope_into(q, k, self.norm_q, self.norm_k, self.eps, rope, q, k)
        if out is None:
            out = torch.empty(batch, seq, HIDDEN, device=qkv.device, dtype=qkv.dtype)
        heads4 = lambda t: t.unflatten(2, (self.heads, HEAD_DIM))
        if sparse is not None:
            sparse_attention_bshd(heads4(q), heads4(k), heads4(v), self.softmax_scale, sparse,
                                  out=heads4(out))
        else:
            attention_bshd(heads4(q), heads4(k), heads4(v), self.softmax_scale, out=heads4(out),
                           precision=self.precision)
        return out

    def project_out(self, attn: torch.Tensor) -> torch.Tensor:
        return linear_bf16(attn, self.w_out, self.b_out)

    def forward(self, hidden_states: torch.Tensor, rope: RopeAxisTable | tuple | None,
                sparse=None) -> torch.Tensor:
        """``sparse``: a ``SparsePlan``; ``hidden_states`` are then in its tile order."""
        if hidden_states.dtype != torch.bfloat16 or hidden_states.shape[-1] != HIDDEN:
            raise ValueError("hidden_states must be BF16 [B, S, 2048]")
        qkv = self.project_qkv(hidden_states)
        return self.project_out(self.core(qkv, rope, sparse=sparse))

    __call__ = forward
