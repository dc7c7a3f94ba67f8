"""Shared comparison helpers for the parity tests."""

from __future__ import annotations

import torch


def bf16_ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise distance in BF16 units in the last place (+0 == -0)."""
    def key(t):
        u = t.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
        neg = (u & 0x8000) != 0
        return torch.where(neg, -(u & 0x7FFF), u)
    return (key(a) - key(b)).abs()


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.double() - b.double()).abs().max())


def attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                   block: int = 4096) -> torch.Tensor:
    """fp32 softmax(Q K^T scale) V on BSHD tensors, chunked over heads and queries."""
    batch, seq, heads, dim = q.shape
    out = torch.empty(batch, seq, heads, dim, dtype=torch.float32, device=q.device)
    for b in range(batch):
        for h in range(heads):
            kf = k[b, :, h].float()
            vf = v[b, :, h].float()
            for s0 in range(0, seq, block):
                qf = q[b, s0:s0 + block, h].float()
                logits = (qf @ kf.T) * scale
                out[b, s0:s0 + block, h] = torch.softmax(logits, dim=-1) @ vf
    return out


def masked_attention_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                          blocks: torch.Tensor, kv_block: int, query_block: int = 128,
                          rows: int = 2048) -> torch.Tensor:
    """fp32 attention over the keys a block pattern keeps (bool [S/query_block,
    S/kv_block] over the sequence order of q/k/v), chunked over heads and queries."""
    batch, seq, heads, dim = q.shape
    blocks = blocks.to(q.device)
    out = torch.empty(batch, seq, heads, dim, dtype=torch.float32, device=q.device)
    for b in range(batch):
        for h in range(heads):
            kf = k[b, :, h].float()
            vf = v[b, :, h].float()
            for s0 in range(0, seq, rows):
                qf = q[b, s0:s0 + rows, h].float()
                keep = blocks[s0 // query_block:(s0 + qf.shape[0] + query_block - 1) // query_block]
                keep = keep.repeat_interleave(query_block, 0)[:qf.shape[0]]
                keep = keep.repeat_interleave(kv_block, 1)
                logits = ((qf @ kf.T) * scale).masked_fill(~keep, float("-inf"))
                out[b, s0:s0 + rows, h] = torch.softmax(logits, dim=-1) @ vf
    return out
