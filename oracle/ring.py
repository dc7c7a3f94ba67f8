"""CPU restatement of the reference's ring attention (pieces with a carried state).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``layers/attention/ring_accumulator.py`` (``_piece`` ``:12-86``,
``piece`` ``:88-100``) in torch fp32 on the CPU: per (batch, head), the key
blocks of 128 tokens of one piece are visited last block first; each block
updates the running max m, rescales the fp32 accumulator and four partial sums
(columns j with (j // 2) % 4 = 0, 1, 2, 3 of the block), and adds P V with P
rounded to the query dtype.  The final piece divides by (z0 + z2) + (z1 + z3).
The state is the tuple (acc [B, H, Nq, D], m [B, H, Nq], z [B, H, Nq, 4]).

``ring_pieces`` runs the reference's ring order
(``models/adapters/eraserdit/nccl_sequence.py:311-330``): the own piece first,
then the piece of ring index r - 1, r - 2, ...

Parity: the reference kernel is Triton on CUDA and cannot run here.  The
restatement is pinned to the identity it must satisfy: over any split of the
keys into pieces its output equals the full fp32 attention of
``oracle.reference_path`` (itself pinned to golden vectors) within fp32 and
P-rounding error (``tests/test_ring_oracle.py``).
"""

from __future__ import annotations

import math

import torch

LOG2E = 1.4426950408889634


def piece(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state=None, final: bool = False,
          scale: float | None = None, block: int = 128):
    """One ring piece on BSHD tensors; returns the next state or the output."""
    batch, nq, heads, dim = q.shape
    nk = k.shape[1]
    c = (dim ** -0.5 if scale is None else scale) * LOG2E
    qf = q.permute(0, 2, 1, 3).float()
    kf = k.permute(0, 2, 1, 3).float()
    vf = v.permute(0, 2, 1, 3).float()
    if state is None:
        acc = torch.zeros(batch, heads, nq, dim)
        m = torch.full((batch, heads, nq), -math.inf)
        z = torch.zeros(batch, heads, nq, 4)
    else:
        acc, m, z = (t.clone() for t in state)
    cols = torch.arange(block)
    group = (cols // 2) % 4  # ring_accumulator.py:44-67: partial sum of column j
    for start in range(((nk + block - 1) // block - 1) * block, -1, -block):
        kb, vb = kf[:, :, start:start + block], vf[:, :, start:start + block]
        s = qf @ kb.transpose(-1, -2)
        new_m = torch.maximum(m, s.amax(dim=-1))
        alpha = torch.exp2((m - new_m) * c)
        alpha = torch.where(torch.isnan(alpha), torch.zeros_like(alpha), alpha)
        p = torch.exp2(s * c - new_m[..., None] * c)
        acc = acc * alpha[..., None]
        n = p.shape[-1]
        for g in range(4):
            part = p[..., group[:n] == g].sum(dim=-1)
            z[..., g] = z[..., g] * alpha + part
        acc = acc + p.to(q.dtype).float() @ vb
        m = new_m
    if final:
        denom = (z[..., 0] + z[..., 2]) + (z[..., 1] + z[..., 3])
        return (acc / denom[..., None]).permute(0, 2, 1, 3)
    return acc, m, z


def ring_pieces(q: torch.Tensor, k_pieces: list[torch.Tensor], v_pieces: list[torch.Tensor],
                ring_rank: int, scale: float | None = None) -> torch.Tensor:
    """Attention of ``q`` over every piece, visited in the ring order of
    ``ring_rank`` (own piece, then r - 1, r - 2, ...)."""
    size = len(k_pieces)
    state = None
    out = None
    for hop in range(size):
        owner = (ring_rank - hop) % size
        result = piece(q, k_pieces[owner], v_pieces[owner], state, final=hop == size - 1,
                       scale=scale)
        if hop == size - 1:
            out = result
        else:
            state = result
    return out
