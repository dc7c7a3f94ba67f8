"""CPU restatement of the reference's DiT self-attention path (torch fp32 / bf16).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA product path and the timed
CPU baseline.  Never imported by ``eraserdit_b200``.

Every function follows one reference site (paths relative to the reference
project root).  The reference's path is Python over torch ops, so this
restatement uses the same torch CPU ops in the same order; where the reference
depends on a third-party implementation that is absent here (diffusers 0.40.0
``RMSNorm``), the restatement follows the reference's own bit-exact description
of it (``layers/operator_fusion/triton/rmsnorm_native.py:25-43``) and the
reference's tests, which treat ``torch.nn.RMSNorm`` and diffusers ``RMSNorm`` as
interchangeable (``tests/test_operator_fusion_precision.py:92``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

HIDDEN = 2048
HEADS = 32
HEAD_DIM = 64
ROPE_BASE = (20, 2048, 2048)  # eraserdit_transformer.py:402-410
ROPE_THETA = 10000.0


# ---------------------------------------------------------------- RoPE table
def rope_frequencies(dim: int = HIDDEN, theta: float = ROPE_THETA) -> torch.Tensor:
    """Per-pair base frequencies, fp32 [dim // 6].

    Follows ``models/dits/eraserdit_transformer.py:194-201``:
    ``theta ** linspace(log_theta(1), log_theta(theta), dim // 6) * pi / 2``.
    """
    freqs = theta ** torch.linspace(
        math.log(1.0, theta), math.log(theta, theta), dim // 6, dtype=torch.float32
    )
    return freqs * math.pi / 2.0


def video_coords(
    batch: int,
    frames: int,
    height: int,
    width: int,
    rope_interpolation_scale=None,
    base=ROPE_BASE,
    patch_size: int = 1,
    patch_size_t: int = 1,
) -> torch.Tensor:
    """Token coordinates [B, F*H*W, 3] (f, h, w), fp32.

    Follows ``models/dits/eraserdit_transformer.py:136-159``: integer grid,
    optionally multiplied by ``rope_interpolation_scale * patch / base`` per axis.
    """
    gf = torch.arange(frames, dtype=torch.float32)
    gh = torch.arange(height, dtype=torch.float32)
    gw = torch.arange(width, dtype=torch.float32)
    grid = torch.stack(torch.meshgrid(gf, gh, gw, indexing="ij"), dim=0)
    grid = grid.unsqueeze(0).repeat(batch, 1, 1, 1, 1)
    if rope_interpolation_scale is not None:
        grid[:, 0:1] = grid[:, 0:1] * rope_interpolation_scale[0] * patch_size_t / base[0]
        grid[:, 1:2] = grid[:, 1:2] * rope_interpolation_scale[1] * patch_size / base[1]
        grid[:, 2:3] = grid[:, 2:3] * rope_interpolation_scale[2] * patch_size / base[2]
    return grid.flatten(2, 4).transpose(1, 2)


def rope_table(
    batch: int,
    frames: int,
    height: int,
    width: int,
    dim: int = HIDDEN,
    rope_interpolation_scale=None,
    theta: float = ROPE_THETA,
) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [B, F*H*W, dim] fp32 exactly as ``LTXVideoRotaryPosEmbed.forward``.

    Follows ``models/dits/eraserdit_transformer.py:161-214``: angle =
    freq * (2 * coord - 1), ordered [..., freq, axis] and flattened, each value
    repeated for the (2i, 2i+1) channel pair; the first ``dim % 6`` channels
    carry cos = 1, sin = 0.
    """
    grid = video_coords(batch, frames, height, width, rope_interpolation_scale)
    freqs = rope_frequencies(dim, theta)
    freqs = freqs * (grid.unsqueeze(-1) * 2 - 1)
    freqs = freqs.transpose(-1, -2).flatten(2)
    cos = freqs.cos().repeat_interleave(2, dim=-1)
    sin = freqs.sin().repeat_interleave(2, dim=-1)
    if dim % 6 != 0:
        cos = torch.cat([torch.ones_like(cos[:, :, : dim % 6]), cos], dim=-1)
        sin = torch.cat([torch.zeros_like(cos[:, :, : dim % 6]), sin], dim=-1)
    return cos, sin


# ------------------------------------------------------------ QK RMSNorm/RoPE
def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """diffusers ``RMSNorm`` (elementwise affine, no bias) over the last dim.

    Follows ``layers/operator_fusion/triton/rmsnorm_native.py:25-43`` (the
    reference's statement of the exact rounding): fp32 mean of squares, rsqrt of
    (mean + eps), ``x * r`` in fp32, rounded to the weight's dtype when that is a
    16-bit float, then multiplied by the weight in that dtype.
    """
    variance = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
    y = x * torch.rsqrt(variance + eps)
    if weight is None:
        return y.to(x.dtype)
    if weight.dtype in (torch.float16, torch.bfloat16):
        y = y.to(weight.dtype)
    return y * weight


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Adjacent-pair RoPE; follows ``models/dits/eraserdit_attention.py:68-79``."""
    x_real, x_imag = x.unflatten(2, (-1, 2)).unbind(-1)
    x_rotated = torch.stack([-x_imag, x_real], dim=-1).flatten(2)
    return (x.float() * cos + x_rotated.float() * sin).to(x.dtype)


def qk_rmsnorm_rope(q, k, q_weight, k_weight, cos, sin, eps):
    """Unfused reference closure; follows ``eraserdit_attention.py:259-265``."""
    return (
        apply_rotary_emb(rms_norm(q, q_weight, eps), cos, sin),
        apply_rotary_emb(rms_norm(k, k_weight, eps), cos, sin),
    )


# --------------------------------------------------------------- attention
def sdpa_bshd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """``SDPAImpl.forward``: BSHD in/out, non-causal, no mask.

    Follows ``layers/attention/backends/sdpa.py:56-80``.
    """
    out = F.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
        attn_mask=None, dropout_p=0.0, is_causal=False, scale=scale,
    )
    return out.transpose(1, 2)


@dataclass
class LayerParams:
    """Weights of one ``attn1`` (``eraserdit_transformer.py:253-263``)."""

    wq: torch.Tensor
    bq: torch.Tensor
    wk: torch.Tensor
    bk: torch.Tensor
    wv: torch.Tensor
    bv: torch.Tensor
    wo: torch.Tensor
    bo: torch.Tensor
    norm_q: torch.Tensor
    norm_k: torch.Tensor
    eps: float

    def to(self, dtype=None, device=None) -> "LayerParams":
        kw = {}
        if dtype is not None:
            kw["dtype"] = dtype
        if device is not None:
            kw["device"] = device
        return LayerParams(
            *(getattr(self, n).to(**kw) for n in
              ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "norm_q", "norm_k")),
            eps=self.eps,
        )


def self_attention_layer(
    x: torch.Tensor,
    p: LayerParams,
    cos: torch.Tensor | None,
    sin: torch.Tensor | None,
    heads: int = HEADS,
    return_core: bool = False,
):
    """One DiT self-attention; follows ``EraserDiTAttentionProcessor.self_attn``
    (``models/dits/eraserdit_attention.py:242-290``) on the unfused SDPA path:
    QKV Linear, QK RMSNorm across heads, RoPE, BSHD view, SDPA with scale
    ``head_dim ** -0.5`` (``:141``), flatten heads, ``to_out[0]`` Linear
    (``:216-229``; ``to_out[1]`` is Dropout(0), the identity at inference).
    """
    q = F.linear(x, p.wq, p.bq)
    k = F.linear(x, p.wk, p.bk)
    v = F.linear(x, p.wv, p.bv)
    q = rms_norm(q, p.norm_q, p.eps)
    k = rms_norm(k, p.norm_k, p.eps)
    if cos is not None:
        q = apply_rotary_emb(q, cos, sin)
        k = apply_rotary_emb(k, cos, sin)
    qb, kb, vb = (t.unflatten(2, (heads, -1)) for t in (q, k, v))
    core = sdpa_bshd(qb, kb, vb, scale=qb.shape[-1] ** -0.5)
    out = F.linear(core.flatten(2, 3).to(q.dtype), p.wo, p.bo)
    if return_core:
        return out, core
    return out


def cross_attention_layer(x: torch.Tensor, enc: torch.Tensor, p: LayerParams,
                          bias: torch.Tensor | None = None, heads: int = HEADS) -> torch.Tensor:
    """``EraserDiTAttentionProcessor.cross_attn`` (``eraserdit_attention.py:292-332``):
    Q from ``x``, K/V from the text ``enc``, RMSNorm across heads on Q and K, no
    RoPE, SDPA with the additive text bias [B, 1, L] (``prepare_attention_mask``
    repeats it per head; ``:301-306``), ``to_out[0]``."""
    batch = x.shape[0]
    q = rms_norm(F.linear(x, p.wq, p.bq), p.norm_q, p.eps)
    k = rms_norm(F.linear(enc, p.wk, p.bk), p.norm_k, p.eps)
    v = F.linear(enc, p.wv, p.bv)
    qh, kh, vh = (t.unflatten(2, (heads, -1)).transpose(1, 2) for t in (q, k, v))
    mask = None if bias is None else bias.reshape(batch, 1, 1, -1).to(q.dtype)
    out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, dropout_p=0.0,
                                         is_causal=False)
    return F.linear(out.transpose(1, 2).flatten(2).to(q.dtype), p.wo, p.bo)


def layer_flops(batch: int, seq: int, hidden: int = HIDDEN, heads: int = HEADS,
                head_dim: int = HEAD_DIM) -> float:
    """Algorithmic FLOPs of one layer: 4 Linear GEMMs + the attention core."""
    return 4 * 2 * batch * seq * hidden * hidden + 4 * batch * heads * seq * seq * head_dim
