"""Cross-attention of the EraserDiT block (``attn2``) on the B200 kernels.

Follows ``EraserDiTAttentionProcessor.cross_attn``
(``models/dits/eraserdit_attention.py:292-332``): Q from the video tokens, K
and V from the text tokens, RMSNorm across heads on Q and on K (no RoPE),
attention with the text padding mask, ``to_out[0]``.  The reference applies
the mask as the additive bias ``(1 - mask) * -10000``
(``eraserdit_transformer.py:484-487``), which gives the padded keys a weight of
exactly 0 in fp32; here the mask becomes each batch entry's count of attended
keys (the mask must be a prefix of ones, as the text encoder's end padding
produces) and the kernel skips the rest.

``apply_fused_cross_q_rmsnorm`` mirrors
``layers/operator_fusion/cross_q_rmsnorm.py:33-49`` (capability reasons,
``RuntimeError`` in forced mode, no fallback).
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch

from . import _native
from .layer import HEAD_DIM, HIDDEN
from .linear import linear_bf16

CROSS_Q_RMSNORM_NATIVE_OP = "cross_q_rmsnorm_native"


def _norm_failure(query: torch.Tensor, norm: Any) -> str | None:
    """The reference's capability reasons (``cross_q_rmsnorm.py:9-30``)."""
    if query.ndim != 3 or query.shape[-1] != 2048 or query.numel() == 0:
        return "query_shape"
    if not query.is_cuda or query.dtype != torch.bfloat16:
        return "query_device_dtype"
    if not query.is_contiguous():
        return "query_layout"
    weight = getattr(norm, "weight", None)
    if weight is None or tuple(weight.shape) != (2048,) or getattr(norm, "bias", None) is not None:
        return "norm_affine"
    if weight.dtype != torch.bfloat16 or weight.device != query.device or not weight.is_contiguous():
        return "weight_device_dtype_layout"
    return None


def rms_norm_rows(x: torch.Tensor, weight: torch.Tensor | None, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """diffusers RMSNorm across all 2048 channels of each row of [B, S, 2048]
    (``erd_qk_norm_rope`` with Q alone)."""
    batch, tokens, hidden = x.shape
    if out is None:
        out = torch.empty_like(x)
    lib = _native.load()
    with torch.cuda.device(x.device):
        rc = lib.erd_qk_norm_rope(
            x.data_ptr(), None, None, x.stride(1), x.stride(0), batch, tokens, hidden,
            _native.ptr(weight), None, float(eps), 0, None, None, 0, 0, None, 0, 0, 0, 0, 0, None,
            out.data_ptr(), None, None, out.stride(1), out.stride(0), HEAD_DIM, 32, 0,
            _native.stream_handle(x.device))
    _native.check(rc, "erd_qk_norm_rope (query only)")
    return out


def apply_fused_cross_q_rmsnorm(query: torch.Tensor, norm: Any, *, decision: Any = None
                                ) -> torch.Tensor:
    failure = _norm_failure(query, norm)
    if failure is not None:
        raise RuntimeError(f"forced {CROSS_Q_RMSNORM_NATIVE_OP} capability check failed: {failure}")
    return rms_norm_rows(query, norm.weight, float(norm.eps))


def mask_lengths(attention_mask: torch.Tensor | None, batch: int, kv_len: int) -> list[int] | None:
    """Attended key count per batch entry from a [B, L] keep-mask (1 / 0) or the
    reference's additive [B, 1, L] bias (0 / -10000); the kept keys must be a prefix."""
    if attention_mask is None:
        return None
    additive = attention_mask.dim() == 3  # the reference's [B, 1, L] bias; [B, L] keep-mask
    m = attention_mask.reshape(batch, -1).float()
    if m.shape[1] != kv_len:
        raise ValueError("the text mask must cover every key")
    keep = (m > -0.5) if additive else (m > 0.5)
    counts = keep.sum(dim=1)
    ar = torch.arange(kv_len, device=keep.device)
    if not bool((keep == (ar[None] < counts[:, None])).all()):
        raise ValueError("the b200 cross-attention supports end-padded text masks only")
    if bool((counts == 0).any()):
        raise ValueError("every batch entry needs at least one unmasked text token")
    return [int(c) for c in counts.tolist()]


def cross_attention_bshd(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                         softmax_scale: float, kv_valid: list[int] | None = None,
                         out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(Q K^T * scale) V with [B, Sq, H, 64] queries and [B, Skv, H, 64]
    keys/values; batch entry b attends its first kv_valid[b] keys."""
    batch, q_len, heads, dim = query.shape
    kv_len = key.shape[1]
    if key.shape != value.shape or key.shape[0] != batch or key.shape[2] != heads or dim != 64:
        raise ValueError("cross-attention needs BSHD queries and equal-shape keys/values")
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    lens = None if kv_valid is None else (ctypes.c_int32 * batch)(*kv_valid)
    lib = _native.load()
    st = lambda t: (t.stride(1), t.stride(2), t.stride(0))
    with torch.cuda.device(query.device):
        rc = lib.erd_attn_fwd_cross_bf16(
            query.data_ptr(), key.data_ptr(), value.data_ptr(), *st(query), *st(key), *st(value),
            batch, heads, q_len, kv_len, lens, 64, float(softmax_scale), out.data_ptr(), *st(out),
            _native.status_word(query.device).data_ptr(), _native.stream_handle(query.device))
    _native.check(rc, "erd_attn_fwd_cross_bf16")
    return out


class EraserDiTCrossAttention:
    """``attn2`` of a block: video queries against text keys/values."""

    def __init__(self, wq, bq, wk, bk, wv, bv, wo, bo, norm_q, norm_k, eps: float,
                 device="cuda", heads: int = 32) -> None:
        device = torch.device(device)
        kw = dict(device=device, dtype=torch.bfloat16)
        lin = lambda w, b: (w.to(**kw).contiguous(), None if b is None else b.to(**kw).contiguous())
        self.wq, self.bq = lin(wq, bq)
        self.w_kv = torch.cat([wk, wv]).to(**kw).contiguous()
        zero = torch.zeros(HIDDEN)
        self.b_kv = torch.cat([zero if b is None else b.float().cpu() for b in (bk, bv)]).to(**kw)
        self.wo, self.bo = lin(wo, bo)
        self.norm_q = None if norm_q is None else norm_q.to(**kw).contiguous()
        self.norm_k = None if norm_k is None else norm_k.to(**kw).contiguous()
        self.eps = float(eps)
        self.heads = heads
        self.scale = HEAD_DIM ** -0.5

    @classmethod
    def from_params(cls, p, device="cuda") -> "EraserDiTCrossAttention":
        return cls(p.wq, p.bq, p.wk, p.bk, p.wv, p.bv, p.wo, p.bo, p.norm_q, p.norm_k, p.eps,
                   device=device)

    def forward(self, hidden_states: torch.Tensor, encoder_hidden_states: torch.Tensor,
                attention_mask: torch.Tensor | None = None) -> torch.Tensor:
        batch, q_len, _ = hidden_states.shape
        kv_len = encoder_hidden_states.shape[1]
        kv_valid = mask_lengths(attention_mask, batch, kv_len)
        q = rms_norm_rows(linear_bf16(hidden_states, self.wq, self.bq), self.norm_q, self.eps)
        kvp = linear_bf16(encoder_hidden_states, self.w_kv, self.b_kv)  # [B, L, 4096]
        k = rms_norm_rows(kvp[..., :HIDDEN].contiguous(), self.norm_k, self.eps)
        v = kvp[..., HIDDEN:]
        heads4 = lambda t: t.unflatten(2, (self.heads, HEAD_DIM))
        core = cross_attention_bshd(heads4(q), heads4(k), heads4(v), self.scale, kv_valid)
        return linear_bf16(core.flatten(2), self.wo, self.bo)

    __call__ = forward
