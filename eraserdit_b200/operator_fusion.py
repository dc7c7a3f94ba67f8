"""QK RMSNorm + RoPE fusion op, mirroring the reference's public dispatch.

``apply_fused_qk_rmsnorm_rope`` keeps the reference signature
(``layers/operator_fusion/qk_rmsnorm_rope.py:80-89``) and its capability
reasons (``:18-77``), and returns what the reference closure returns
(``models/dits/eraserdit_attention.py:259-265``).  Unlike the reference there
is no fallback to the closure: an unsupported input raises ``RuntimeError``,
which is the reference's forced-mode behaviour (``:117-121``).
"""

from __future__ import annotations

from typing import Any

import torch

from . import _native
from .rotary import RopeAxisTable

QK_RMSNORM_ROPE_OP = "qk_rmsnorm_rope"
_WIDTH = 2048


def _norm_weight(norm: Any) -> torch.Tensor | None:
    return getattr(norm, "weight", None)


def capability_failure(query, key, query_norm, key_norm, freqs) -> str | None:
    """Reference reason strings for an unsupported call (``qk_rmsnorm_rope.py:18-77``),
    without the eps pin: eps is a kernel argument here (1e-5 and 1e-6 are both used)."""
    if freqs is None:
        return "rotary_missing"
    table_mode = isinstance(freqs, RopeAxisTable)
    if not table_mode and (not isinstance(freqs, tuple) or len(freqs) != 2):
        return "rotary_contract"
    if not isinstance(query, torch.Tensor) or not isinstance(key, torch.Tensor):
        return "tensor_contract"
    if query.ndim != 3 or key.shape != query.shape:
        return "qk_shape"
    if query.shape[-1] != _WIDTH:
        return "hidden_width"
    if query.dtype != torch.bfloat16 or key.dtype != torch.bfloat16:
        return "qk_dtype"
    if not query.is_cuda or query.device != key.device:
        return "qk_device"
    if query.stride(-1) != 1 or key.stride(-1) != 1 or query.stride() != key.stride():
        return "qk_layout"
    if table_mode:
        if freqs.table.device != query.device:
            return "rotary_device"
        if freqs.tokens != query.shape[1]:
            return "rotary_shape"
    else:
        cos, sin = freqs
        if not isinstance(cos, torch.Tensor) or not isinstance(sin, torch.Tensor):
            return "tensor_contract"
        if cos.shape != query.shape or sin.shape != query.shape:
            return "rotary_shape"
        if cos.dtype != torch.float32 or sin.dtype != torch.float32:
            return "rotary_dtype"
        if cos.device != query.device or sin.device != query.device:
            return "rotary_device"
        if not cos.is_contiguous() or not sin.is_contiguous():
            return "rotary_layout"
    for norm in (query_norm, key_norm):
        weight = _norm_weight(norm)
        if weight is not None:
            if weight.shape != (_WIDTH,):
                return "norm_weight_shape"
            if weight.dtype != torch.bfloat16:
                return "norm_weight_dtype"
            if weight.device != query.device:
                return "norm_weight_device"
            if not weight.is_contiguous():
                return "norm_weight_layout"
    if getattr(query_norm, "bias", None) is not None or getattr(key_norm, "bias", None) is not None:
        return "norm_bias"
    qe = float(getattr(query_norm, "eps", float("nan")))
    ke = float(getattr(key_norm, "eps", float("nan")))
    if qe != ke or not qe > 0:
        return "norm_epsilon"
    return None


def qk_norm_rope_into(query, key, q_weight, k_weight, eps, freqs, q_out, k_out,
                      *, value=None, v_out=None, token_offset: int = 0,
                      out_token_stride=None, out_batch_stride=None, out_head_stride=64,
                      heads_per_dest: int = 32, out_dest_stride: int = 0) -> None:
    """Enqueue ``erd_qk_norm_rope`` with explicit output addressing (see the header)."""
    lib = _native.load()
    batch, tokens, hidden = query.shape
    out_token_stride = q_out.stride(1) if out_token_stride is None else out_token_stride
    out_batch_stride = q_out.stride(0) if out_batch_stride is None else out_batch_stride
    grid_index = None
    if isinstance(freqs, RopeAxisTable):
        mode, cos, sin, tts, tbs = 2, None, None, 0, 0
        axis, nfreq, gf, gh, gw = freqs.table, freqs.nfreq, freqs.frames, freqs.height, freqs.width
        grid_index = freqs.grid_index
    elif freqs is None:
        mode, cos, sin, tts, tbs = 0, None, None, 0, 0
        axis, nfreq, gf, gh, gw = None, 0, 0, 0, 0
    else:
        cos, sin = freqs
        mode, tts, tbs = 1, cos.stride(1), cos.stride(0)
        axis, nfreq, gf, gh, gw = None, 0, 0, 0, 0
    device = query.device
    with torch.cuda.device(device):
        rc = lib.erd_qk_norm_rope(
            query.data_ptr(), key.data_ptr(), _native.ptr(value),
            query.stride(1), query.stride(0), batch, tokens, hidden,
            _native.ptr(q_weight), _native.ptr(k_weight), float(eps), mode,
            _native.ptr(cos), _native.ptr(sin), tts, tbs, _native.ptr(axis), nfreq, gf, gh, gw,
            int(token_offset), _native.ptr(grid_index), q_out.data_ptr(), k_out.data_ptr(),
            _native.ptr(v_out),
            out_token_stride, out_batch_stride, out_head_stride, heads_per_dest, out_dest_stride,
            _native.stream_handle(device))
    _native.check(rc, "erd_qk_norm_rope")


def qk_norm_rope_peer_into(query, key, value, q_weight, k_weight, eps, freqs, dest_bases,
                           k_offset: int, v_offset: int, *, token_offset: int,
                           out_token_stride: int, out_batch_stride: int, out_head_stride: int,
                           heads_per_dest: int) -> None:
    """Enqueue ``erd_qk_norm_rope_peer``: head group g of every token is stored
    at device address ``dest_bases[g]`` (another rank's receive buffer)."""
    import ctypes
    lib = _native.load()
    batch, tokens, hidden = query.shape
    if not isinstance(freqs, RopeAxisTable):
        raise ValueError("the peer prologue takes a RopeAxisTable")
    bases = (ctypes.c_void_p * len(dest_bases))(*dest_bases)
    device = query.device
    with torch.cuda.device(device):
        rc = lib.erd_qk_norm_rope_peer(
            query.data_ptr(), key.data_ptr(), _native.ptr(value), query.stride(1),
            query.stride(0), batch, tokens, hidden, _native.ptr(q_weight), _native.ptr(k_weight),
            float(eps), 2, None, None, 0, 0, freqs.table.data_ptr(), freqs.nfreq, freqs.frames,
            freqs.height, freqs.width, int(token_offset), _native.ptr(freqs.grid_index), bases,
            len(dest_bases), int(k_offset), int(v_offset), out_token_stride, out_batch_stride,
            out_head_stride, heads_per_dest, _native.stream_handle(device))
    _native.check(rc, "erd_qk_norm_rope_peer")


def apply_fused_qk_rmsnorm_rope(query: torch.Tensor, key: torch.Tensor, query_norm: Any,
                                key_norm: Any, freqs, *, decision: Any = None,
                                reference: Any = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused ``rope(norm_q(q)), rope(norm_k(k))`` on [B, S, 2048] BF16.

    ``freqs`` is the reference's ``(cos, sin)`` pair of fp32 [B, S, 2048]
    tables or a :class:`RopeAxisTable`.  ``decision`` and ``reference`` are
    accepted for signature compatibility; there is no fallback.
    """
    del decision, reference
    failure = capability_failure(query, key, query_norm, key_norm, freqs)
    if failure is not None:
        raise RuntimeError(f"forced {QK_RMSNORM_ROPE_OP} capability check failed: {failure}")
    q_out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    k_out = torch.empty(key.shape, dtype=key.dtype, device=key.device)
    qk_norm_rope_into(query, key, _norm_weight(query_norm), _norm_weight(key_norm),
                      float(query_norm.eps), freqs, q_out, k_out)
    return q_out, k_out
