"""FP8 (E4M3) shared QKV projection.

Mirrors ``SharedQKV`` / ``read_calibration`` (``layers/quantization/qkv_fp8.py:16-63``):
one round-to-nearest E4M3 quantisation of the activations with a static,
calibrated per-layer scale, and E4M3 weights with one scale per projection
(amax / 448).  The reference runs three ``scaled_mm`` calls; here the three
weights are concatenated into one [6144, 2048] E4M3 matrix with a per-column
scale vector (the activation scale times each projection's weight scale over
its 2048 columns), so that one tcgen05 E4M3 GEMM (``erd_linear_fp8``: FP32
accumulation, scale and bias in the epilogue, BF16 out) writes the
interleaved Q|K|V buffer the fused prologue reads.  The activation quantiser
is ``erd_quantize_e4m3``.
"""

from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

import torch

from . import _native

E4M3_MAX = 448.0


def read_calibration(path) -> tuple[dict, str]:
    """The reference's per-block QKV calibration file (28 completed layers)."""
    raw = Path(path).read_bytes()
    data = json.loads(raw)
    if (not data.get("completed") or not data.get("all_holdout_within_range")
            or len(data.get("layers", [])) != 28):
        raise ValueError("QKV calibration requires all 28 layers and completed holdout validation")
    for i, layer in enumerate(data["layers"]):
        scale = layer.get("scale")
        if (layer.get("block") != i or not isinstance(scale, (int, float))
                or not math.isfinite(scale) or scale <= 0):
            raise ValueError(f"invalid QKV scale at block {i}")
    return data, hashlib.sha256(raw).hexdigest()


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor E4M3 weight and its scale (``qkv_fp8.py:39-42``)."""
    wf = w.detach().float()
    maximum = wf.abs().amax()
    scale = torch.where(maximum > 0, maximum / E4M3_MAX, torch.ones_like(maximum))
    return (wf / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn), scale


def quantize_activation(x: torch.Tensor, scale: float, out: torch.Tensor | None = None
                        ) -> torch.Tensor:
    """E4M3 of BF16 ``x`` with the static scale (``erd_quantize_e4m3``)."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous() or x.numel() % 16:
        raise ValueError("FP8 QKV needs contiguous CUDA BF16 activations, numel % 16 == 0")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    lib = _native.load()
    with torch.cuda.device(x.device):
        rc = lib.erd_quantize_e4m3(x.data_ptr(), out.data_ptr(), x.numel(), float(scale),
                                   _native.stream_handle(x.device))
    _native.check(rc, "erd_quantize_e4m3")
    return out


class SharedQKV:
    """FP8 Q|K|V projection of one layer with a static activation scale."""

    def __init__(self, wq, bq, wk, bk, wv, bv, scale: float, device) -> None:
        device = torch.device(device)
        if not (isinstance(scale, (int, float)) and math.isfinite(scale) and scale > 0):
            raise ValueError("the activation scale must be a positive finite number")
        parts, scales = [], []
        for w in (wq, wk, wv):
            if tuple(w.shape) != (2048, 2048):
                raise ValueError("QKV FP8 requires 2048 x 2048 projections")
            q8, s = quantize_weight(w.to(device))
            parts.append(q8)
            scales.append(s)
        self.weight = torch.cat(parts).contiguous()  # [6144, 2048] E4M3
        self.weight_scales = torch.stack(scales)      # per projection
        self.scale_b = self.weight_scales.repeat_interleave(2048).view(1, -1).contiguous()
        # per output column: activation scale x the column's weight scale
        self.col_scale = (self.scale_b.view(-1) * float(scale)).float().contiguous()
        zero = torch.zeros(2048, device=device)
        self.bias = torch.cat([zero if b is None else b.to(device).float() for b in (bq, bk, bv)]
                              ).to(torch.bfloat16).contiguous()
        self.activation_scale = float(scale)
        self.device = device
        self.calls = 0

    @classmethod
    def from_attention_module(cls, attn, scale: float, device) -> "SharedQKV":
        return cls(attn.to_q.weight, attn.to_q.bias, attn.to_k.weight, attn.to_k.bias,
                   attn.to_v.weight, attn.to_v.bias, scale, device)

    def project(self, x: torch.Tensor) -> torch.Tensor:
        """[..., 2048] BF16 -> interleaved [..., 6144] BF16 (Q | K | V per token)."""
        rows = x.numel() // x.shape[-1]
        quant = quantize_activation(x.contiguous(), self.activation_scale).view(rows, 2048)
        y = torch.empty(rows, 6144, device=x.device, dtype=torch.bfloat16)
        if rows:
            lib = _native.load()
            with torch.cuda.device(x.device):
                rc = lib.erd_linear_fp8(quant.data_ptr(), 2048, self.weight.data_ptr(), 2048,
                                        self.col_scale.data_ptr(), self.bias.data_ptr(),
                                        y.data_ptr(), 6144, rows, 6144, 2048,
                                        _native.status_word(x.device).data_ptr(),
                                        _native.stream_handle(x.device))
            _native.check(rc, "erd_linear_fp8")
        self.calls += 1
        return y.view(*x.shape[:-1], 6144)

    def __call__(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The reference's interface: (q, k, v) views of the projected buffer."""
        y = self.project(x)
        return y[..., :2048], y[..., 2048:4096], y[..., 4096:]
