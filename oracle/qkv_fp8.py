"""CPU restatement of the FP8 shared QKV projection (test infrastructure only).

Follows ``SharedQKV`` (``layers/quantization/qkv_fp8.py:29-63``) and its
activation quantiser ``_quant_fp8_tensor`` (``layers/quantization/eraserdit_fp8.py:60-69``):
q = E4M3_RN(clamp(x / s, -448, 448)); weights E4M3 with scale amax / 448 per
projection; y = (q * s) @ (w8 * ws)^T + bias, accumulated in fp32, rounded to
BF16.  (The reference's ``use_fast_accum`` accumulation is restated as fp32.)
"""

from __future__ import annotations

import torch

E4M3_MAX = 448.0


def quantize_activation(x: torch.Tensor, scale: float) -> torch.Tensor:
    return (x.float() / scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)


def quantize_weight(w: torch.Tensor):
    wf = w.float()
    m = wf.abs().amax()
    s = m / E4M3_MAX if float(m) > 0 else torch.tensor(1.0)
    return (wf / s).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn), s


def shared_qkv(x: torch.Tensor, weights, biases, scale: float) -> torch.Tensor:
    """[..., 2048] -> [..., 6144] (Q | K | V), BF16."""
    xq = quantize_activation(x, scale).float() * scale
    outs = []
    for w, b in zip(weights, biases):
        w8, ws = quantize_weight(w)
        y = xq @ (w8.float() * ws).t()
        if b is not None:
            y = y + b.float()
        outs.append(y)
    return torch.cat(outs, dim=-1).to(torch.bfloat16)
