"""CPU restatement of the SageAttention-style FP8 attention the benchmark specifies.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Quantization (with the reference's K smoothing and V
scaling from ``layers/attention/backends/sage_peripheral.py:7-24,63,76-77``):

- K is smoothed by its mean over tokens per (batch, head, channel), the
  difference rounded to BF16 (``sage_peripheral.py:15-16``);
- Q and smoothed K are quantised to E4M3 with one scale per 128-token block
  (``amax / 448``; multiply by ``448 / amax``, round to nearest, saturate);
- V is quantised to E4M3 with one scale per (batch, head, channel) over all
  tokens (``amax / 448``);
- P = exp(S - rowmax) <= 1 is quantised to E4M3 after scaling by 448; the row
  sum uses the unquantised P; both products accumulate in FP32.

The Sage kernels themselves (SageAttention eb615cf, INT8 QK) are not
available here; their numerics are parity-unpinned in the reference too.  The
bar for this path is the north star's: cosine >= 0.995 against fp32 SDPA.
"""

from __future__ import annotations

import torch

E4M3_MAX = 448.0
BLOCK = 128


def e4m3(x: torch.Tensor) -> torch.Tensor:
    """Round to E4M3 (nearest even), saturating at +-448, back to fp32."""
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()


def _block_quant(x: torch.Tensor) -> torch.Tensor:
    """Per 128-token block quantise-dequantise of [B, S, H, D] (tokens dim 1)."""
    batch, seq, heads, dim = x.shape
    pad = (-seq) % BLOCK
    xp = torch.nn.functional.pad(x, (0, 0, 0, 0, 0, pad))
    xb = xp.view(batch, -1, BLOCK, heads, dim)
    amax = xb.abs().amax(dim=(2, 4), keepdim=True)
    safe = torch.where(amax > 0, amax, torch.full_like(amax, E4M3_MAX))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = e4m3(xb * (E4M3_MAX / safe)) * scale
    return q.view(batch, -1, heads, dim)[:, :seq]


def quantize(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Dequantised Q, smoothed K and V as the FP8 kernels see them (fp32 BSHD)."""
    qf, kf, vf = q.float(), k.float(), v.float()
    kmean = kf.mean(dim=1, keepdim=True)
    ks = (kf - kmean).bfloat16().float()
    qd = _block_quant(qf)
    kd = _block_quant(ks)
    vamax = vf.abs().amax(dim=1, keepdim=True)
    sv = torch.where(vamax > 0, vamax / E4M3_MAX, torch.ones_like(vamax))
    vd = e4m3(vf / sv) * sv
    return qd, kd, vd


def sage_fp8_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float
                       ) -> torch.Tensor:
    """FP8 attention on BSHD inputs (fp32 result); P quantised against the row max."""
    qd, kd, vd = quantize(q, k, v)
    qh, kh, vh = (t.transpose(1, 2) for t in (qd, kd, vd))
    s = (qh @ kh.transpose(-1, -2)) * scale
    p = torch.exp(s - s.amax(dim=-1, keepdim=True))
    l = p.sum(dim=-1, keepdim=True)
    p8 = e4m3(p * E4M3_MAX) / E4M3_MAX
    return ((p8 @ vh) / l).transpose(1, 2)
