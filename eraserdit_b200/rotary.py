"""LTX 3D rotary embedding in factored (per-axis) form.

Mirrors ``LTXVideoRotaryPosEmbed`` (``models/dits/eraserdit_transformer.py:115-214``,
instantiated at ``:402-410`` with dim 2048, base (20, 2048, 2048), theta 1e4).
The reference materialises cos/sin tables of shape [B, F*H*W, 2048] in fp32
(267 MB each at 2 x 32640 tokens).  Every entry is cos/sin of
``freq[k] * (2 * coord_axis - 1)`` for one of three axes, so the same values
are stored here once per (axis, coordinate, frequency): (F + H + W) * 341
float2 entries (300 KB at 16 x 34 x 60), built on the device by
``erd_rope_axis_table`` and read by the fused QK-norm/RoPE kernel.

The 341 base frequencies are computed with the reference's own torch
expression (``:194-201``) on the host, once per table, so that they are
bit-identical to the reference's; all per-token work runs on the device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _native


def base_frequencies(dim: int = 2048, theta: float = 10000.0) -> torch.Tensor:
    """``theta ** linspace(log_theta(1), log_theta(theta), dim // 6) * pi / 2`` (fp32)."""
    freqs = theta ** torch.linspace(math.log(1.0, theta), math.log(theta, theta), dim // 6,
                                    dtype=torch.float32)
    return freqs * math.pi / 2.0


@dataclass
class RopeAxisTable:
    """Device table of (cos, sin) per (axis, coordinate, frequency)."""

    table: torch.Tensor  # float32 [(F + H + W) * nfreq * 2]
    frames: int
    height: int
    width: int
    nfreq: int
    # Optional device int32 [F*H*W]: grid position (f*H*W + h*W + w) of the
    # token at each sequence position, when tokens are not in raster order.
    grid_index: torch.Tensor | None = None

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    def in_order(self, grid_index: torch.Tensor) -> "RopeAxisTable":
        """The same table for a sequence laid out in another token order."""
        index = grid_index.to(device=self.table.device, dtype=torch.int32).contiguous()
        if index.numel() != self.tokens:
            raise ValueError("grid_index needs one entry per token")
        return RopeAxisTable(self.table, self.frames, self.height, self.width, self.nfreq, index)

    def full(self, batch: int = 1, dim: int = 2048) -> tuple[torch.Tensor, torch.Tensor]:
        """Expand to the reference's [B, F*H*W, dim] cos/sin tables (for tests and
        for callers of the table-based fusion interface)."""
        t = self.table.view(-1, 2)
        nf, dev = self.nfreq, self.table.device
        f = torch.arange(self.frames, device=dev).repeat_interleave(self.height * self.width)
        h = torch.arange(self.height, device=dev).repeat_interleave(self.width).repeat(self.frames)
        w = torch.arange(self.width, device=dev).repeat(self.frames * self.height)
        k = torch.arange(nf, device=dev)
        base = torch.tensor([0, self.frames * nf, (self.frames + self.height) * nf], device=dev)
        coords = torch.stack([f, h, w], dim=-1)  # [S, 3]
        idx = base.view(1, 1, 3) + coords.view(-1, 1, 3) * nf + k.view(1, nf, 1)  # [S, nf, 3]
        vals = t[idx.flatten(1)]  # [S, nf*3, 2]
        cos = vals[..., 0].repeat_interleave(2, dim=-1)
        sin = vals[..., 1].repeat_interleave(2, dim=-1)
        pad = dim % 6
        if pad:
            cos = torch.cat([torch.ones_like(cos[:, :pad]), cos], dim=-1)
            sin = torch.cat([torch.zeros_like(sin[:, :pad]), sin], dim=-1)
        if self.grid_index is not None:
            idx = self.grid_index.long().to(cos.device)
            cos, sin = cos[idx], sin[idx]
        return (cos.unsqueeze(0).expand(batch, -1, -1).contiguous(),
                sin.unsqueeze(0).expand(batch, -1, -1).contiguous())


class LTXVideoRotaryPosEmbed:
    """Drop-in for the reference class's constructor; ``forward`` returns a
    :class:`RopeAxisTable` instead of the two dense tables."""

    def __init__(self, dim: int = 2048, base_num_frames: int = 20, base_height: int = 2048,
                 base_width: int = 2048, patch_size: int = 1, patch_size_t: int = 1,
                 theta: float = 10000.0) -> None:
        if dim != 2048:
            raise ValueError("the fused QK-norm/RoPE kernel supports dim 2048 (32 x 64 heads)")
        self.dim = dim
        self.base_num_frames = base_num_frames
        self.base_height = base_height
        self.base_width = base_width
        self.patch_size = patch_size
        self.patch_size_t = patch_size_t
        self.theta = theta
        self._freqs: dict[torch.device, torch.Tensor] = {}

    def freqs(self, device: torch.device) -> torch.Tensor:
        cached = self._freqs.get(device)
        if cached is None:
            cached = base_frequencies(self.dim, self.theta).to(device)
            self._freqs[device] = cached
        return cached

    def forward(self, num_frames: int, height: int, width: int,
                rope_interpolation_scale=None, device: torch.device | str = "cuda") -> RopeAxisTable:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("the RoPE axis table is built on a CUDA device")
        lib = _native.load()
        freqs = self.freqs(device)
        nfreq = freqs.numel()
        table = torch.empty((num_frames + height + width) * nfreq * 2, dtype=torch.float32,
                            device=device)
        if rope_interpolation_scale is None:
            scale = (1.0, 1.0, 1.0)
            use_scale = 0
        else:
            scale = tuple(float(s) for s in rope_interpolation_scale)
            use_scale = 1
        with torch.cuda.device(device):
            rc = lib.erd_rope_axis_table(
                freqs.data_ptr(), nfreq, num_frames, height, width, use_scale, scale[0], scale[1],
                scale[2], float(self.patch_size_t), float(self.patch_size),
                float(self.base_num_frames), float(self.base_height), float(self.base_width),
                table.data_ptr(), _native.stream_handle(device))
        _native.check(rc, "erd_rope_axis_table")
        return RopeAxisTable(table, num_frames, height, width, nfreq)

    __call__ = forward
