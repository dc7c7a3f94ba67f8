"""Seeded synthetic inputs for the benchmark configurations.

The reference quotes its numbers on real videos; these generators stand in for
them with the shapes and distributions the benchmark configurations name:
hidden states N(0, 1), Linear weights N(0, 0.02) with zero bias, RMSNorm
weight 1 (or a random affine weight for stricter parity cases), on the latent
grid F x H x W.  The benchmark and the tests draw from the same generators.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

HIDDEN = 2048


@dataclass(frozen=True)
class LayerConfig:
    batch: int
    frames: int
    height: int
    width: int
    eps: float = 1e-6
    seed: int = 0
    random_norm_weight: bool = False

    @property
    def seq(self) -> int:
        return self.frames * self.height * self.width


CONFIG0 = LayerConfig(batch=1, frames=2, height=8, width=12, eps=1e-6, seed=0)
CONFIG1 = LayerConfig(batch=2, frames=16, height=34, width=60, eps=1e-6, seed=1)


@dataclass
class LayerWeights:
    """Weights of one ``attn1`` (``to_q/to_k/to_v``, ``to_out[0]``, ``norm_q/norm_k``)."""

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

    def to(self, dtype=None, device=None) -> "LayerWeights":
        kw = {}
        if dtype is not None:
            kw["dtype"] = dtype
        if device is not None:
            kw["device"] = device
        return LayerWeights(
            *(getattr(self, n).to(**kw) for n in
              ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "norm_q", "norm_k")),
            eps=self.eps,
        )


def make_params(seed: int, eps: float, random_norm_weight: bool = False,
                hidden: int = HIDDEN, device="cpu") -> LayerWeights:
    """fp32 weights N(0, 0.02), zero biases, unit (or U(0.2, 1.8)) norm weights."""
    g = torch.Generator(device=device).manual_seed(seed + 1000)
    w = [torch.randn(hidden, hidden, generator=g, device=device) * 0.02 for _ in range(4)]
    zeros = [torch.zeros(hidden, device=device) for _ in range(4)]
    if random_norm_weight:
        nq = torch.rand(hidden, generator=g, device=device) * 1.6 + 0.2
        nk = torch.rand(hidden, generator=g, device=device) * 1.6 + 0.2
    else:
        nq = torch.ones(hidden, device=device)
        nk = torch.ones(hidden, device=device)
    return LayerWeights(w[0], zeros[0], w[1], zeros[1], w[2], zeros[2], w[3], zeros[3],
                        nq, nk, eps)


def make_hidden(cfg: LayerConfig, hidden: int = HIDDEN, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(cfg.seed)
    return torch.randn(cfg.batch, cfg.seq, hidden, generator=g, device=device)
