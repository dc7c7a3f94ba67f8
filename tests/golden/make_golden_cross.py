"""Golden fixtures for the cross-attention (``attn2``) path, from the reference.

    python tests/golden/make_golden_cross.py /path/to/reference

Runs ``EraserDiTAttentionProcessor.cross_attn`` through the processor's
``__call__`` on the CPU in fp32 behind the diffusers stub of ``make_golden.py``.
The stub attention module restates diffusers' ``Attention.prepare_attention_mask``
for an unpadded mask (repeat the [B, 1, L] bias once per head on dim 0).
Inputs: configuration-0 weights and hidden states, 24 seeded text tokens with an
end-padded mask per batch entry converted to the reference's -10000 bias.
Writes ``cross_golden.npz`` (selected rows and checksums).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from make_golden import DiffusersRMSNorm, checksums, install_diffusers_stub, rows  # noqa: E402

from eraserdit_b200.synthetic import CONFIG0, LayerConfig, make_hidden, make_params  # noqa: E402

TEXT_TOKENS = 24
TEXT_VALID = (17, 9)  # attended prefix per batch entry


def cross_inputs():
    """Batch-2 configuration-0 layer inputs plus the text tokens and bias."""
    cfg = LayerConfig(**{**CONFIG0.__dict__, "batch": 2})
    p = make_params(cfg.seed, cfg.eps, random_norm_weight=True)
    x = make_hidden(cfg)
    g = torch.Generator().manual_seed(55)
    enc = torch.randn(cfg.batch, TEXT_TOKENS, 2048, generator=g)
    keep = torch.zeros(cfg.batch, TEXT_TOKENS)
    for b, n in enumerate(TEXT_VALID):
        keep[b, :n] = 1
    bias = ((1 - keep) * -10000.0).unsqueeze(1)  # eraserdit_transformer.py:484-487
    return cfg, p, x, enc, keep, bias


def main(reference: Path) -> None:
    install_diffusers_stub()
    sys.path.insert(0, str(reference))
    from models.dits.eraserdit_attention import EraserDiTAttentionProcessor

    cfg, p, x, enc, keep, bias = cross_inputs()
    attn = torch.nn.Module()
    attn.heads = 32
    attn.to_q, attn.to_k, attn.to_v = (torch.nn.Linear(2048, 2048) for _ in range(3))
    attn.to_out = torch.nn.ModuleList([torch.nn.Linear(2048, 2048), torch.nn.Dropout(0.0)])
    attn.norm_q = DiffusersRMSNorm(2048, eps=p.eps)
    attn.norm_k = DiffusersRMSNorm(2048, eps=p.eps)
    with torch.no_grad():
        for lin, w, b in ((attn.to_q, p.wq, p.bq), (attn.to_k, p.wk, p.bk),
                          (attn.to_v, p.wv, p.bv), (attn.to_out[0], p.wo, p.bo)):
            lin.weight.copy_(w)
            lin.bias.copy_(b)
        attn.norm_q.weight.copy_(p.norm_q)
        attn.norm_k.weight.copy_(p.norm_k)

    def prepare_attention_mask(mask, target_length, batch_size, out_dim=3):
        # diffusers Attention.prepare_attention_mask for current length == target
        assert mask.shape[-1] == target_length and out_dim == 3
        return mask.repeat_interleave(attn.heads, dim=0)

    attn.prepare_attention_mask = prepare_attention_mask
    processor = EraserDiTAttentionProcessor(attention_backend="sdpa")
    with torch.no_grad():
        out = processor(attn.eval(), x, encoder_hidden_states=enc, attention_mask=bias)
    result = {"cross0_fp32_rows": rows(out)}
    for key, value in checksums(out).items():
        result[f"cross0_fp32_{key}"] = np.asarray(value)
    np.savez_compressed(HERE / "cross_golden.npz", **result)
    print("wrote", HERE / "cross_golden.npz", tuple(out.shape))


if __name__ == "__main__":
    main(Path(sys.argv[1]))
