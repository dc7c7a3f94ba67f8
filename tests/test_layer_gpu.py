"""Whole self-attention layer: CUDA path vs the reference's fp32 result."""
import numpy as np
import pytest
import torch

from oracle import reference_path as ref
from eraserdit_b200.synthetic import CONFIG0, CONFIG1, LayerConfig, make_hidden, make_params
from tests.helpers import attention_fp32, cosine, max_abs

pytestmark = pytest.mark.gpu

ROWS = list(range(0, 192, 24)) + [191]


def _layer(params):
    from eraserdit_b200.layer import EraserDiTSelfAttention
    return EraserDiTSelfAttention.from_params(params.to(torch.bfloat16), device="cuda")


def _rope(cfg):
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    return LTXVideoRotaryPosEmbed()(cfg.frames, cfg.height, cfg.width)


@pytest.mark.parametrize("random_norm", [False, True])
def test_config0_against_fp32_oracle(golden, random_norm):
    cfg = LayerConfig(**{**CONFIG0.__dict__, "random_norm_weight": random_norm})
    p = make_params(cfg.seed, cfg.eps, random_norm_weight=random_norm)
    x = make_hidden(cfg)
    # fp32 oracle on the BF16-representable inputs the CUDA path consumes
    p16 = p.to(torch.bfloat16).to(torch.float32)
    cos, sin = ref.rope_table(1, cfg.frames, cfg.height, cfg.width)
    with torch.no_grad():
        want = ref.self_attention_layer(x.bfloat16().float(), p16, cos, sin)
    got = _layer(p)(x.bfloat16().cuda(), _rope(cfg)).float().cpu()
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.9999
    if not random_norm:
        # and against the reference processor's own fp32 output (fp32 weights)
        gold = torch.from_numpy(golden["layer0_fp32_rows"])
        assert cosine(got[:, ROWS], gold) >= 0.999


def test_config1_full_size_against_fp32_gpu():
    """2 x 32640 tokens: compare with an fp32 GPU evaluation of the same math."""
    cfg = CONFIG1
    p = make_params(cfg.seed, cfg.eps, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(cfg.seed)
    x = torch.randn(cfg.batch, cfg.seq, 2048, generator=g, device="cuda").bfloat16()
    rope = _rope(cfg)
    layer = _layer(p)
    got = layer(x, rope)
    # fp32 reference on the BF16 weights / inputs, same RoPE table
    p16 = p.to(torch.bfloat16).to(torch.float32)
    cos, sin = rope.full(cfg.batch)
    with torch.no_grad():
        xf = x.float()
        q = ref.apply_rotary_emb(ref.rms_norm(torch.nn.functional.linear(xf, p16.wq, p16.bq),
                                              p16.norm_q, cfg.eps), cos, sin)
        k = ref.apply_rotary_emb(ref.rms_norm(torch.nn.functional.linear(xf, p16.wk, p16.bk),
                                              p16.norm_k, cfg.eps), cos, sin)
        v = torch.nn.functional.linear(xf, p16.wv, p16.bv)
        core = attention_fp32(q.unflatten(2, (32, 64)), k.unflatten(2, (32, 64)),
                              v.unflatten(2, (32, 64)), 0.125)
        want = torch.nn.functional.linear(core.flatten(2), p16.wo, p16.bo)
    assert torch.isfinite(got).all()
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.9999
