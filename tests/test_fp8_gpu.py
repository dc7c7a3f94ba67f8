"""FP8 (Sage-style E4M3) attention: north-star bar against fp32 SDPA, tighter
bar against the CPU restatement of the same quantization, segmented inputs,
the layer and the Ulysses path."""
import pytest
import torch

from oracle import sage_fp8
from tests.helpers import attention_fp32, cosine

pytestmark = pytest.mark.gpu

FP8_MIN_COSINE = 0.995  # north star: FP8 within cosine >= 0.995 of fp32 SDPA


def _inputs(batch, seq, heads, seed, amp=1.0, kshift=0.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda: torch.randn(batch, seq, heads, 64, generator=g, device="cuda") * amp
    q, k, v = mk(), mk(), mk()
    k = k + kshift  # a common offset along tokens: removed by the K smoothing
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


@pytest.mark.parametrize("batch,seq,heads,kshift", [(1, 128, 1, 0.0), (1, 129, 2, 0.0),
                                                    (2, 700, 3, 3.0), (1, 2049, 2, 0.0),
                                                    (1, 4096, 4, 1.0)])
def test_fp8_against_fp32_and_oracle(batch, seq, heads, kshift):
    from eraserdit_b200 import _native
    from eraserdit_b200.attention import AttentionMetadata, B200FP8AttentionImpl
    q, k, v = _inputs(batch, seq, heads, seed=seq, kshift=kshift)
    out = B200FP8AttentionImpl(heads, 64, 0.125).forward(q, k, v, AttentionMetadata())
    assert _native.read_status(q.device) == 0
    assert torch.isfinite(out).all()
    want = attention_fp32(q, k, v, 0.125)
    assert cosine(out, want) >= FP8_MIN_COSINE
    emulated = sage_fp8.sage_fp8_attention(q.cpu(), k.cpu(), v.cpu(), 0.125)
    assert cosine(out.cpu(), emulated) >= 0.999


def test_fp8_segmented_matches_contiguous():
    from eraserdit_b200.attention import _segmented_call, attention_bshd, fp8_workspace
    nseg, seg_len, batch, heads = 3, 300, 2, 2
    lens = [300, 299, 297]
    g = torch.Generator(device="cuda").manual_seed(4)
    recv = torch.zeros(nseg, seg_len, 3, batch, heads, 64, device="cuda", dtype=torch.bfloat16)
    for s, n in enumerate(lens):
        recv[s, :n] = torch.randn(n, 3, batch, heads, 64, generator=g, device="cuda").bfloat16()
    full = lambda i: torch.cat([recv[s, :n, i].permute(1, 0, 2, 3) for s, n in enumerate(lens)], 1)
    q, k, v = full(0), full(1), full(2)
    out = torch.zeros(nseg, seg_len, batch, heads, 64, device="cuda", dtype=torch.bfloat16)
    r = recv.view(-1)
    chunk = batch * heads * 64
    st = (3 * chunk, 64, heads * 64, seg_len * 3 * chunk)
    _segmented_call("erd_attn_fwd_fp8", r, r[chunk:], r[2 * chunk:], out, 0.125, batch=batch,
                    heads=heads, seg_len=seg_len, nseg=nseg, seg_lens=lens, q_strides=st,
                    k_strides=st, v_strides=st,
                    o_strides=(chunk, 64, heads * 64, seg_len * chunk),
                    extra=fp8_workspace(q.device, batch, heads, seg_len, nseg))
    got = torch.cat([out[s, :n].permute(1, 0, 2, 3) for s, n in enumerate(lens)], 1)
    want = attention_fp32(q, k, v, 0.125)
    assert cosine(got, want) >= FP8_MIN_COSINE
    contiguous = attention_bshd(q.contiguous(), k.contiguous(), v.contiguous(), 0.125,
                                precision="fp8")
    # different 128-token quantization blocks: two valid FP8 results, each within the bar
    assert cosine(got, contiguous) >= FP8_MIN_COSINE


def test_fp8_layer_and_ulysses():
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.ulysses import emulate_ranks
    from eraserdit_b200.synthetic import make_params
    p = make_params(5, 1e-6, device="cuda").to(torch.bfloat16)
    bf16 = EraserDiTSelfAttention.from_params(p, device="cuda")
    fp8 = EraserDiTSelfAttention.from_params(p, device="cuda", precision="fp8")
    rope = LTXVideoRotaryPosEmbed()(3, 8, 12)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, 288, 2048, generator=g, device="cuda").bfloat16()
    ref = bf16(x, rope)
    one = fp8(x, rope)
    assert cosine(one, ref) >= FP8_MIN_COSINE
    sp = torch.cat(emulate_ranks(fp8, 4, x, rope), dim=1)
    assert cosine(sp, ref) >= FP8_MIN_COSINE
    assert cosine(sp, one) >= FP8_MIN_COSINE
