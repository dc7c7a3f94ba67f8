"""FP8 shared QKV projection: the activation quantiser bit for bit and the
projection against the CPU restatement of the reference's SharedQKV, and the
layer with it against the BF16 layer."""
import pytest
import torch

from oracle import qkv_fp8 as oracle
from tests.helpers import cosine, max_abs

pytestmark = pytest.mark.gpu


def _weights(seed):
    g = torch.Generator().manual_seed(seed)
    ws = [torch.randn(2048, 2048, generator=g) * 0.02 for _ in range(3)]
    bs = [torch.randn(2048, generator=g) * 0.1 for _ in range(3)]
    return [w.bfloat16() for w in ws], [b.bfloat16() for b in bs]


def test_activation_quantiser_bitwise():
    from eraserdit_b200.qkv_fp8 import quantize_activation
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(3, 1000, 2048, generator=g) * 3).bfloat16()
    x[0, 0, :4] = torch.tensor([1e4, -1e4, 0.0, -0.0]).bfloat16()  # saturation and zeros
    scale = 0.0123
    got = quantize_activation(x.cuda(), scale).cpu()
    want = oracle.quantize_activation(x, scale)
    assert torch.equal(got.view(torch.uint8), want.view(torch.uint8))


def test_shared_qkv_against_restatement():
    from eraserdit_b200.qkv_fp8 import SharedQKV
    ws, bs = _weights(2)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 4096, 2048, generator=g).bfloat16()
    scale = float(x.float().abs().amax()) / 448
    qkv = SharedQKV(ws[0], bs[0], ws[1], bs[1], ws[2], bs[2], scale, "cuda")
    got = qkv.project(x.cuda()).float().cpu()
    want = oracle.shared_qkv(x, ws, bs, scale).float()
    assert cosine(got, want) >= 0.99999
    assert max_abs(got, want) <= 2e-2
    q, k, v = qkv(x.cuda())
    assert torch.equal(torch.cat([q, k, v], -1).cpu(), qkv.project(x.cuda()).cpu())
    # and against torch's scaled_mm on the same E4M3 operands (the reference's
    # product): both accumulate in fp32 and round once to BF16, so they differ
    # by at most about one BF16 rounding of the result (plus summation order
    # where the bias cancels the product)
    from eraserdit_b200.qkv_fp8 import quantize_activation
    xq = quantize_activation(x.cuda(), scale).view(-1, 2048)
    lib = torch._scaled_mm(xq, qkv.weight.t(),
                           scale_a=torch.full((xq.shape[0], 1), scale, device="cuda"),
                           scale_b=qkv.scale_b, bias=qkv.bias, out_dtype=torch.bfloat16).float()
    ours = qkv.project(x.cuda()).view(-1, 6144).float()
    assert bool(((ours - lib).abs() <= lib.abs() * 2.0 ** -7 + 2e-3).all())
    assert cosine(ours, lib) >= 0.99999


def test_layer_with_fp8_qkv():
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.synthetic import make_params
    p = make_params(4, 1e-6, device="cuda").to(torch.bfloat16)
    layer = EraserDiTSelfAttention.from_params(p, device="cuda")
    rope = LTXVideoRotaryPosEmbed()(4, 16, 24)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, 4 * 16 * 24, 2048, generator=g, device="cuda").bfloat16()
    want = layer(x, rope)
    layer.enable_qkv_fp8(float(x.float().abs().amax()) / 448, p.wq, p.bq, p.wk, p.bk, p.wv, p.bv)
    got = layer(x, rope)
    assert layer.qkv_fp8.calls == 1
    assert cosine(got, want) >= 0.995  # E4M3 activations and weights in the projection
