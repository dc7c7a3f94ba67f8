"""Cross-attention (attn2): the oracle against the reference's own output
(golden), the text-mask handling on the host, and (GPU) the kernel and module
against fp32."""
from pathlib import Path
import sys

import numpy as np
import pytest
import torch

from oracle import reference_path as ref
from tests.helpers import cosine, max_abs

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from make_golden_cross import cross_inputs  # noqa: E402

ROWS = list(range(0, 192, 24)) + [191]


def test_oracle_matches_reference_cross_attn():
    g = np.load(GOLDEN / "cross_golden.npz")
    cfg, p, x, enc, keep, bias = cross_inputs()
    with torch.no_grad():
        out = ref.cross_attention_layer(x, enc, p, bias)
    # fp32 on another host CPU differs in the last bits (BLAS paths): 5e-6 on values ~0.5
    np.testing.assert_allclose(out[:, ROWS].numpy(), g["cross0_fp32_rows"], rtol=0, atol=5e-6)
    np.testing.assert_allclose(out.double().square().sum(-1).numpy(),
                               g["cross0_fp32_token_sumsq"], rtol=1e-5)


def test_mask_lengths():
    from eraserdit_b200.cross_attention import mask_lengths
    keep = torch.tensor([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1]], dtype=torch.float32)
    assert mask_lengths(keep, 2, 5) == [3, 5]
    bias = ((1 - keep) * -10000.0).unsqueeze(1)  # the reference's additive form
    assert mask_lengths(bias, 2, 5) == [3, 5]
    assert mask_lengths(torch.zeros(2, 1, 5), 2, 5) == [5, 5]  # additive, nothing padded
    assert mask_lengths(None, 2, 5) is None
    with pytest.raises(ValueError):
        mask_lengths(torch.tensor([[0, 1, 1, 1, 1.0]]), 1, 5)  # not a prefix
    with pytest.raises(ValueError):
        mask_lengths(torch.zeros(1, 5), 1, 5)  # nothing attended


@pytest.mark.gpu
@pytest.mark.parametrize("q_len,kv_len,valid", [(192, 24, (17, 9)), (4096, 300, (300, 1)),
                                                 (1000, 129, None)])
def test_cross_kernel_against_fp32(q_len, kv_len, valid):
    from eraserdit_b200.cross_attention import cross_attention_bshd
    g = torch.Generator(device="cuda").manual_seed(q_len)
    mk = lambda n: torch.randn(2, n, 4, 64, generator=g, device="cuda").bfloat16()
    q, k, v = mk(q_len), mk(kv_len), mk(kv_len)
    got = cross_attention_bshd(q, k, v, 0.125, list(valid) if valid else None)
    lens = list(valid) if valid else [kv_len, kv_len]
    want = torch.empty(2, q_len, 4, 64, device="cuda")
    for b in range(2):
        n = lens[b]
        s = torch.einsum("qhd,khd->hqk", q[b].float(), k[b, :n].float()) * 0.125
        want[b] = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v[b, :n].float())
    assert torch.isfinite(got).all()
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.9999


@pytest.mark.gpu
def test_cross_module_against_oracle():
    from eraserdit_b200.cross_attention import EraserDiTCrossAttention
    cfg, p, x, enc, keep, bias = cross_inputs()
    p16 = p.to(torch.bfloat16)
    layer = EraserDiTCrossAttention.from_params(p16, device="cuda")
    got = layer(x.bfloat16().cuda(), enc.bfloat16().cuda(), bias.cuda()).float().cpu()
    with torch.no_grad():
        want = ref.cross_attention_layer(x.bfloat16().float(), enc.bfloat16().float(),
                                         p16.to(torch.float32), bias)
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.9999
    # and the raw keep-mask form gives the same
    again = layer(x.bfloat16().cuda(), enc.bfloat16().cuda(), keep.cuda()).float().cpu()
    assert torch.equal(again, got)
