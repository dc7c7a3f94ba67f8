"""Fused QK RMSNorm + RoPE kernel vs the reference closure (golden fixtures) and the oracle."""
import pytest
import torch

from oracle import reference_path as ref
from eraserdit_b200.synthetic import CONFIG0, CONFIG1
from tests.helpers import bf16_ulp_distance

pytestmark = pytest.mark.gpu


class Norm:
    def __init__(self, weight, eps):
        self.weight, self.eps, self.bias = weight, eps, None


def _fusion():
    from eraserdit_b200.operator_fusion import apply_fused_qk_rmsnorm_rope
    return apply_fused_qk_rmsnorm_rope


def _assert_close_bf16(got, want, max_frac=1e-3):
    """Kernel and reference differ only in the order of the fp32 sum of squares.
    That moves a normalised value by at most one BF16 ulp, rarely; after RoPE a
    cancelling pair can turn that into several ulps of a near-zero result, so
    the bound is absolute (one ulp of the row scale) plus a mismatch budget and
    the reference's own rel-RMSE bar for fused QK norm/RoPE (< 1e-3,
    tests/test_qk_fast_fusion.py:55-57 of the reference)."""
    got, want = got.cpu(), want.cpu()
    d = bf16_ulp_distance(got, want)
    assert float((d > 0).float().mean()) <= max_frac
    diff = (got.float() - want.float()).abs()
    row_scale = want.float().abs().amax(dim=-1, keepdim=True)
    assert bool((diff <= row_scale * 2.0 ** -7).all()), float((diff / row_scale).max())
    rel = ((got.float() - want.float()).square().mean()
           / want.float().square().mean().clamp_min(1e-30)).sqrt()
    assert float(rel) < 1e-3


@pytest.mark.parametrize("tag", ["a", "b"])
def test_matches_reference_closure_golden(golden, tag):
    bf = lambda key: torch.from_numpy(golden[f"qk_{tag}_{key}"]).view(torch.bfloat16)
    angles = torch.from_numpy(golden[f"qk_{tag}_angles"])
    eps = float(golden[f"qk_{tag}_eps"])
    q, k = bf("q").cuda(), bf("k").cuda()
    q0, k0 = q.clone(), k.clone()
    freqs = (angles.cos().cuda(), angles.sin().cuda())
    oq, ok = _fusion()(q, k, Norm(bf("wq").cuda(), eps), Norm(bf("wk").cuda(), eps), freqs)
    torch.cuda.synchronize()
    _assert_close_bf16(oq, bf("out_q"))
    _assert_close_bf16(ok, bf("out_k"))
    assert torch.equal(q, q0) and torch.equal(k, k0)


@pytest.mark.parametrize("shape,amp,eps", [((1, 1, 2048), 1.0, 1e-5), ((2, 257, 2048), 0.001, 1e-6),
                                           ((2, 33, 2048), 100.0, 1e-5), ((3, 64, 2048), 1.0, 1e-6)])
def test_matches_oracle_random(shape, amp, eps):
    g = torch.Generator().manual_seed(813 + shape[1])
    q = (torch.randn(shape, generator=g) * amp).bfloat16()
    k = (torch.randn(shape, generator=g) * amp).bfloat16()
    wq = (torch.rand(2048, generator=g) * 4 - 2).bfloat16()
    wk = (torch.rand(2048, generator=g) * 1.6 + 0.2).bfloat16()
    angles = torch.randn(shape, generator=g)
    cos, sin = angles.cos(), angles.sin()
    want_q, want_k = ref.qk_rmsnorm_rope(q, k, wq, wk, cos, sin, eps)
    oq, ok = _fusion()(q.cuda(), k.cuda(), Norm(wq.cuda(), eps), Norm(wk.cuda(), eps),
                       (cos.cuda(), sin.cuda()))
    _assert_close_bf16(oq, want_q)
    _assert_close_bf16(ok, want_k)


def test_norm_without_weight_and_no_rope():
    from eraserdit_b200.operator_fusion import qk_norm_rope_into
    g = torch.Generator().manual_seed(5)
    q = torch.randn(2, 40, 2048, generator=g).bfloat16()
    k = torch.randn(2, 40, 2048, generator=g).bfloat16()
    qd, kd = q.cuda(), k.cuda()
    oq, ok = torch.empty_like(qd), torch.empty_like(kd)
    qk_norm_rope_into(qd, kd, None, None, 1e-6, None, oq, ok)
    _assert_close_bf16(oq, ref.rms_norm(q, None, 1e-6))
    _assert_close_bf16(ok, ref.rms_norm(k, None, 1e-6))


@pytest.mark.parametrize("cfg,scale", [(CONFIG0, None), (CONFIG0, (8 / 25, 32.0, 32.0)),
                                       (CONFIG1, None), (CONFIG1, (8 / 25, 32.0, 32.0))])
def test_axis_table_matches_reference_table(cfg, scale):
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    rope = LTXVideoRotaryPosEmbed()
    table = rope(cfg.frames, cfg.height, cfg.width, rope_interpolation_scale=scale)
    cos, sin = table.full(1)
    want_cos, want_sin = ref.rope_table(1, cfg.frames, cfg.height, cfg.width,
                                        rope_interpolation_scale=scale)
    assert float((cos.cpu() - want_cos).abs().max()) <= 1e-6
    assert float((sin.cpu() - want_sin).abs().max()) <= 1e-6


def test_axis_mode_equals_table_mode_and_layouts():
    """Axis-table RoPE == full-table RoPE (bitwise); head-major / destination-major
    outputs and the V copy are exact permutations; in-place == out-of-place."""
    from eraserdit_b200.operator_fusion import qk_norm_rope_into
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    F_, H_, W_ = 3, 5, 7
    S, B = F_ * H_ * W_, 2
    table = LTXVideoRotaryPosEmbed()(F_, H_, W_)
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, S, 6144, generator=g, device="cuda").bfloat16()
    q, k, v = qkv[..., :2048], qkv[..., 2048:4096], qkv[..., 4096:]
    wq = torch.rand(2048, generator=g, device="cuda").bfloat16()
    wk = torch.rand(2048, generator=g, device="cuda").bfloat16()
    cos, sin = table.full(B)
    oq1, ok1 = torch.empty(B, S, 2048, device="cuda", dtype=torch.bfloat16), torch.empty(
        B, S, 2048, device="cuda", dtype=torch.bfloat16)
    qk_norm_rope_into(q, k, wq, wk, 1e-6, (cos, sin), oq1, ok1)
    oq2, ok2 = torch.empty_like(oq1), torch.empty_like(ok1)
    qk_norm_rope_into(q, k, wq, wk, 1e-6, table, oq2, ok2)
    assert torch.equal(oq1, oq2) and torch.equal(ok1, ok2)
    # Ulysses send layout [dest][qkv][B][H/N][S][D] for N = 4
    n, hl = 4, 8
    send = torch.empty(n, 3, B, hl, S, 64, device="cuda", dtype=torch.bfloat16)
    chunk = B * hl * S * 64
    qk_norm_rope_into(q, k, wq, wk, 1e-6, table, send[:, 0], send[:, 1], value=v, v_out=send[:, 2],
                      out_token_stride=64, out_batch_stride=hl * S * 64, out_head_stride=S * 64,
                      heads_per_dest=hl, out_dest_stride=3 * chunk)
    expect = lambda t: t.unflatten(2, (n, hl, 64)).permute(2, 0, 3, 1, 4)
    assert torch.equal(send[:, 0], expect(oq2))
    assert torch.equal(send[:, 1], expect(ok2))
    assert torch.equal(send[:, 2], expect(v))
    # in place, inside the interleaved QKV buffer
    qk_norm_rope_into(q, k, wq, wk, 1e-6, table, q, k)
    assert torch.equal(q, oq2) and torch.equal(k, ok2)
