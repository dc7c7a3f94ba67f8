"""The CPU oracle reproduces the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from oracle import reference_path as ref
from eraserdit_b200.synthetic import CONFIG0, make_hidden, make_params

ROWS = list(range(0, 192, 24)) + [191]


def _rows(t):
    return t[:, ROWS].float().numpy()


# torch's vectorised CPU cos/sin can differ in the last bit between host CPUs
# (instruction-set paths); the fixtures were generated on one host, so the
# table is compared to 1e-6 (|cos|, |sin| <= 1; on that host it is bit-exact).
ROPE_ATOL = 1e-6
BF16_HOST_ATOL = 4e-3


def test_rope_table_matches_reference_class(golden):
    c = CONFIG0
    cos, sin = ref.rope_table(c.batch, c.frames, c.height, c.width)
    np.testing.assert_allclose(_rows(cos), golden["rope_int_cos_rows"], rtol=0, atol=ROPE_ATOL)
    np.testing.assert_allclose(_rows(sin), golden["rope_int_sin_rows"], rtol=0, atol=ROPE_ATOL)
    assert cos.double().sum().item() == pytest.approx(float(golden["rope_int_cos_sum"]),
                                                      abs=ROPE_ATOL * cos.numel())
    cos_s, sin_s = ref.rope_table(c.batch, c.frames, c.height, c.width,
                                  rope_interpolation_scale=(8.0 / 25.0, 32.0, 32.0))
    np.testing.assert_allclose(_rows(cos_s), golden["rope_scaled_cos_rows"], rtol=0,
                               atol=ROPE_ATOL)
    np.testing.assert_allclose(_rows(sin_s), golden["rope_scaled_sin_rows"], rtol=0,
                               atol=ROPE_ATOL)


def test_layer_fp32_matches_reference_processor(golden):
    c = CONFIG0
    p = make_params(c.seed, c.eps)
    x = make_hidden(c)
    cos, sin = ref.rope_table(c.batch, c.frames, c.height, c.width)
    with torch.no_grad():
        out, core = ref.self_attention_layer(x, p, cos, sin, return_core=True)
    np.testing.assert_allclose(_rows(out), golden["layer0_fp32_rows"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(_rows(core.flatten(2, 3)), golden["core0_fp32_rows"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(out.double().sum(dim=(0, 1)).numpy(), golden["layer0_fp32_channel_sum"],
                               rtol=0, atol=1e-4)
    np.testing.assert_allclose(out.double().square().sum(-1).numpy(), golden["layer0_fp32_token_sumsq"],
                               rtol=1e-5)


def test_layer_bf16_matches_reference_processor(golden):
    c = CONFIG0
    p = make_params(c.seed, c.eps).to(torch.bfloat16)
    x = make_hidden(c).bfloat16()
    cos, sin = ref.rope_table(c.batch, c.frames, c.height, c.width)
    with torch.no_grad():
        out = ref.self_attention_layer(x, p, cos, sin)
    got, want = _rows(out), golden["layer0_bf16_rows"]
    # CPU BF16 GEMMs round differently on hosts with native BF16 dot products
    # (AVX512-BF16/AMX) than on the host that made the fixtures, where this is
    # bit-exact; across hosts the rows agree to a few BF16 steps of the
    # output's scale (|out| <= 0.43 here, one step 2^-9).
    np.testing.assert_allclose(got, want, rtol=0, atol=BF16_HOST_ATOL)
    cos = float((got * want).sum() / np.sqrt((got * got).sum() * (want * want).sum()))
    assert cos >= 0.99999


@pytest.mark.parametrize("tag", ["a", "b"])
def test_qk_rmsnorm_rope_bit_exact(golden, tag):
    bf = lambda k: torch.from_numpy(golden[f"qk_{tag}_{k}"]).view(torch.bfloat16)
    angles = torch.from_numpy(golden[f"qk_{tag}_angles"])
    eps = float(golden[f"qk_{tag}_eps"])
    oq, ok = ref.qk_rmsnorm_rope(bf("q"), bf("k"), bf("wq"), bf("wk"), angles.cos(), angles.sin(), eps)
    assert torch.equal(oq.view(torch.int16), bf("out_q").view(torch.int16))
    assert torch.equal(ok.view(torch.int16), bf("out_k").view(torch.int16))
