"""erd_linear_bf16 (the projections' tcgen05 GEMM) against an fp32 linear and
torch's BF16 F.linear on the same operands."""
import pytest
import torch

from tests.helpers import bf16_ulp_distance, cosine

pytestmark = pytest.mark.gpu


def _operands(m, n, k, seed, bias=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    b = (torch.randn(n, generator=g, device="cuda") * 0.5).bfloat16() if bias else None
    return x, w, b


def _fp32(x, w, b):
    y = x.float() @ w.float().T
    return y if b is None else y + b.float()


@pytest.mark.parametrize("m,n,k", [(192, 6144, 2048), (8160, 2048, 2048), (1, 256, 64),
                                   (300, 512, 192), (65280, 6144, 2048)])
def test_linear_matches_fp32_and_f_linear(m, n, k):
    from eraserdit_b200.linear import linear_bf16
    from eraserdit_b200 import _native
    x, w, b = _operands(m, n, k, seed=m + n)
    got = linear_bf16(x, w, b)
    assert _native.read_status(x.device) == 0
    want = _fp32(x, w, b)
    # one BF16 rounding of an fp32 sum: half an ulp of |y| (2^-8 relative) plus
    # summation-order effects far below it
    assert bool(((got.float() - want).abs() <= want.abs() * 2.0 ** -8 + 1e-3).all())
    assert cosine(got, want) >= 0.99999
    lib = torch.nn.functional.linear(x, w, b)
    ulps = bf16_ulp_distance(got, lib)
    assert int(ulps.max()) <= 1 and float((ulps > 0).float().mean()) < 0.01


def test_linear_without_bias_and_strided_rows():
    """The output projection reads rows with a stride (a view of a wider
    buffer); no bias; the result goes into a caller's buffer."""
    from eraserdit_b200.linear import linear_bf16
    x_full, w, _ = _operands(1000, 2048, 4096, seed=3)
    x = x_full[:, 1024:3072]  # row stride 4096, k = 2048
    w = w[:, :2048].contiguous()
    out = torch.full((1000, 2048), float("nan"), device="cuda", dtype=torch.bfloat16)
    linear_bf16(x, w, None, out=out)
    want = _fp32(x, w, None)
    assert bool(((out.float() - want).abs() <= want.abs() * 2.0 ** -8 + 1e-3).all())


def test_linear_batched_view_and_errors():
    from eraserdit_b200.linear import linear_bf16
    x, w, b = _operands(2 * 500, 2048, 2048, seed=5)
    x3 = x.view(2, 500, 2048)
    y = linear_bf16(x3, w, b)
    assert y.shape == (2, 500, 2048)
    want = _fp32(x, w, b)
    assert bool(((y.view(1000, 2048).float() - want).abs() <= want.abs() * 2.0 ** -8 + 1e-3).all())
    with pytest.raises(ValueError):
        linear_bf16(x, w[:200], b[:200])  # n not a multiple of 256
    with pytest.raises(ValueError):
        linear_bf16(x[:, :100], w[:, :100], b)  # k not a multiple of 64


def test_linear_rows_of_wider_slots():
    """[B, L, k] rows that are a prefix of [B, L_slot, k] slots (the peer
    exchange's output-projection input with an uneven partition)."""
    from eraserdit_b200.linear import linear_bf16
    x_slots, w, b = _operands(2 * 700, 2048, 2048, seed=9)
    x = x_slots.view(2, 700, 2048)[:, :513]
    y = linear_bf16(x, w, b)
    want = torch.stack([_fp32(x[i], w, b) for i in range(2)])
    assert y.shape == (2, 513, 2048)
    assert bool(((y.float() - want).abs() <= want.abs() * 2.0 ** -8 + 1e-3).all())


@pytest.mark.parametrize("batch,tokens,n,col0,group", [(2, 4080, 6144, 4096, 256),
                                                       (2, 300, 6144, 4096, 1024),
                                                       (1, 517, 1024, 512, 128),
                                                       (3, 129, 768, 0, 256)])
def test_scatter_columns_equal_plain_product(batch, tokens, n, col0, group):
    """erd_linear_bf16_scatter: the columns below col0 land in `out`, the rest in
    the destination buffers at (b * batch_stride + t * token_stride + column
    within the group), bit for bit what erd_linear_bf16 computes."""
    from eraserdit_b200 import _native
    from eraserdit_b200.linear import linear_bf16, linear_bf16_scatter
    k = 2048
    g = torch.Generator(device="cuda").manual_seed(batch * tokens + n)
    x = torch.randn(batch, tokens, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    bias = (torch.randn(n, generator=g, device="cuda") * 0.5).bfloat16()
    want = linear_bf16(x, w, bias)
    ndest = (n - col0) // group
    batch_stride, token_stride = group + 64, batch * (group + 64) + 8
    dests = [torch.full((tokens * token_stride + batch * batch_stride,), -7.0,
                        device="cuda", dtype=torch.bfloat16) for _ in range(ndest)]
    out = torch.zeros(batch, tokens, n, device="cuda", dtype=torch.bfloat16)
    linear_bf16_scatter(x, w, bias, out, col0, [d.data_ptr() for d in dests], group,
                        batch_stride, token_stride)
    assert _native.read_status(x.device) == 0
    assert torch.equal(out[..., :col0], want[..., :col0])
    assert bool((out[..., col0:] == 0).all())  # scattered columns never touch out
    for gi, d in enumerate(dests):
        idx = (torch.arange(batch, device="cuda")[:, None, None] * batch_stride
               + torch.arange(tokens, device="cuda")[None, :, None] * token_stride
               + torch.arange(group, device="cuda")[None, None, :])
        assert torch.equal(d[idx], want[..., col0 + gi * group:col0 + (gi + 1) * group])
        hit = torch.zeros_like(d, dtype=torch.bool)
        hit[idx.flatten()] = True
        assert bool((d[~hit] == -7.0).all())  # nothing else written


def test_scatter_rejects_bad_layouts():
    from eraserdit_b200.linear import linear_bf16_scatter
    x = torch.zeros(1, 8, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(512, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(1, 8, 512, device="cuda", dtype=torch.bfloat16)
    d = torch.zeros(4096, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):  # 3 x 128 columns do not cover n - col0 = 256
        linear_bf16_scatter(x, w, None, out, 256, [d.data_ptr()] * 3, 128, 0, 256)
    with pytest.raises(RuntimeError):  # group width not a power of two
        linear_bf16_scatter(x, w, None, out, 256, [d.data_ptr()], 192, 0, 256)
    with pytest.raises(RuntimeError):  # col0 not a multiple of 256
        linear_bf16_scatter(x, w, None, out, 128, [d.data_ptr()] * 3, 128, 0, 256)
