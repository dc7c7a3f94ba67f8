"""tcgen05 attention kernel vs an fp32 torch reference on the GPU."""
import pytest
import torch

from tests.helpers import attention_fp32, cosine, max_abs

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2     # north star: BF16 within max-abs 2e-2 ...
MIN_COSINE = 0.9999  # ... and cosine >= 0.9999 against fp32 SDPA


def _impl():
    from eraserdit_b200.attention import B200AttentionImpl
    return B200AttentionImpl(32, 64, 0.125)


def _inputs(batch, seq, heads, seed, amp=1.0, layout="bshd"):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if layout == "bshd":
        mk = lambda: (torch.randn(batch, seq, heads, 64, generator=g, device="cuda") * amp).bfloat16()
        return mk(), mk(), mk()
    if layout == "bhsd":
        mk = lambda: (torch.randn(batch, heads, seq, 64, generator=g, device="cuda") * amp
                      ).bfloat16().transpose(1, 2)
        return mk(), mk(), mk()
    qkv = (torch.randn(batch, seq, 3, heads, 64, generator=g, device="cuda") * amp).bfloat16()
    return qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]


def _check(out, q, k, v, scale=0.125):
    from eraserdit_b200 import _native
    want = attention_fp32(q, k, v, scale)
    assert _native.read_status(q.device) == 0
    assert torch.isfinite(out).all()
    assert max_abs(out, want) <= MAX_ABS
    assert cosine(out, want) >= MIN_COSINE


@pytest.mark.parametrize("batch,seq,heads", [(1, 1, 1), (1, 127, 2), (1, 128, 1), (1, 129, 2),
                                             (1, 192, 32), (2, 300, 3), (1, 1000, 2),
                                             (2, 4081, 2), (1, 8192, 4)])
def test_shapes(batch, seq, heads):
    q, k, v = _inputs(batch, seq, heads, seed=seq)
    from eraserdit_b200.attention import AttentionMetadata
    out = _impl().forward(q, k, v, AttentionMetadata())
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    _check(out, q, k, v)


@pytest.mark.parametrize("layout", ["bhsd", "packed"])
def test_strided_layouts(layout):
    q, k, v = _inputs(2, 777, 4, seed=3, layout=layout)
    from eraserdit_b200.attention import AttentionMetadata
    _check(_impl().forward(q, k, v, AttentionMetadata()), q, k, v)


@pytest.mark.parametrize("amp", [4.0, 12.0])
def test_peaked_softmax_rescaling(amp):
    """Large logits make the running max grow often (exercises the O rescale path)."""
    q, k, v = _inputs(1, 2049, 2, seed=7, amp=1.0)
    q = (q.float() * amp).bfloat16()
    from eraserdit_b200.attention import AttentionMetadata
    _check(_impl().forward(q, k, v, AttentionMetadata()), q, k, v)


def test_segmented_sequence():
    """The all-to-all receive layout: nseg segments of seg_len tokens, head-major."""
    from eraserdit_b200 import _native
    nseg, seg_len, batch, heads = 3, 200, 2, 4
    g = torch.Generator(device="cuda").manual_seed(21)
    recv = torch.randn(nseg, 3, batch, heads, seg_len, 64, generator=g, device="cuda").bfloat16()
    full = lambda i: recv[:, i].permute(1, 0, 3, 2, 4).reshape(batch, nseg * seg_len, heads, 64)
    q, k, v = full(0), full(1), full(2)
    out = torch.zeros(nseg, batch, seg_len, heads, 64, device="cuda", dtype=torch.bfloat16)
    lib = _native.load()
    ss, qs = 3 * batch * heads * seg_len * 64, batch * heads * seg_len * 64
    strides = [64, seg_len * 64, heads * seg_len * 64, ss]
    rc = lib.erd_attn_fwd_bf16(
        recv[:, 0].data_ptr(), recv[:, 1].data_ptr(), recv[:, 2].data_ptr(), *strides, *strides,
        *strides, batch, heads, seg_len, nseg, None, 64, 0.125, out.data_ptr(),
        heads * 64, 64, seg_len * heads * 64, batch * seg_len * heads * 64,
        _native.status_word(q.device).data_ptr(), _native.stream_handle(q.device))
    _native.check(rc, "erd_attn_fwd_bf16")
    assert qs > 0
    got = out.permute(1, 0, 2, 3, 4).reshape(batch, nseg * seg_len, heads, 64)
    _check(got, q, k, v)


def test_deterministic_and_stream_safe():
    q, k, v = _inputs(2, 1500, 3, seed=9)
    from eraserdit_b200.attention import AttentionMetadata
    a = _impl().forward(q, k, v, AttentionMetadata())
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        b = _impl().forward(q, k, v, AttentionMetadata())
    torch.cuda.current_stream().wait_stream(stream)
    assert torch.equal(a, b)


def test_probe_and_rejections():
    from eraserdit_b200.attention import (AttentionCapability, AttentionMetadata,
                                          B200AttentionBackend)
    dev = torch.device("cuda")
    assert B200AttentionBackend.probe(AttentionCapability(dev, torch.bfloat16, 64)).supported
    assert not B200AttentionBackend.probe(AttentionCapability(dev, torch.float16, 64)).supported
    assert not B200AttentionBackend.probe(AttentionCapability(dev, torch.bfloat16, 128)).supported
    q, k, v = _inputs(1, 16, 2, seed=1)
    with pytest.raises(ValueError):
        _impl().forward(q, k, v, AttentionMetadata(attn_mask=torch.ones(1, dtype=torch.bool)))
    with pytest.raises(ValueError):
        _impl().forward(q.float(), k.float(), v.float(), AttentionMetadata())


@pytest.mark.parametrize("batch,seq", [(2, 0), (0, 16)])
def test_empty_inputs_return_empty_output(batch, seq):
    """An empty sequence or batch gives an empty output (as the reference's
    SDPA does) and launches nothing."""
    from eraserdit_b200 import _native
    from eraserdit_b200.attention import AttentionMetadata
    q = torch.empty(batch, seq, 4, 64, device="cuda", dtype=torch.bfloat16)
    out = _impl().forward(q, q, q, AttentionMetadata())
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    assert _native.read_status(q.device) == 0
