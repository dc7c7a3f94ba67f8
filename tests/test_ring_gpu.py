"""Ring attention kernels and the USP layer on one GPU.

- ``piece`` (the ``ring_accumulator.piece`` drop-in) over uneven pieces against
  fp32 attention over all keys and against the oracle's ring restatement;
- Ulysses x Ring ranks emulated on one GPU: the reference ring mode equals the
  Ulysses layer at degree U * R bit for bit (every query row meets the same key
  tiles in the same order), the streaming mode matches the single-GPU layer."""
import pytest
import torch

from oracle import ring as oracle_ring
from tests.helpers import attention_fp32, cosine, max_abs

pytestmark = pytest.mark.gpu


def _qkv(batch, nq, nk, heads, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda n: torch.randn(batch, n, heads, 64, generator=g, device="cuda").bfloat16()
    return mk(nq), mk(nk), mk(nk)


def test_single_final_piece_equals_attention_kernel():
    from eraserdit_b200.attention import attention_bshd
    from eraserdit_b200.ring import piece
    q, k, v = _qkv(2, 300, 300, 3, seed=1)
    assert torch.equal(piece(q, k, v, final=True, scale=0.125), attention_bshd(q, k, v, 0.125))


@pytest.mark.parametrize("nq,pieces,batch,heads", [(300, [257, 128, 75], 2, 3),
                                                    (128, [1, 513], 1, 2),
                                                    (1000, [333, 334, 333, 1000], 2, 4)])
def test_pieces_match_fp32_attention(nq, pieces, batch, heads):
    from eraserdit_b200 import _native
    from eraserdit_b200.ring import piece
    q, k, v = _qkv(batch, nq, sum(pieces), heads, seed=nq + len(pieces))
    state = None
    for i, (ks, vs) in enumerate(zip(k.split(pieces, dim=1), v.split(pieces, dim=1))):
        last = i == len(pieces) - 1
        state = piece(q, ks.contiguous(), vs.contiguous(), state, final=last, scale=0.125)
    out = state
    assert _native.read_status(q.device) == 0
    want = attention_fp32(q, k, v, 0.125)
    assert max_abs(out, want) <= 2e-2  # BF16 bar of the north star
    assert cosine(out, want) >= 0.9999
    # the restated reference accumulator over the same pieces (CPU)
    ks = [t.cpu() for t in k.split(pieces, dim=1)]
    vs = [t.cpu() for t in v.split(pieces, dim=1)]
    ref = oracle_ring.ring_pieces(q[:, :64].cpu(), ks, vs, len(pieces) - 1, scale=0.125)
    assert max_abs(out[:, :64].cpu(), ref) <= 2e-2
    assert cosine(out[:, :64].cpu(), ref) >= 0.9999


def test_piece_rejects_foreign_state_and_small_buffer():
    from eraserdit_b200.ring import RingState, piece, ring_attention_into
    q, k, v = _qkv(1, 200, 200, 2, seed=3)
    state = piece(q, k, v, scale=0.125)
    with pytest.raises(ValueError):
        piece(q[:, :100].contiguous(), k, v, state, final=True)
    small = RingState(1, 2, 100, 1, q.device)  # sized for 100 queries, used for 200
    st = lambda t: (t.stride(1), t.stride(2), t.stride(0), 0)
    with pytest.raises(RuntimeError):
        ring_attention_into(q, k, v, None, 0.125, batch=1, heads=2, seg_len=200, q_seg_lens=[200],
                            kv_seg_len=200, kv_seg_lens=[200], q_strides=st(q), k_strides=st(k),
                            v_strides=st(v), o_strides=(0, 0, 0, 0), state=small, state_mode=2)


def _setup(frames, height, width, batch, seed):
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.synthetic import make_params
    p = make_params(seed, 1e-6, random_norm_weight=True, device="cuda")
    layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda")
    rope = LTXVideoRotaryPosEmbed()(frames, height, width)
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(batch, frames * height * width, 2048, generator=g, device="cuda").bfloat16()
    return layer, rope, x


@pytest.mark.parametrize("ulysses,ring,grid", [(2, 2, (2, 8, 12)), (1, 4, (1, 7, 11)),
                                               (4, 2, (3, 5, 7)), (2, 4, (2, 8, 12))])
def test_reference_mode_bitwise_equals_ulysses(ulysses, ring, grid):
    from eraserdit_b200 import _native
    from eraserdit_b200.ring import emulate_usp_ranks
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(*grid, 2, seed=ulysses * 10 + ring)
    usp = emulate_usp_ranks(layer, ulysses, ring, x, rope, mode="reference")
    uly = emulate_ranks(layer, ulysses * ring, x, rope)
    assert _native.read_status(x.device) == 0
    for a, b in zip(usp, uly):
        assert torch.equal(a, b)


@pytest.mark.parametrize("ulysses,ring,grid", [(2, 2, (2, 8, 12)), (1, 4, (1, 7, 11)),
                                               (4, 2, (3, 5, 7)), (1, 2, (2, 8, 12))])
def test_streaming_mode_matches_single_gpu(ulysses, ring, grid):
    from eraserdit_b200 import _native
    from eraserdit_b200.ring import emulate_usp_ranks
    layer, rope, x = _setup(*grid, 2, seed=ulysses + 7 * ring)
    want = layer(x, rope)
    got = torch.cat(emulate_usp_ranks(layer, ulysses, ring, x, rope, mode="streaming"), dim=1)
    assert _native.read_status(x.device) == 0
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.99999


def test_streaming_full_size_ring8():
    """Configuration 1's sequence as 8 ring pieces of 4080 tokens (U = 1,
    R = 8, emulated): the carried state over eight launches per rank gives the
    single-GPU layer's output."""
    from eraserdit_b200.ring import emulate_usp_ranks
    layer, rope, x = _setup(16, 34, 60, 1, seed=1)
    want = layer(x, rope)
    got = torch.cat(emulate_usp_ranks(layer, 1, 8, x, rope, mode="streaming"), dim=1)
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.99999


@pytest.mark.parametrize("mode", ["reference", "streaming"])
@pytest.mark.parametrize("ulysses,ring,grid", [(2, 2, (2, 8, 12)), (2, 2, (1, 7, 11)),
                                               (4, 2, (3, 5, 7)), (2, 4, (2, 8, 12))])
def test_peer_transport_bitwise_equal_nccl_layout(ulysses, ring, grid, mode):
    """The peer-memory Ulysses exchanges inside every ring index (prologue and
    last attention launch storing into the group peers' buffers) give exactly
    the all-to-all layout's result, with even and uneven shards."""
    from eraserdit_b200 import _native
    from eraserdit_b200.ring import emulate_usp_ranks
    layer, rope, x = _setup(*grid, 2, seed=3 * ulysses + ring)
    nccl = emulate_usp_ranks(layer, ulysses, ring, x, rope, mode=mode)
    peer = emulate_usp_ranks(layer, ulysses, ring, x, rope, mode=mode, transport="peer")
    assert _native.read_status(x.device) == 0
    for a, b in zip(nccl, peer):
        assert torch.equal(a, b)
