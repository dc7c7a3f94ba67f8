"""The ring-piece restatement (oracle/ring.py) against full attention on the CPU.

The reference's ring accumulator is a Triton kernel and cannot run here; its
restatement is pinned by the identity every ring order must satisfy: the
attention over all pieces equals the full attention of the golden-pinned
``oracle.reference_path.sdpa_bshd``."""
import pytest
import torch

from oracle import ring as oracle_ring
from oracle.reference_path import sdpa_bshd
from tests.helpers import cosine, max_abs


def _qkv(batch, nq, nk, heads, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, nq, heads, 64, generator=g).to(dtype)
    k = torch.randn(batch, nk, heads, 64, generator=g).to(dtype)
    v = torch.randn(batch, nk, heads, 64, generator=g).to(dtype)
    return q, k, v


@pytest.mark.parametrize("pieces,ring_rank", [([200], 0), ([100, 37, 133], 0),
                                              ([128, 128, 1, 64], 2), ([5, 300], 1)])
def test_pieces_equal_full_attention_fp32(pieces, ring_rank):
    q, k, v = _qkv(2, 70, sum(pieces), 3, torch.float32, seed=len(pieces) + ring_rank)
    ks, vs = list(k.split(pieces, dim=1)), list(v.split(pieces, dim=1))
    got = oracle_ring.ring_pieces(q, ks, vs, ring_rank, scale=0.125)
    want = sdpa_bshd(q, k, v, 0.125).float()
    assert max_abs(got, want) <= 2e-6


def test_pieces_bf16_p_rounding_within_bf16_bar():
    """With BF16 operands P is rounded to BF16 before P V, as in the
    reference kernel: the result stays inside the BF16 bar against fp32."""
    q, k, v = _qkv(1, 129, 400, 2, torch.bfloat16, seed=7)
    ks, vs = list(k.split([150, 250], dim=1)), list(v.split([150, 250], dim=1))
    got = oracle_ring.ring_pieces(q, ks, vs, 1, scale=0.125)
    want = sdpa_bshd(q.float(), k.float(), v.float(), 0.125).float()
    assert max_abs(got, want) <= 2e-2
    assert cosine(got, want) >= 0.9999


def test_state_carries_between_calls():
    q, k, v = _qkv(1, 10, 260, 1, torch.float32, seed=3)
    state = oracle_ring.piece(q, k[:, :130], v[:, :130])
    out = oracle_ring.piece(q, k[:, 130:], v[:, 130:], state, final=True)
    assert max_abs(out, sdpa_bshd(q, k, v, 64 ** -0.5).float()) <= 2e-6
