"""Ulysses SP layer: N ranks emulated on one GPU (same buffers and kernels as the
NCCL path, chunks exchanged by copies) against the single-GPU layer output."""
import pytest
import torch

from eraserdit_b200.synthetic import make_params
from tests.helpers import cosine, max_abs

pytestmark = pytest.mark.gpu


def _setup(frames, height, width, batch, seed):
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    p = make_params(seed, 1e-6, random_norm_weight=True, device="cuda")
    layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda")
    rope = LTXVideoRotaryPosEmbed()(frames, height, width)
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(batch, frames * height * width, 2048, generator=g, device="cuda").bfloat16()
    return layer, rope, x


@pytest.mark.parametrize("degree,grid,batch", [(2, (2, 8, 12), 2), (4, (2, 8, 12), 1),
                                               (8, (2, 8, 12), 2), (4, (1, 7, 11), 2),
                                               (8, (3, 5, 7), 1)])
def test_emulated_ranks_match_single_gpu(degree, grid, batch):
    from eraserdit_b200 import _native
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(*grid, batch, seed=degree + grid[0])
    want = layer(x, rope)
    got = torch.cat(emulate_ranks(layer, degree, x, rope), dim=1)
    assert _native.read_status(x.device) == 0
    assert got.shape == want.shape
    assert max_abs(got, want) <= 1e-2  # one BF16 ulp at |y| ~ 1: KV blocks split per segment
    assert cosine(got, want) >= 0.99999


def test_sp8_full_size_matches_single_gpu():
    """Config 2 at SP8 (4080 tokens per rank), emulated: same layer output."""
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(16, 34, 60, 2, seed=1)
    want = layer(x, rope)
    got = torch.cat(emulate_ranks(layer, 8, x, rope), dim=1)
    assert max_abs(got, want) <= 1e-2  # one BF16 ulp at |y| ~ 1: KV blocks split per segment
    assert cosine(got, want) >= 0.99999


@pytest.mark.parametrize("degree,chunks", [(2, 2), (2, 4), (4, 2), (8, 4)])
def test_head_chunks_bitwise_equal_unchunked(degree, chunks):
    """The head-chunk layout changes only the exchange granularity: every
    rank's output equals the unchunked one bit for bit (as the reference's
    tests/test_ulysses_overlap.py:38-45 requires)."""
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(2, 8, 12, 2, seed=degree)
    plain = emulate_ranks(layer, degree, x, rope, head_chunks=1)
    chunked = emulate_ranks(layer, degree, x, rope, head_chunks=chunks)
    for a, b in zip(plain, chunked):
        assert torch.equal(a, b)


@pytest.mark.parametrize("degree,grid", [(2, (2, 8, 12)), (4, (2, 8, 12)), (8, (2, 8, 12)),
                                         (2, (1, 7, 11)), (4, (1, 7, 11)), (8, (3, 5, 7))])
def test_peer_transport_bitwise_equal_nccl_layout(degree, grid):
    """The peer-memory exchange (prologue and attention epilogue storing into
    the peers' buffers, rows landing in the output projection's input layout)
    gives exactly the all-to-all path's result, with even and uneven shards."""
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(*grid, 2, seed=10 + degree)
    nccl = emulate_ranks(layer, degree, x, rope)
    peer = emulate_ranks(layer, degree, x, rope, transport="peer")
    for a, b in zip(nccl, peer):
        assert torch.equal(a, b)


@pytest.mark.parametrize("degree,grid", [(2, (1, 7, 11)), (4, (2, 8, 12)), (8, (3, 5, 7))])
def test_peer_v_from_projection_epilogue_bitwise_equal(degree, grid):
    """V stored into the peers' slots by the QKV projection's epilogue
    (erd_linear_bf16_scatter) or copied by the prologue: the same result."""
    from eraserdit_b200.ulysses import emulate_ranks
    layer, rope, x = _setup(*grid, 2, seed=30 + degree)
    copied = emulate_ranks(layer, degree, x, rope, transport="peer", v_scatter=False)
    scattered = emulate_ranks(layer, degree, x, rope, transport="peer", v_scatter=True)
    for a, b in zip(copied, scattered):
        assert torch.equal(a, b)


def test_peer_wait_times_out_and_reports_failure():
    """Failure detection without a GPU fault: a wait on a flag that nothing
    sets ends after its limit with a status bit; a negative epoch (a failed
    peer phase) ends it at once with another; the context stays usable."""
    import time
    from eraserdit_b200 import _native
    from eraserdit_b200.peer_exchange import PHASE_IN, PeerBuffers, signal, wait
    dev = torch.device("cuda", 0)
    bufs = PeerBuffers({"recv1": 1024, "recv2": 1024}, dev)
    bufs.connect_local([bufs])
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = _native.stream_handle(dev)
    t0 = time.perf_counter()
    wait(bufs, PHASE_IN, 1, 7, status, stream, timeout_ns=50_000_000)
    torch.cuda.synchronize()
    assert int(status.item()) == 0x10 and time.perf_counter() - t0 < 5
    status.zero_()
    signal(bufs, PHASE_IN, 0, 1, -8, stream)
    wait(bufs, PHASE_IN, 1, 8, status, stream, timeout_ns=2_000_000_000)
    torch.cuda.synchronize()
    assert int(status.item()) == 0x20
    status.zero_()
    signal(bufs, PHASE_IN, 0, 1, 9, stream)
    wait(bufs, PHASE_IN, 1, 9, status, stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert float(torch.ones(4, device=dev).sum()) == 4.0  # the context is fine
    bufs.close()


@pytest.mark.parametrize("degree,kind", [(4, "fp8"), (8, "sparse")])
def test_peer_transport_fp8_and_sparse(degree, kind):
    """FP8 and block-sparse attention over the peer-memory exchange: the same
    result as their all-to-all path."""
    from eraserdit_b200 import sparse_pattern as sp
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.mask_sta import SparsePlan
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.ulysses import emulate_ranks
    p = make_params(21, 1e-6, device="cuda")
    if kind == "fp8":
        layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda",
                                                   precision="fp8")
        grid, plan = (2, 8, 12), None
    else:
        layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda")
        geom = sp.StaGeometry(grid=(8, 16, 32), window=(1, 3, 2), kv_block=128)
        grid = geom.grid
        plan = SparsePlan.from_mask(sp.ellipse_masks(grid, seed=4, semi_axes=(2, 4)), geom, "cuda")
    rope = LTXVideoRotaryPosEmbed()(*grid)
    g = torch.Generator(device="cuda").manual_seed(22)
    x = torch.randn(2, grid[0] * grid[1] * grid[2], 2048, generator=g, device="cuda").bfloat16()
    nccl = emulate_ranks(layer, degree, x, rope, sparse=plan)
    peer = emulate_ranks(layer, degree, x, rope, sparse=plan, transport="peer")
    for a, b in zip(nccl, peer):
        assert torch.equal(a, b)


@pytest.mark.parametrize("degree", [2, 8])
def test_attention_level_hook(degree):
    """The reference's SP hook contract (partition, then attention(q, k, v, impl,
    metadata) on the local [B, L_rank, H, 64] tensors): equal to single-GPU
    attention over the whole sequence."""
    from eraserdit_b200.attention import attention_bshd
    from eraserdit_b200.ulysses import emulate_attention_hook
    layer, _, _ = _setup(2, 8, 12, 1, seed=30 + degree)
    g = torch.Generator(device="cuda").manual_seed(31)
    q, k, v = [torch.randn(2, 190, 32, 64, generator=g, device="cuda").bfloat16() for _ in range(3)]
    parts = emulate_attention_hook(layer, degree, q, k, v)
    got = torch.cat(parts, dim=1)
    want = attention_bshd(q, k, v, 0.125)
    assert max_abs(got, want) <= 1e-2
    assert cosine(got, want) >= 0.99999
