"""Block-sparse (mask-aware) attention: the tile-skipping kernel against fp32
attention over the same block pattern, the dense kernel, the segmented
(sequence-parallel) layout, the MaskSTA drop-in and the whole layer."""
import pytest
import torch

from eraserdit_b200 import sparse_pattern as sp
from oracle import mask_sta as oracle_sta
from oracle import reference_path as ref
from tests.helpers import cosine, masked_attention_fp32, max_abs

pytestmark = pytest.mark.gpu

MAX_ABS, MIN_COSINE = 2e-2, 0.9999  # the BF16 bar of the dense path

SMALL = sp.StaGeometry(grid=(8, 16, 32), tile=(4, 2, 4), window=(1, 3, 2), protect=(3, 5, 5),
                       query_block=128, kv_block=128)


def _qkv(batch, seq, heads, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(batch, seq, heads, 64, generator=g, device="cuda").bfloat16()
            for _ in range(3)]


def _plan(blocks, kv_block, **kw):
    from eraserdit_b200.mask_sta import SparsePlan
    return SparsePlan(blocks, kv_block, "cuda", **kw)


def _small_blocks(geom, seed):
    mask = sp.ellipse_masks(geom.grid, seed=seed, semi_axes=(2, 4))
    return sp.block_mask(mask, geom)


def test_full_pattern_is_bitwise_dense():
    from eraserdit_b200.attention import attention_bshd
    from eraserdit_b200.mask_sta import sparse_attention_bshd
    q, k, v = _qkv(2, 4096, 3, seed=1)
    plan = _plan(torch.ones(32, 32, dtype=torch.bool), 128)
    got = sparse_attention_bshd(q, k, v, 0.125, plan)
    want = attention_bshd(q, k, v, 0.125)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("kv_block", [64, 128])
@pytest.mark.parametrize("seed", [5, 6])
def test_sparse_against_masked_fp32(kv_block, seed):
    from eraserdit_b200 import _native
    from eraserdit_b200.mask_sta import sparse_attention_bshd
    geom = sp.StaGeometry(**{**SMALL.__dict__, "kv_block": kv_block})
    blocks = _small_blocks(geom, seed)
    assert 0 < int(blocks.sum()) < blocks.numel()  # really sparse, really something
    plan = _plan(blocks, kv_block)
    q, k, v = _qkv(2, geom.tokens, 3, seed=seed)
    got = sparse_attention_bshd(q, k, v, 0.125, plan)
    assert _native.read_status(q.device) == 0
    want = masked_attention_fp32(q, k, v, 0.125, blocks, kv_block)
    assert torch.isfinite(got).all()
    assert max_abs(got, want) <= MAX_ABS
    assert cosine(got, want) >= MIN_COSINE


def test_tiny_case_against_cpu_oracle():
    from eraserdit_b200.mask_sta import sparse_attention_bshd
    geom = sp.StaGeometry(grid=(4, 8, 16), tile=(4, 2, 4), window=(1, 2, 2), query_block=128,
                          kv_block=64)
    order, tiles = oracle_sta.tile_layout(geom.grid, geom.tile)
    rows = oracle_sta.background(geom.grid, geom.tile, geom.window, 128, 64)
    mask = torch.zeros(geom.grid)
    mask[1, 2, 3] = 1.0
    prot = oracle_sta.protected(mask.tolist(), order, geom.grid, geom.protect, 128)
    rows = [[b or p for b in row] for row, p in zip(rows, prot)]
    blocks = torch.tensor(rows)
    assert torch.equal(blocks, sp.block_mask(mask, geom))
    q, k, v = _qkv(1, geom.tokens, 2, seed=9)
    got = sparse_attention_bshd(q, k, v, 0.125, _plan(blocks, 64)).float().cpu()
    token_mask = sp.attention_mask(blocks, 64)
    want = oracle_sta.masked_attention(q.cpu(), k.cpu(), v.cpu(), 0.125, token_mask)
    assert max_abs(got, want) <= MAX_ABS
    assert cosine(got, want) >= MIN_COSINE


def test_segmented_layout_matches_contiguous():
    """Sequence-parallel receive layout: segments of whole 128-token blocks in
    padded slots give the same result as the contiguous sequence."""
    from eraserdit_b200.mask_sta import sparse_attention_bshd, sparse_attention_into
    geom = SMALL
    blocks = _small_blocks(geom, 7)
    batch, heads, seq = 2, 2, geom.tokens
    q, k, v = _qkv(batch, seq, heads, seed=7)
    want = sparse_attention_bshd(q, k, v, 0.125, _plan(blocks, 128))
    seg_blocks = [9, 8, 8, 7]
    tps = 10
    slot = tps * 128
    nseg = len(seg_blocks)
    lens = [n * 128 for n in seg_blocks]
    recv = torch.zeros(nseg, slot, 3, batch, heads, 64, device="cuda", dtype=torch.bfloat16)
    t0 = 0
    for s, n in enumerate(lens):
        for i, x in enumerate((q, k, v)):
            recv[s, :n, i] = x[:, t0:t0 + n].permute(1, 0, 2, 3)
        t0 += n
    out = torch.zeros(nseg, slot, batch, heads, 64, device="cuda", dtype=torch.bfloat16)
    r = recv.view(-1)
    chunk = batch * heads * 64
    st = (3 * chunk, 64, heads * 64, slot * 3 * chunk)
    plan = _plan(blocks, 128, seg_blocks=seg_blocks, tiles_per_seg=tps)
    sparse_attention_into(r, r[chunk:], r[2 * chunk:], out, 0.125, plan, batch=batch,
                          heads=heads, seg_len=slot, nseg=nseg, seg_lens=lens, q_strides=st,
                          k_strides=st, v_strides=st,
                          o_strides=(chunk, 64, heads * 64, slot * chunk))
    got = torch.cat([out[s, :n].permute(1, 0, 2, 3) for s, n in enumerate(lens)], 1)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_gather_tokens():
    from eraserdit_b200.mask_sta import gather_tokens
    x = _qkv(2, 1000, 4, seed=3)[0]
    index = torch.randperm(1000, device="cuda").to(torch.int32)[:700]
    got = gather_tokens(x, index)
    assert torch.equal(got, x[:, index.long()])


def test_mask_sta_dropin_reference_geometry():
    """The reference's operator interface and pattern (1 x 32640 tokens, 64-token
    key blocks), inputs and output in raster order."""
    from eraserdit_b200.mask_sta import current_mask_sta, mask_sta_window
    geom = sp.REFERENCE_GEOMETRY
    mask = sp.ellipse_masks(geom.grid, seed=3).float().view(1, 1, *geom.grid).cuda()
    q, k, v = _qkv(1, geom.tokens, 2, seed=11)
    with torch.inference_mode(), mask_sta_window(mask, geom.grid) as op:
        assert current_mask_sta() is op
        got = op(q, k, v, 0.125)
        again = op(q, k, v, 0.125)
        report = op.report()
    assert current_mask_sta() is None and op.report()["closed"]
    assert report["calls"] == 2 and 0.3 < report["keep_fraction"] < 0.8
    assert torch.equal(got, again)
    order, _ = sp.tile_order(geom)
    blocks = sp.block_mask(mask.cpu(), geom)
    o = order.cuda()
    want_tiles = masked_attention_fp32(q[:, o], k[:, o], v[:, o], 0.125, blocks, 64)
    want = torch.empty_like(want_tiles)
    want[:, o] = want_tiles
    assert max_abs(got, want) <= MAX_ABS
    assert cosine(got, want) >= MIN_COSINE


def test_config4_layer_against_fp32():
    """The sparse benchmark configuration: 2 x 32640 tokens in tile order, the
    3 x 9 x 9-cell window, ellipse masks; the whole layer against fp32."""
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.mask_sta import SparsePlan
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.synthetic import make_params
    geom = sp.CONFIG4_GEOMETRY
    mask = sp.ellipse_masks(geom.grid, seed=3)
    plan = SparsePlan.from_mask(mask, geom, "cuda")
    p = make_params(1, 1e-6, device="cuda")
    layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda")
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2, geom.tokens, 2048, generator=g, device="cuda").bfloat16()
    rope = LTXVideoRotaryPosEmbed()(*geom.grid)
    got = layer(x, rope, sparse=plan)
    p16 = p.to(torch.bfloat16).to(torch.float32)
    cos, sin = rope.in_order(plan.order).full(2)
    with torch.no_grad():
        xf = x.float()
        q = ref.apply_rotary_emb(ref.rms_norm(torch.nn.functional.linear(xf, p16.wq, p16.bq),
                                              p16.norm_q, 1e-6), cos, sin)
        k = ref.apply_rotary_emb(ref.rms_norm(torch.nn.functional.linear(xf, p16.wk, p16.bk),
                                              p16.norm_k, 1e-6), cos, sin)
        v = torch.nn.functional.linear(xf, p16.wv, p16.bv)
        core = masked_attention_fp32(q.unflatten(2, (32, 64)), k.unflatten(2, (32, 64)),
                                     v.unflatten(2, (32, 64)), 0.125, plan.blocks, 128)
        want = torch.nn.functional.linear(core.flatten(2), p16.wo, p16.bo)
    assert torch.isfinite(got).all()
    assert max_abs(got, want) <= MAX_ABS
    assert cosine(got, want) >= MIN_COSINE


@pytest.mark.parametrize("degree", [2, 8])
def test_sparse_ulysses_emulated(degree):
    """Configuration 4 at SP2 / SP8 (all ranks in one process, same buffers and
    kernels as the NCCL path) against the single-GPU sparse layer."""
    from eraserdit_b200.layer import EraserDiTSelfAttention
    from eraserdit_b200.mask_sta import SparsePlan
    from eraserdit_b200.rotary import LTXVideoRotaryPosEmbed
    from eraserdit_b200.synthetic import make_params
    from eraserdit_b200.ulysses import emulate_ranks
    geom = sp.CONFIG4_GEOMETRY
    plan = SparsePlan.from_mask(sp.ellipse_masks(geom.grid, seed=3), geom, "cuda")
    p = make_params(1, 1e-6, device="cuda")
    layer = EraserDiTSelfAttention.from_params(p.to(torch.bfloat16), device="cuda")
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(2, geom.tokens, 2048, generator=g, device="cuda").bfloat16()
    rope = LTXVideoRotaryPosEmbed()(*geom.grid)
    one = layer(x, rope, sparse=plan)
    parts = emulate_ranks(layer, degree, x, rope, sparse=plan)
    assert [t.shape[1] % 128 for t in parts] == [0] * degree  # whole blocks per rank
    got = torch.cat(parts, dim=1)
    assert max_abs(got, one) <= 1e-2
    assert cosine(got, one) >= 0.99999
