"""FP8 attention over the library's static scratch (no allocation in the call)
against erd_attn_fwd_fp8 with a caller-owned workspace, through the C ABI.

Two calls in a row with different shapes and data (the second smaller, so that
stale bytes from the first would show), each within the FP8 path's tolerance
of the workspace entry point; calls after the first allocate nothing (device
free memory and torch's reserved memory unchanged), including an uneven
two-segment shape after a larger call; a shape whose workspace exceeds the
scratch is refused before anything is enqueued."""
import ctypes

import pytest
import torch

from tests.helpers import cosine
from tests.test_fp8_gpu import FP8_MIN_COSINE, _inputs

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 64 << 20  # ERD_FP8_STATIC_SCRATCH_BYTES
ERR_TOO_LARGE = -6


def _strides(t):
    # BSHD contiguous, in elements: token, head, batch, segment
    return (t.stride(1), t.stride(2), t.stride(0), 0)


def _call(lib, name, q, k, v, out, status, extra=()):
    batch, seq, heads, _ = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return getattr(lib, name)(q.data_ptr(), k.data_ptr(), v.data_ptr(), *_strides(q),
                              *_strides(k), *_strides(v), batch, heads, seq, 1, None, 64, 0.125,
                              out.data_ptr(), *_strides(out), *extra, status.data_ptr(), stream)


def _with_workspace(lib, q, k, v):
    batch, seq, heads, _ = q.shape
    nbytes = int(lib.erd_attn_fp8_workspace_bytes(batch, heads, seq, 1))
    ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(lib, "erd_attn_fwd_fp8", q, k, v, out, status,
                 extra=(base, ctypes.c_size_t(nbytes))) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


def test_static_scratch_matches_workspace_entry_twice():
    from eraserdit_b200 import _native
    lib = _native.load()
    cases = [(1, 4096, 4, 1.0, 11), (2, 700, 3, 3.0, 12)]
    for batch, seq, heads, kshift, seed in cases:
        q, k, v = _inputs(batch, seq, heads, seed=seed, kshift=kshift)
        assert int(lib.erd_attn_fp8_workspace_bytes(batch, heads, seq, 1)) <= SCRATCH_BYTES
        out = torch.full_like(q, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert _call(lib, "erd_attn_fwd_fp8_static_scratch", q, k, v, out, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.isfinite(out).all()
        want = _with_workspace(lib, q, k, v)
        assert cosine(out, want) >= FP8_MIN_COSINE


def _free_bytes():
    free, _ = torch.cuda.mem_get_info()
    return free


def _segmented(lib, name, r, seg_len, seg_lens, heads, out, status, extra=()):
    """Self-attention over Q/K/V interleaved per token in `r` [B, nseg*seg_len, 3, H, 64]
    as nseg segments of seg_len slots with seg_lens valid tokens each."""
    batch = r.shape[0]
    nseg = len(seg_lens)
    ts, hs, bs, ss = r.stride(1), r.stride(3), r.stride(0), seg_len * r.stride(1)
    os_ = (out.stride(1), out.stride(2), out.stride(0), seg_len * out.stride(1))
    lens = (ctypes.c_int32 * nseg)(*seg_lens)
    q, k, v = r[:, :, 0], r[:, :, 1], r[:, :, 2]
    stream = torch.cuda.current_stream().cuda_stream
    return getattr(lib, name)(q.data_ptr(), k.data_ptr(), v.data_ptr(), ts, hs, bs, ss,
                              ts, hs, bs, ss, ts, hs, bs, ss, batch, heads, seg_len, nseg, lens,
                              64, 0.125, out.data_ptr(), *os_, *extra, status.data_ptr(), stream)


def test_static_scratch_allocates_nothing_and_serves_uneven_segments():
    """After the first (address-lookup) call, later calls leave the device's
    free memory and torch's reserved memory unchanged; an uneven two-segment
    shape (padding tiles inside segments) that follows a larger call, whose
    bytes are still in the array, matches the workspace entry point."""
    from eraserdit_b200 import _native
    lib = _native.load()
    big = _inputs(1, 4096, 4, seed=21, kshift=2.0)
    out_big = torch.empty_like(big[0])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(lib, "erd_attn_fwd_fp8_static_scratch", *big, out_big, status) == 0
    torch.cuda.synchronize()
    free0, reserved0 = _free_bytes(), torch.cuda.memory_reserved()

    seg_len, seg_lens, heads = 700, [700, 513], 3
    g = torch.Generator(device="cuda").manual_seed(22)
    r = torch.randn(2, 2 * seg_len, 3, heads, 64, generator=g, device="cuda").bfloat16()
    r[:, :, 1] += 1.5  # a shared key offset, as the smoothing removes
    out = torch.full((2, 2 * seg_len, heads, 64), float("nan"), device="cuda",
                     dtype=torch.bfloat16)
    for _ in range(2):
        assert _segmented(lib, "erd_attn_fwd_fp8_static_scratch", r, seg_len, seg_lens, heads,
                          out, status) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.cuda.memory_reserved() == reserved0
        # another process on the device could only lower it; one allocation of
        # ours (2 MiB granularity at least) would show
        assert _free_bytes() >= free0 - (1 << 20)

    nbytes = int(lib.erd_attn_fp8_workspace_bytes(2, heads, seg_len, 2))
    ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 1023) // 1024 * 1024
    want = torch.full_like(out, float("nan"))
    assert _segmented(lib, "erd_attn_fwd_fp8", r, seg_len, seg_lens, heads, want, status,
                      extra=(base, ctypes.c_size_t(nbytes))) == 0
    torch.cuda.synchronize()
    for s, n in enumerate(seg_lens):
        rows = slice(s * seg_len, s * seg_len + n)
        assert torch.isfinite(out[:, rows]).all()
        assert cosine(out[:, rows], want[:, rows]) >= FP8_MIN_COSINE


def test_static_scratch_rejects_oversize_shape():
    from eraserdit_b200 import _native
    lib = _native.load()
    batch, seq, heads = 1, 32640, 32  # one config-1 batch item: about 200 MB of workspace
    assert int(lib.erd_attn_fp8_workspace_bytes(batch, heads, seq, 1)) > SCRATCH_BYTES
    q = torch.zeros(batch, seq, heads, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.full_like(q, 7.0)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(lib, "erd_attn_fwd_fp8_static_scratch", q, q, q, out, status) == ERR_TOO_LARGE
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was enqueued
    assert b"limit" in lib.erd_error_string(ERR_TOO_LARGE)
