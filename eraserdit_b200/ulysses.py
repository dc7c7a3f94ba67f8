"""Ulysses sequence-parallel self-attention over NCCL.

The B200 equivalent of ``DistributedSequenceRank.attention``
(``models/adapters/eraserdit/nccl_sequence.py:43-103,235-332``, Ulysses axis)
wrapped around one EraserDiT self-attention layer
(``models/dits/eraserdit_attention.py:242-290``).  Each of N ranks holds the
floor-partitioned token range of the sequence (``mesh.py:163-169``) and all
2048 channels of its tokens:

1. QKV projection of the local tokens (``erd_linear_bf16``);
2. ``erd_qk_norm_rope`` normalises Q/K across all heads (the norm needs every
   head, so it runs before the exchange), applies 3D RoPE at the tokens'
   global grid positions, and writes Q/K/V straight into the send buffer,
   grouped by destination rank: ``send1[dest][token][qkv][b][head % Hl][d]``
   with Hl = H / N heads per rank (the packing copy of
   ``layers/attention/qkv_packing.py`` disappears into the prologue);
3. all-to-all: rank r receives every source's tokens for its Hl heads into
   ``recv1[src][slot token][qkv][b][hl][d]`` (token-major chunks, so a
   shorter source fills a prefix of its slot);
4. ``erd_attn_fwd_bf16`` attends over the N received segments directly (one
   TMA descriptor, per-segment lengths) and writes each output row into the
   return buffer of its owner: ``send2[dest][flag | token][b][hl][d]``;
5. inverse all-to-all; each chunk carries a leading error flag so that a
   rank whose attention failed is reported by every peer (the protocol of
   ``layers/attention/sequence_parallel.py:257-300``) after all ranks have
   entered both collectives;
6. heads are gathered back per token and ``to_out[0]`` is applied (``erd_linear_bf16``).

The two collectives are the only data-path communication; with CFG the
Ulysses group is one branch's ranks (``eraserdit_b200.topology``).

Head chunks (``head_chunks=C``, the reference's overlap pipeline
``nccl_sequence.py:105-216``): each rank's Hl heads are split into C chunks of
Hl / C.  The prologue writes the send buffer chunk-major
(``send1[dest][chunk][token][qkv][b][head][d]``) so that every (destination,
chunk) block is contiguous; then, on a communication stream, the exchange of
chunk c + 1 runs while chunk c attends on the compute stream, and the finished
chunk c returns while chunk c + 1 attends.  Every rank enqueues the exchanges
in the same order (in 0, in 1, out 0, in 2, out 1, ...).

With ``transport="peer"`` both exchanges become stores into peer memory over
NVLink (``peer_exchange.PeerBuffers``, CUDA IPC mappings): the prologue
writes each head group straight into the destination rank's ``recv1`` slot,
the attention epilogue writes each output row straight into the token owner's
``recv2``, and a release/acquire epoch flag per (rank, phase) orders the
phases (``erd_peer_signal`` / ``erd_peer_wait``, bounded).  No send buffer, no
NCCL call and no unpacking copy remain on the data path.

With a block-sparse plan (``sparse=``) the sequence is in the plan's tile
order, ranks own whole 128-token blocks (a floor partition of the blocks), and
step 4 runs ``erd_attn_fwd_sparse_bf16`` with the plan's lists translated to
the received segments.
"""

from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _native
from .layer import HEAD_DIM, HIDDEN, EraserDiTSelfAttention
from .linear import linear_bf16_scatter
from .operator_fusion import qk_norm_rope_into
from .rotary import RopeAxisTable
from .sequence_sharding import block_bounds, block_lengths, floor_bounds, floor_lengths

FLAG = 8  # elements reserved at the head of every returned chunk (16 bytes)


class SequenceParallelPeerError(RuntimeError):
    """Another rank of the Ulysses group failed between the two exchanges."""

    def __init__(self, peer_ranks: tuple[int, ...]) -> None:
        self.peer_ranks = peer_ranks
        super().__init__("sequence-parallel attention failed on peer rank(s): "
                         + ", ".join(str(r) for r in peer_ranks))


Exchange = Callable[[list, list], None]


def peer_exchange(group, group_ranks: tuple[int, ...], index: int) -> Exchange:
    """All-to-all of per-peer contiguous chunks as one batch of point-to-point
    sends/receives (NCCL runs the batch as one grouped launch; gloo supports it
    too).  ``group_ranks`` are the global ranks of the group, ``index`` this
    rank's position in it."""
    def run(outputs: list, inputs: list) -> None:
        ops = []
        for i, peer in enumerate(group_ranks):
            if i == index:
                outputs[i].copy_(inputs[i])
                continue
            ops.append(dist.P2POp(dist.isend, inputs[i], peer, group))
            ops.append(dist.P2POp(dist.irecv, outputs[i], peer, group))
        if ops:
            for work in dist.batch_isend_irecv(ops):
                work.wait()
    return run


@dataclass
class _Step:
    batch: int
    length: int
    lengths: list
    start: int
    send1: torch.Tensor  # [dest][chunk][token][qkv][b][hc][d]
    recv1: torch.Tensor  # [chunk][src][slot token][qkv][b][hc][d]
    send2: torch.Tensor  # [chunk][dest][FLAG | token][b][hc][d]
    recv2: torch.Tensor  # [chunk][src][FLAG | token][b][hc][d]
    failed: bool = False
    chunks: int = 1


class UlyssesSelfAttention:
    """One self-attention layer with Ulysses sequence parallelism on ``degree`` ranks."""

    def __init__(self, layer: EraserDiTSelfAttention, degree: int, rank: int,
                 exchange: Exchange, group_ranks: tuple[int, ...] | None = None,
                 sparse=None, head_chunks: int | None = None, transport: str = "nccl",
                 group=None) -> None:
        if layer.heads % degree:
            raise ValueError("attention heads must be divisible by Ulysses degree")
        if degree > 16:
            raise ValueError("at most 16 Ulysses ranks (attention segment limit)")
        self.layer = layer
        self.degree = degree
        self.rank = rank
        self.exchange = exchange
        self.group_ranks = group_ranks or tuple(range(degree))
        self.local_heads = layer.heads // degree
        self._buffers: dict[tuple, tuple] = {}
        self.calls = 0
        if sparse is not None and layer.precision != "bf16":
            raise ValueError("the block-sparse path computes in BF16")
        self.sparse = sparse
        self._sparse_segments: dict[int, object] = {}
        self.head_chunks = head_chunks  # None: select_head_chunks per call
        self._comm_stream = None
        # A list here collects (start, end) CUDA events around every attention
        # launch on the stream it is enqueued on (for the benchmark's roofline).
        self.attention_events: list | None = None
        # With the peer transport, a list here collects one dict per call of
        # CUDA events at the phase boundaries (QKV GEMM, prologue + signal,
        # wait for Q/K/V, attention + signal, wait for the rows, output GEMM).
        self.phase_events: list | None = None
        self._marks: dict | None = None
        if transport not in ("nccl", "peer"):
            raise ValueError("transport must be 'nccl' or 'peer'")
        if transport == "peer" and (head_chunks or 1) != 1:
            raise ValueError("the peer transport exchanges all heads at once (one head chunk)")
        self.transport = transport
        self.group = group
        self._peer: dict[tuple, object] = {}
        self._epoch = 0
        # Peer transport: a call's status word is copied to pinned host memory
        # on the stream and inspected ``status_lag`` calls later (or in
        # drain()), so that no host synchronisation sits between consecutive
        # layers: with the default lag of 2 the host enqueues call k + 1 while
        # call k runs, and waits only for call k - 1 to have finished.
        self.status_lag = 2
        # Peer transport: store V from the QKV projection's epilogue (None:
        # use_v_scatter's measured policy).
        self.v_scatter: bool | None = None
        self._pending: list = []
        self._status_pool: list = []

    def _bounds(self, length: int, rank: int) -> tuple[int, int]:
        if self.sparse is not None:
            return block_bounds(length, self.degree, rank)
        return floor_bounds(length, self.degree, rank)

    def _lengths(self, length: int) -> list[int]:
        if self.sparse is not None:
            return block_lengths(length, self.degree)
        return floor_lengths(length, self.degree)

    # ------------------------------------------------------------ partition
    def partition(self, length: int) -> slice:
        if length < self.degree:
            raise ValueError("sequence length must be at least SP degree")
        self.length = length  # the reference hook's contract: attention() follows partition()
        start, end = self._bounds(length, self.rank)
        return slice(start, end)

    def linear_scope(self, model, mode):
        """The reference's hook (``mesh.py:172-270``) pads the projections' GEMM
        rows to keep BF16 results identical across SP degrees; here projections
        run on the local rows only, so the scope changes nothing."""
        del model, mode
        return nullcontext()

    def chunks_for(self, length: int) -> int:
        if self.head_chunks is not None:
            chunks = self.head_chunks
        else:
            chunks = select_head_chunks(self.degree, length, self.local_heads,
                                        sparse=self.sparse is not None)
        if chunks < 1 or self.local_heads % chunks:
            raise ValueError("head chunks must divide the heads per rank")
        return chunks

    def _buffers_for(self, batch: int, length: int, device, dtype, chunks: int = 1):
        key = (batch, length, device, dtype, chunks)
        cached = self._buffers.get(key)
        if cached is None:
            n, hc = self.degree, self.local_heads // chunks
            lengths = self._lengths(length)
            lmax, lme = max(lengths), lengths[self.rank]
            row1 = 3 * batch * hc * HEAD_DIM
            row2 = batch * hc * HEAD_DIM
            send1 = torch.empty(n, chunks, lme, 3, batch, hc, HEAD_DIM, device=device, dtype=dtype)
            # Zeroed once: slot rows past a shorter source's length stay finite.
            recv1 = torch.zeros(chunks, n, lmax, 3, batch, hc, HEAD_DIM, device=device,
                                dtype=dtype)
            send2 = torch.zeros(chunks, n, FLAG + lmax * row2, device=device, dtype=dtype)
            recv2 = torch.empty(chunks, n, FLAG + lme * row2, device=device, dtype=dtype)
            cached = (lengths, send1, recv1, send2, recv2, row1, row2)
            self._buffers[key] = cached
        return cached

    # --------------------------------------------------------------- phases
    def pre(self, x_local: torch.Tensor, rope, length: int) -> _Step:
        """QKV projection + fused norm/RoPE straight into the send buffer."""
        batch = x_local.shape[0]
        chunks = self.chunks_for(length)
        lengths, send1, recv1, send2, recv2, row1, _ = self._buffers_for(
            batch, length, x_local.device, x_local.dtype, chunks)
        start, end = self._bounds(length, self.rank)
        if x_local.shape[1] != end - start:
            raise ValueError("local sequence length must match the rank's partition")
        if (self.sparse is not None and isinstance(rope, RopeAxisTable)
                and rope.grid_index is None):
            rope = rope.in_order(self.sparse.order)
        qkv = self.layer.project_qkv(x_local)
        q, k, v = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN], qkv[..., 2 * HIDDEN:]
        hc = self.local_heads // chunks
        chunk = batch * hc * HEAD_DIM
        base = send1.view(-1)
        # (destination, head chunk) groups are contiguous blocks of L_rank tokens
        qk_norm_rope_into(
            q, k, self.layer.norm_q, self.layer.norm_k, self.layer.eps, rope,
            base[0:], base[chunk:], value=v, v_out=base[2 * chunk:], token_offset=start,
            out_token_stride=row1, out_batch_stride=hc * HEAD_DIM, out_head_stride=HEAD_DIM,
            heads_per_dest=hc, out_dest_stride=(end - start) * row1)
        return _Step(batch, length, lengths, start, send1, recv1, send2, recv2, chunks=chunks)

    def send_recv_1(self, step: _Step, chunk: int = 0) -> tuple[list, list]:
        outputs = [step.recv1[chunk, s, :step.lengths[s]] for s in range(self.degree)]
        inputs = [step.send1[d, chunk] for d in range(self.degree)]
        return outputs, inputs

    def attend(self, step: _Step, chunk: int = 0) -> None:
        """Attention over the received segments; rows go to their owners' chunks."""
        events = self.attention_events
        try:
            if events is not None:
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
            self._attend(step, chunk)
            if events is not None:
                end.record()
                events.append((start, end))
            step.send2[chunk, :, :FLAG].zero_()
        except Exception:
            step.failed = True
            step.send2[chunk, :, :FLAG].fill_(1.0)
            raise
        finally:
            self.calls += 1

    def _attend(self, step: _Step, chunk: int = 0) -> None:
        from .attention import _segmented_call, fp8_workspace
        n, b = self.degree, step.batch
        hc = self.local_heads // step.chunks  # heads of this chunk
        lmax = max(step.lengths)
        row1 = 3 * b * hc * HEAD_DIM  # one received token: q | k | v of every batch and head
        qkv_gap = b * hc * HEAD_DIM   # from q to k (and k to v) inside a received token
        r = step.recv1[chunk].view(-1)
        o = step.send2[chunk].view(-1)[FLAG:]
        strides = (row1, HEAD_DIM, hc * HEAD_DIM, lmax * row1)  # token, head, batch, segment
        o_strides = (qkv_gap, HEAD_DIM, hc * HEAD_DIM, FLAG + lmax * qkv_gap)
        q, k, v = r, r[qkv_gap:], r[2 * qkv_gap:]
        if self.sparse is not None:
            from .mask_sta import sparse_attention_into
            plan = self._sparse_segments.get(step.length)
            if plan is None:
                plan = self.sparse.for_segments([l // 128 for l in step.lengths], lmax // 128)
                self._sparse_segments[step.length] = plan
            sparse_attention_into(q, k, v, o, self.layer.softmax_scale, plan, batch=b, heads=hc,
                                  seg_len=lmax, nseg=n, seg_lens=step.lengths, q_strides=strides,
                                  k_strides=strides, v_strides=strides, o_strides=o_strides)
            return
        fp8 = self.layer.precision == "fp8"
        extra = fp8_workspace(r.device, b, hc, lmax, n) if fp8 else ()
        _segmented_call("erd_attn_fwd_fp8" if fp8 else "erd_attn_fwd_bf16", q, k, v, o,
                        self.layer.softmax_scale, batch=b, heads=hc, seg_len=lmax, nseg=n,
                        seg_lens=step.lengths, q_strides=strides, k_strides=strides,
                        v_strides=strides, o_strides=o_strides, extra=extra)

    def send_recv_2(self, step: _Step, chunk: int = 0) -> tuple[list, list]:
        row2 = step.batch * (self.local_heads // step.chunks) * HEAD_DIM
        outputs = [step.recv2[chunk, s] for s in range(self.degree)]
        inputs = [step.send2[chunk, d, :FLAG + step.lengths[d] * row2]
                  for d in range(self.degree)]
        return outputs, inputs

    def gather_heads(self, step: _Step) -> torch.Tensor:
        """Peer error check and the heads of this rank's tokens, [B, L_rank, 2048]."""
        flags = step.recv2[:, :, 0].float().amax(dim=0)
        if step.failed:
            raise RuntimeError("local sequence-parallel attention failed")
        bad = torch.nonzero(flags != 0).flatten().tolist()
        if bad:
            raise SequenceParallelPeerError(tuple(self.group_ranks[i] for i in bad))
        lme = step.lengths[self.rank]
        n, c, b = self.degree, step.chunks, step.batch
        hc = self.local_heads // c
        # head = source rank * Hl + chunk * Hc + head within the chunk
        heads = step.recv2[:, :, FLAG:].view(c, n, lme, b, hc, HEAD_DIM)
        return heads.permute(3, 2, 1, 0, 4, 5).reshape(b, lme, n * c * hc * HEAD_DIM)

    def post(self, step: _Step) -> torch.Tensor:
        """Peer error check, head gather, output projection."""
        return self.layer.project_out(self.gather_heads(step))

    # ------------------------------------------- attention-level SP hook
    def attention_pre(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      length: int) -> _Step:
        """Pack this rank's normalised, rotated [B, L_rank, H, 64] Q/K/V into the
        send buffer (the reference's ``pack_qkv``, ``qkv_packing.py:31-48``)."""
        batch, lme, heads, dim = query.shape
        if heads != self.layer.heads or dim != HEAD_DIM:
            raise ValueError("query must be [B, L_rank, heads, 64]")
        lengths, send1, recv1, send2, recv2, _, _ = self._buffers_for(
            batch, length, query.device, query.dtype, 1)
        if lme != lengths[self.rank]:
            raise ValueError("local sequence length must match the rank's partition")
        n, hl = self.degree, self.local_heads
        for i, x in enumerate((query, key, value)):
            # send1[dest][0][token][qkv][b][head][d] <- x[b][token][dest * hl + head][d]
            send1[:, 0, :, i] = x.view(batch, lme, n, hl, dim).permute(2, 1, 0, 3, 4)
        start, _ = self._bounds(length, self.rank)
        return _Step(batch, length, lengths, start, send1, recv1, send2, recv2)

    def attention(self, query, key, value, impl=None, metadata=None) -> torch.Tensor:
        """The reference's SP hook (``nccl_sequence.py:235-260``): attention of
        this rank's [B, L_rank, H, 64] queries over the whole sequence; returns
        [B, L_rank, H, 64].  ``partition(length)`` must have been called."""
        if impl is not None and (getattr(impl, "causal", False) or getattr(impl, "dropout", 0)):
            raise ValueError("distributed DiT self-attention requires noncausal SDPA, dropout 0")
        if metadata is not None and getattr(metadata, "attn_mask", None) is not None:
            raise ValueError("distributed DiT self-attention requires an unmasked SDPA")
        length = getattr(self, "length", None)
        if length is None:
            raise RuntimeError("call partition(length) before attention()")
        step = self.attention_pre(query, key, value, length)
        self.exchange(*self.send_recv_1(step))
        error = None
        try:
            self.attend(step)
        except Exception as exc:  # every rank still enters the second exchange
            error = exc
        self.exchange(*self.send_recv_2(step))
        if error is not None:
            raise error
        return self.gather_heads(step).view(query.shape)

    # ----------------------------------------------------- peer transport
    def peer_buffers(self, batch: int, length: int, device, connect=True):
        """This rank's receive buffers for a shape, mapped into the group's
        ranks (collective over ``group`` on first use)."""
        from .peer_exchange import PeerBuffers
        key = (batch, length, str(device))
        bufs = self._peer.get(key)
        if bufs is None:
            lengths = self._lengths(length)
            hl = self.local_heads
            # recv2 is the output projection's input, [b][token slot][src][hl][d]:
            # every source's rows land in place, no head gather follows.
            sizes = {"recv1": 2 * self.degree * max(lengths) * 3 * batch * hl * HEAD_DIM,
                     "recv2": 2 * batch * max(lengths) * self.degree * hl * HEAD_DIM}
            bufs = PeerBuffers(sizes, torch.device(device))
            if connect:
                bufs.connect_group(self.group, self.rank, self.degree)
            self._peer[key] = bufs
        return bufs

    def drain(self, keep: int = 0) -> None:
        """Wait for the peer-transport calls still pending, all but the newest
        ``keep``, oldest first, and raise the error of the first that failed."""
        while len(self._pending) > keep:
            event, host, bufs, epoch, n = self._pending.pop(0)
            event.synchronize()
            status = int(host[0])
            self._status_pool.append(host)
            if status:
                # a later call may have moved the flags on: the ranks whose
                # flag is not this call's epoch are named when it is still there
                flags = bufs.view("flags", 32, torch.int32)[16:16 + n].tolist()
                bad = tuple(self.group_ranks[i] for i, f in enumerate(flags) if f != epoch)
                raise SequenceParallelPeerError(bad or tuple(self.group_ranks))

    def _status_to_host(self, word: torch.Tensor, bufs, n: int) -> None:
        """Copy this call's status word to pinned host memory on the stream,
        clear it, and queue it for drain()."""
        host = (self._status_pool.pop() if self._status_pool
                else torch.empty(1, dtype=torch.int32, pin_memory=True))
        host.copy_(word, non_blocking=True)
        word.zero_()
        event = torch.cuda.Event()
        event.record()
        self._pending.append((event, host, bufs, self._epoch, n))

    def close(self) -> None:
        """Release the peer buffers (after every rank's last call has finished)."""
        try:
            self.drain()
        finally:
            for bufs in self._peer.values():
                bufs.close()
            self._peer = {}

    def _mark(self, name: str) -> None:
        if self._marks is not None:
            event = torch.cuda.Event(enable_timing=True)
            event.record()
            self._marks[name] = event

    def peer_pre(self, x_local: torch.Tensor, rope, length: int):
        """QKV projection, then the prologue stores Q/K/V into the peers' recv1."""
        from .operator_fusion import qk_norm_rope_peer_into
        from .peer_exchange import PHASE_IN, signal
        batch = x_local.shape[0]
        n, hl = self.degree, self.local_heads
        lengths = self._lengths(length)
        lmax = max(lengths)
        start, end = self._bounds(length, self.rank)
        if x_local.shape[1] != end - start:
            raise ValueError("local sequence length must match the rank's partition")
        bufs = self.peer_buffers(batch, length, x_local.device)
        if (self.sparse is not None and isinstance(rope, RopeAxisTable)
                and rope.grid_index is None):
            rope = rope.in_order(self.sparse.order)
        self._epoch += 1
        row1, qkv_gap = 3 * batch * hl * HEAD_DIM, batch * hl * HEAD_DIM
        # our slot in destination d's recv1[src = this rank][slot token][qkv][b][hl][d]
        dest = [bufs.peers["recv1"][d] + 2 * self.rank * lmax * row1 for d in range(n)]
        if (self.v_scatter if self.v_scatter is not None else use_v_scatter(n)) and (
                self.layer.qkv_fp8 is None and x_local.is_contiguous()):
            # V needs no norm: the projection's epilogue stores it straight
            # into the destinations' slots, and the prologue carries Q and K.
            qkv = torch.empty(batch, end - start, 3 * HIDDEN, device=x_local.device,
                              dtype=x_local.dtype)
            linear_bf16_scatter(x_local, self.layer.w_qkv, self.layer.b_qkv, qkv, 2 * HIDDEN,
                                [d + 2 * 2 * qkv_gap for d in dest], hl * HEAD_DIM,
                                hl * HEAD_DIM, row1)
            v = None
        else:
            qkv = self.layer.project_qkv(x_local)
            v = qkv[..., 2 * HIDDEN:]
        self._mark("qkv")
        q, k = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN]
        qk_norm_rope_peer_into(q, k, v, self.layer.norm_q, self.layer.norm_k, self.layer.eps,
                               rope, dest, qkv_gap, 2 * qkv_gap, token_offset=start,
                               out_token_stride=row1, out_batch_stride=hl * HEAD_DIM,
                               out_head_stride=HEAD_DIM, heads_per_dest=hl)
        stream = _native.stream_handle(x_local.device)
        signal(bufs, PHASE_IN, self.rank, n, self._epoch, stream)
        self._mark("prologue")
        return bufs, lengths, batch

    def peer_attend(self, bufs, lengths, batch) -> bool:
        """Wait for every rank's Q/K/V, attend, store rows into the owners' recv2."""
        import ctypes
        from .peer_exchange import PHASE_IN, PHASE_OUT, signal, wait
        n, hl = self.degree, self.local_heads
        lmax = max(lengths)
        device = bufs.device
        stream = _native.stream_handle(device)
        status = _native.status_word(device)
        wait(bufs, PHASE_IN, n, self._epoch, status, stream)
        self._mark("wait_in")
        row1, qkv_gap = 3 * batch * hl * HEAD_DIM, batch * hl * HEAD_DIM
        base = bufs.local["recv1"]
        # this rank's heads of every owner's tokens: owner s's recv2[b][token][self.rank]
        seg_out = (ctypes.c_void_p * n)(*[bufs.peers["recv2"][s] + 2 * self.rank * hl * HEAD_DIM
                                          for s in range(n)])
        lens = (ctypes.c_int32 * n)(*lengths)
        strides = (row1, HEAD_DIM, hl * HEAD_DIM, lmax * row1)
        lib = _native.load()
        events = self.attention_events
        if events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        common = (base, base + 2 * qkv_gap, base + 4 * qkv_gap, *strides, *strides, *strides,
                  batch, hl, lmax, n, lens, HEAD_DIM, float(self.layer.softmax_scale), seg_out,
                  n * hl * HEAD_DIM, HEAD_DIM, lmax * n * hl * HEAD_DIM)
        with torch.cuda.device(device):
            if self.sparse is not None:
                plan = self._sparse_segments.get(sum(lengths))  # keyed by sequence length
                if plan is None:
                    plan = self.sparse.for_segments([l // 128 for l in lengths], lmax // 128)
                    self._sparse_segments[sum(lengths)] = plan
                rc = lib.erd_attn_fwd_sparse_bf16_peer(*common, *plan.launch_args(),
                                                       status.data_ptr(), stream)
            elif self.layer.precision == "fp8":
                from .attention import fp8_workspace
                ws, ws_bytes = fp8_workspace(device, batch, hl, lmax, n)
                rc = lib.erd_attn_fwd_fp8_peer(*common, ws, ws_bytes, status.data_ptr(), stream)
            else:
                rc = lib.erd_attn_fwd_bf16_peer(*common, status.data_ptr(), stream)
        if events is not None:
            e1.record()
            events.append((e0, e1))
        self.calls += 1
        # every rank still signals, a failed one with the negative epoch
        signal(bufs, PHASE_OUT, self.rank, n, self._epoch if rc == 0 else -self._epoch, stream)
        self._mark("attention")
        return rc == 0

    def peer_post(self, bufs, lengths, batch, ok: bool) -> torch.Tensor:
        """Wait for every rank's rows, check the status, gather heads, project."""
        from .peer_exchange import PHASE_OUT, wait
        n, hl = self.degree, self.local_heads
        device = bufs.device
        word = _native.status_word(device)
        wait(bufs, PHASE_OUT, n, self._epoch, word, _native.stream_handle(device))
        self._mark("wait_out")
        if not ok:
            raise RuntimeError("local sequence-parallel attention failed")
        self._status_to_host(word, bufs, n)  # inspected by a later call's drain()
        lme, lmax = lengths[self.rank], max(lengths)
        heads = bufs.view("recv2", batch * lmax * n * hl * HEAD_DIM, torch.bfloat16)
        return self.layer.project_out(heads.view(batch, lmax, n * hl * HEAD_DIM)[:, :lme])

    def _forward_peer(self, x_local: torch.Tensor, rope, length: int) -> torch.Tensor:
        self.drain(keep=max(self.status_lag, 1) - 1)  # earlier calls' status (complete by now)
        self._marks = {} if self.phase_events is not None else None
        self._mark("start")
        bufs, lengths, batch = self.peer_pre(x_local, rope, length)
        ok = self.peer_attend(bufs, lengths, batch)
        out = self.peer_post(bufs, lengths, batch, ok)
        if self._marks is not None:
            self._mark("out_proj")
            self.phase_events.append(self._marks)
            self._marks = None
        return out

    # -------------------------------------------------------------- forward
    def forward(self, x_local: torch.Tensor, rope, length: int) -> torch.Tensor:
        """Layer output for this rank's tokens [B, L_rank, 2048]."""
        if self.transport == "peer":
            return self._forward_peer(x_local, rope, length)
        step = self.pre(x_local, rope, length)
        if step.chunks > 1 and x_local.is_cuda:
            return self._forward_pipelined(step)
        error = None
        for c in range(step.chunks):
            out1, in1 = self.send_recv_1(step, c)
            self.exchange(out1, in1)
            try:
                self.attend(step, c)
            except Exception as exc:  # every rank still enters the second exchange
                error = error or exc
            out2, in2 = self.send_recv_2(step, c)
            self.exchange(out2, in2)
        if error is not None:
            raise error
        return self.post(step)

    def _forward_pipelined(self, step: _Step) -> torch.Tensor:
        """Exchanges on a communication stream, attention on the current one:
        in(c + 1) and out(c) overlap attend(c + 1) / attend(c)."""
        device = step.send1.device
        current = torch.cuda.current_stream(device)
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device=device)
        comm = self._comm_stream
        comm.wait_stream(current)  # send buffers written by the prologue

        def exchange_in(c):
            with torch.cuda.stream(comm):
                self.exchange(*self.send_recv_1(step, c))
                ready = torch.cuda.Event()
                ready.record(comm)
            return ready

        error = None
        try:
            ready = exchange_in(0)
            for c in range(step.chunks):
                current.wait_event(ready)
                try:
                    self.attend(step, c)
                except Exception as exc:  # every rank still enters every exchange
                    error = error or exc
                done = torch.cuda.Event()
                done.record(current)
                if c + 1 < step.chunks:
                    ready = exchange_in(c + 1)
                with torch.cuda.stream(comm):
                    comm.wait_event(done)
                    self.exchange(*self.send_recv_2(step, c))
        finally:
            current.wait_stream(comm)
        if error is not None:
            raise error
        return self.post(step)

    __call__ = forward


def use_v_scatter(degree: int) -> bool:
    """Whether the peer transport's QKV projection stores V into the peers'
    slots from its epilogue (``erd_linear_bf16_scatter``, 128-byte row pieces
    staged through shared memory) instead of the prologue copying it.
    Measured per layer (QKV GEMM + prologue, same box, with / without): 2 ranks
    0.830 / 0.903 ms, 8 ranks 0.286-0.295 / 0.317-0.322 ms (3.434 / 3.465 ms a
    layer)."""
    del degree
    return True


def select_head_chunks(degree: int, length: int, local_heads: int, *, sparse: bool = False) -> int:
    """Head chunks of the overlap pipeline for one Ulysses layer call.

    Mirrors ``layers/attention/ulysses_policy.py:5-17``: a measured policy that
    depends only on shapes, so that every rank takes the same collective steps.
    Measured on 8 B200s at 2 x 32640 tokens (ms per layer, 1 / 2 / 4 chunks):
    SP2 14.14 / 14.04 / 14.42, SP4 7.34 / 7.26 / 7.84, SP8 3.94 / 4.23 / 4.20,
    SP8 sparse 1.92 / 1.91, SP4 FP8 8.59 / 8.68.  The exchanges are 5-8 % of a
    layer over NVLink, so overlapping them gains at most 1 %, and smaller
    attention launches (fewer heads per chunk) lose more than that at SP8: one
    exchange per direction everywhere.
    """
    del degree, length, local_heads, sparse
    return 1


def emulate_attention_hook(layer: EraserDiTSelfAttention, degree: int, q: torch.Tensor,
                           k: torch.Tensor, v: torch.Tensor) -> list[torch.Tensor]:
    """All ranks of the attention-level hook in one process (chunks exchanged
    by copies); q/k/v are the full [B, S, H, 64] tensors, each rank gets its
    slice.  Returns every rank's [B, L_rank, H, 64] output."""
    length = q.shape[1]
    ranks = [UlyssesSelfAttention(layer, degree, r, exchange=None) for r in range(degree)]
    steps = []
    for r in ranks:
        sl = r.partition(length)
        steps.append(r.attention_pre(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                     v[:, sl].contiguous(), length))

    def all_to_all(pairs):
        for dst in range(degree):
            outputs, _ = pairs[dst]
            for src in range(degree):
                outputs[src].copy_(pairs[src][1][dst])

    all_to_all([r.send_recv_1(s) for r, s in zip(ranks, steps)])
    for r, s in zip(ranks, steps):
        r.attend(s)
    all_to_all([r.send_recv_2(s) for r, s in zip(ranks, steps)])
    return [r.gather_heads(s).view(q.shape[0], -1, q.shape[2], 64) for r, s in zip(ranks, steps)]


def emulate_ranks(layer: EraserDiTSelfAttention, degree: int, x: torch.Tensor, rope,
                  sparse=None, head_chunks: int | None = None, transport: str = "nccl",
                  v_scatter: bool | None = None) -> list[torch.Tensor]:
    """Run all ``degree`` ranks of the Ulysses layer inside one process on one
    device, exchanging chunks by copies (the same buffers and kernels as the
    NCCL path).  Returns each rank's output; used to check the data layout on
    a single GPU."""
    length = x.shape[1]
    ranks = [UlyssesSelfAttention(layer, degree, r, exchange=None, sparse=sparse,
                                  head_chunks=head_chunks, transport=transport)
             for r in range(degree)]
    for r in ranks:
        r.v_scatter = v_scatter
    if transport == "peer":
        # every phase of every rank is enqueued before any rank waits on it
        bufs = [r.peer_buffers(x.shape[0], length, x.device, connect=False) for r in ranks]
        for b in bufs:
            b.connect_local(bufs)
        pre = [r.peer_pre(x[:, r.partition(length)].contiguous(), rope, length) for r in ranks]
        oks = [r.peer_attend(*args) for r, args in zip(ranks, pre)]
        outs = [r.peer_post(*args, ok) for r, args, ok in zip(ranks, pre, oks)]
        torch.cuda.synchronize(x.device)
        for r in ranks:
            r.close()  # raises a failed peer's error
        return outs
    steps = []
    for r in ranks:
        sl = r.partition(length)
        steps.append(r.pre(x[:, sl].contiguous(), rope, length))

    def all_to_all(pairs):
        for dst in range(degree):
            outputs, _ = pairs[dst]
            for src in range(degree):
                outputs[src].copy_(pairs[src][1][dst])

    for c in range(steps[0].chunks):
        all_to_all([r.send_recv_1(s, c) for r, s in zip(ranks, steps)])
        for r, s in zip(ranks, steps):
            r.attend(s, c)
        all_to_all([r.send_recv_2(s, c) for r, s in zip(ranks, steps)])
    return [r.post(s) for r, s in zip(ranks, steps)]
