"""Ring attention and Ulysses x Ring (USP) sequence parallelism on the B200 kernels.

Mirrors the ring axis of ``DistributedSequenceRank``
(``models/adapters/eraserdit/nccl_sequence.py``): the K/V rotation ``_rotate``
(``:218-233``), the three ring modes of ``attention`` (``:235-332``) and the
Ulysses lengths of a ring group (``:55-56,86-87``); and
``ring_accumulator.piece`` (``layers/attention/ring_accumulator.py:88-100``).

Ranks form a ``ulysses x ring`` grid (``DiTTopology``: ulysses is the faster
axis, so sequence-parallel rank = u + U * r).  The floor partition runs over
all U * R ranks; the U ranks of one ring index hold one contiguous ring piece
of the sequence.  Per layer:

1. QKV projection and the fused norm / RoPE prologue write Q, K and V of the
   local tokens into a send buffer grouped by Ulysses destination
   (``send1[qkv][dest][token][b][head][d]``, H / U heads per destination);
2. three Ulysses exchanges (Q, K, V) deliver the ring piece of this rank's
   ring index for its H / U heads: ``recv_q[src][slot token][b][head][d]``
   and the K / V blocks ``kbuf[piece][src][slot token][b][head][d]``;
3. the ring: K / V blocks travel to ring index r + 1 and arrive from r - 1
   (``_rotate``), in one of three modes
   - ``"reference"``: every piece is kept (``kbuf`` holds all R pieces) and
     ``erd_attn_fwd_ring_bf16`` attends once over the U * R key segments; the
     result is the full-sequence attention, bit for bit the Ulysses result
     at degree U * R;
   - ``"streaming"``: two piece slots; piece t attends with the carried fp32
     softmax state while piece t + 1 rotates on a communication stream;
   - ``"online"``: the reference's flash + log-sum-exp merge mode; here the
     same as ``"streaming"`` (the carried state is already fp32, which is what
     that mode's merge approximates);
4. output rows go to the Ulysses send buffer of their owners and return with
   the inverse exchange; heads are gathered and projected as in Ulysses.

With ``transport="peer"`` steps 2 and 4 become stores over NVLink inside each
Ulysses group, as on the Ulysses path: the prologue writes Q, K and V into the
group peers' receive region, the last attention launch writes rows into the
owners' output-projection input, and epoch flags order the phases; the
rotation stays NCCL.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native
from .attention import _check_operand, validate_bshd_qkv
from .layer import HEAD_DIM, HIDDEN, EraserDiTSelfAttention
from .operator_fusion import qk_norm_rope_into
from .sequence_sharding import floor_bounds, floor_lengths
from .ulysses import FLAG, UlyssesSelfAttention, _Step

RING_MODES = ("reference", "streaming", "online")
STATE_READ, STATE_WRITE = 1, 2


# ------------------------------------------------------------------ kernel calls
def ring_attention_into(q, k, v, out, softmax_scale: float, *, batch: int, heads: int,
                        seg_len: int, q_seg_lens: list[int], kv_seg_len: int,
                        kv_seg_lens: list[int], q_strides, k_strides, v_strides, o_strides,
                        seg_out=None, state: "RingState | None" = None,
                        state_mode: int = 0) -> None:
    """Enqueue ``erd_attn_fwd_ring_bf16`` (strides: token, head, batch, segment).
    ``q``/``k``/``v``/``out`` are tensors or raw device addresses; ``out`` may be
    None when the state is written."""
    lib = _native.load()
    addr = lambda t: t if isinstance(t, int) else (None if t is None else t.data_ptr())
    device = q.device if isinstance(q, torch.Tensor) else torch.device("cuda",
                                                                       torch.cuda.current_device())
    qn, kn = len(q_seg_lens), len(kv_seg_lens)
    qlens = (ctypes.c_int32 * qn)(*q_seg_lens)
    klens = (ctypes.c_int32 * kn)(*kv_seg_lens)
    outs = None if seg_out is None else (ctypes.c_void_p * qn)(*seg_out)
    sbuf, sbytes = (None, 0) if state is None else (state.buffer.data_ptr(), state.nbytes)
    with torch.cuda.device(device):
        rc = lib.erd_attn_fwd_ring_bf16(
            addr(q), addr(k), addr(v), *q_strides, *k_strides, *v_strides, batch, heads, seg_len,
            qn, qlens, kv_seg_len, kn, klens, HEAD_DIM, float(softmax_scale), addr(out),
            *o_strides, outs, sbuf, sbytes, int(state_mode),
            _native.status_word(device).data_ptr(), _native.stream_handle(device))
    _native.check(rc, "erd_attn_fwd_ring_bf16")


class RingState:
    """Carried softmax state of one sequence of ring pieces (device memory:
    unnormalised fp32 O plus the running max and sum of every query row)."""

    def __init__(self, batch: int, heads: int, seg_len: int, q_nseg: int, device) -> None:
        nbytes = int(_native.load().erd_ring_state_bytes(batch, heads, seg_len, q_nseg))
        if nbytes <= 0:
            raise ValueError("invalid ring state shape")
        self.shape = (batch, heads, seg_len, q_nseg)
        self.nbytes = nbytes
        self.buffer = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.pieces = 0


def piece(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: RingState | None = None,
          final: bool = False, scale: float | None = None):
    """Drop-in for ``ring_accumulator.piece``: attend BSHD queries ``q``
    [B, Nq, H, 64] to one piece of keys / values [B, Nk, H, 64] (BF16),
    continuing ``state``.  Returns the state to pass to the next piece, or with
    ``final`` the [B, Nq, H, 64] output over every piece seen."""
    validate_bshd_qkv(q, k, v)
    if q.dtype != torch.bfloat16 or not q.is_cuda or q.shape[-1] != HEAD_DIM:
        raise ValueError("ring pieces need CUDA bfloat16 BSHD tensors with head_dim 64")
    if q.shape[2] != k.shape[2]:
        raise ValueError("ring pieces need equal query and key/value heads")
    batch, nq, heads, _ = q.shape
    nk = k.shape[1]
    if nq == 0 or nk == 0:
        raise ValueError("ring pieces need at least one query and one key")
    for name, t in (("query", q), ("key", k), ("value", v)):
        _check_operand(name, t)
    scale = HEAD_DIM ** -0.5 if scale is None else float(scale)
    first = state is None
    if first and not final:
        state = RingState(batch, heads, nq, 1, q.device)
    if state is not None and state.shape != (batch, heads, nq, 1):
        raise ValueError("the ring state belongs to another query shape")
    mode = (0 if first else STATE_READ) | (0 if final else STATE_WRITE)
    out = torch.empty_like(q, memory_format=torch.contiguous_format) if final else None
    st = lambda t: (t.stride(1), t.stride(2), t.stride(0), 0)
    ring_attention_into(q, k, v, out, scale, batch=batch, heads=heads, seg_len=nq,
                        q_seg_lens=[nq], kv_seg_len=nk, kv_seg_lens=[nk], q_strides=st(q),
                        k_strides=st(k), v_strides=st(v),
                        o_strides=st(out) if final else (0, 0, 0, 0),
                        state=state if mode else None, state_mode=mode)
    if final:
        return out
    state.pieces += 1
    return state


# --------------------------------------------------------------- ring exchange
def ring_rotate(group, ring_ranks: tuple[int, ...], index: int):
    """The reference's ``_rotate`` transfer: send to ring index + 1, receive
    from index - 1, as one batch of point-to-point operations."""
    size = len(ring_ranks)

    def run(sends: list, recvs: list) -> None:
        nxt, prv = ring_ranks[(index + 1) % size], ring_ranks[(index - 1) % size]
        ops = []
        for s, r in zip(sends, recvs):
            ops.append(dist.P2POp(dist.isend, s, nxt, group))
            ops.append(dist.P2POp(dist.irecv, r, prv, group))
        for work in dist.batch_isend_irecv(ops):
            work.wait()
    return run


class UspSelfAttention(UlyssesSelfAttention):
    """One self-attention layer with Ulysses (degree U) x Ring (degree R)
    sequence parallelism; ``rank`` is the Ulysses index and ``ring_rank`` the
    ring index of this process."""

    def __init__(self, layer: EraserDiTSelfAttention, degree: int, rank: int, exchange,
                 ring_degree: int, ring_rank: int, rotate, group_ranks=None,
                 mode: str = "reference", transport: str = "nccl", group=None) -> None:
        super().__init__(layer, degree, rank, exchange, group_ranks=group_ranks, head_chunks=1,
                         transport=transport, group=group)
        if mode not in RING_MODES:
            raise ValueError(f"ring mode must be one of {RING_MODES}")
        if layer.precision != "bf16":
            raise ValueError("ring attention computes in BF16")
        if ring_degree < 1 or not 0 <= ring_rank < ring_degree:
            raise ValueError("ring rank must be inside the ring degree")
        if mode == "reference" and degree * ring_degree > 16:
            raise ValueError("the reference ring mode attends at most 16 key segments")
        self.ring_degree = ring_degree
        self.ring_rank = ring_rank
        self.rotate = rotate
        self.mode = mode
        self.sp_degree = degree * ring_degree
        self.sp_rank = rank + degree * ring_rank
        self._usp: dict[tuple, tuple] = {}
        self._peer_state: dict[tuple, RingState] = {}
        self.calls_ring = 0
        # diagnostics of the reference's rank object (nccl_sequence.py:19-20,262,274,281)
        self.effective_attention = None
        self.partial_attention_dtype = None

    # ------------------------------------------------------------ partition
    def _bounds(self, length: int, rank: int) -> tuple[int, int]:
        return floor_bounds(length, self.sp_degree, rank + self.degree * self.ring_rank)

    def _lengths(self, length: int) -> list[int]:
        """Token counts of this ring index's Ulysses ranks (``nccl_sequence.py:55-56``)."""
        return self.piece_lengths(length, self.ring_rank)

    def piece_lengths(self, length: int, ring_index: int) -> list[int]:
        full = floor_lengths(length, self.sp_degree)
        return full[ring_index * self.degree:(ring_index + 1) * self.degree]

    def partition(self, length: int) -> slice:
        if length < self.sp_degree:
            raise ValueError("sequence length must be at least SP degree")
        self.length = length
        start, end = self._bounds(length, self.rank)
        return slice(start, end)

    def chunks_for(self, length: int) -> int:
        return 1

    # The Ulysses object's single attention launch and its peer phases do not
    # apply to the ring layout; the ring object has its own.
    def _attend(self, step, chunk: int = 0) -> None:
        raise TypeError("UspSelfAttention attends through ring_attention()")

    def peer_pre(self, *args, **kwargs):
        raise TypeError("UspSelfAttention's peer phases are usp_peer_pre/_wait_in/_signal_out/_post")

    peer_attend = peer_post = peer_pre

    def _slots(self) -> int:
        """K/V piece slots: every piece (reference mode) or two (streaming)."""
        return self.ring_degree if self.mode == "reference" else min(2, self.ring_degree)

    def _exchange_slot(self) -> int:
        """The slot the Ulysses exchange fills with this ring index's piece."""
        return self.ring_rank if self.mode == "reference" else 0

    # -------------------------------------------------------------- buffers
    def _usp_buffers(self, batch: int, length: int, device, dtype):
        key = (batch, length, str(device), dtype)
        cached = self._usp.get(key)
        if cached is None:
            n, hl = self.degree, self.local_heads
            lengths = self._lengths(length)
            lmax = max(floor_lengths(length, self.sp_degree))
            row = batch * hl * HEAD_DIM
            lme = lengths[self.rank]
            slots = self._slots()
            send1 = torch.empty(3, n, lme, row, device=device, dtype=dtype)
            # Zeroed once: slot rows past a shorter source's tokens stay finite
            # (zero V rows times zero weights).
            recv_q = torch.zeros(n, lmax, row, device=device, dtype=dtype)
            kbuf = torch.zeros(slots, n, lmax, row, device=device, dtype=dtype)
            vbuf = torch.zeros(slots, n, lmax, row, device=device, dtype=dtype)
            send2 = torch.zeros(1, n, FLAG + lmax * row, device=device, dtype=dtype)
            recv2 = torch.empty(1, n, FLAG + lme * row, device=device, dtype=dtype)
            state = None
            if self.mode != "reference" and self.ring_degree > 1 and device.type == "cuda":
                state = RingState(batch, hl, lmax, n, device)
            cached = (lengths, lmax, send1, recv_q, kbuf, vbuf, send2, recv2, state)
            self._usp[key] = cached
        return cached

    # --------------------------------------------------------------- phases
    def pre(self, x_local: torch.Tensor, rope, length: int) -> _Step:
        """QKV projection + fused norm / RoPE into ``send1[qkv][dest]``."""
        batch = x_local.shape[0]
        bufs = self._usp_buffers(batch, length, x_local.device, x_local.dtype)
        send1 = bufs[2]
        start, end = self._bounds(length, self.rank)
        if x_local.shape[1] != end - start:
            raise ValueError("local sequence length must match the rank's partition")
        qkv = self.layer.project_qkv(x_local)
        q, k, v = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN], qkv[..., 2 * HIDDEN:]
        hl, lme = self.local_heads, end - start
        row = batch * hl * HEAD_DIM
        qk_norm_rope_into(q, k, self.layer.norm_q, self.layer.norm_k, self.layer.eps, rope,
                          send1[0], send1[1], value=v, v_out=send1[2], token_offset=start,
                          out_token_stride=row, out_batch_stride=hl * HEAD_DIM,
                          out_head_stride=HEAD_DIM, heads_per_dest=hl,
                          out_dest_stride=lme * row)
        return self._step(batch, length, bufs)

    def _step(self, batch: int, length: int, bufs: tuple) -> _Step:
        lengths, lmax, send1, recv_q, kbuf, vbuf, send2, recv2, state = bufs
        start, _ = self._bounds(length, self.rank)
        step = _Step(batch, length, lengths, start, send1, recv_q, send2, recv2)
        step.kbuf, step.vbuf, step.state, step.lmax = kbuf, vbuf, state, lmax
        return step

    def attention_pre(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      length: int) -> _Step:
        """Pack this rank's normalised, rotated [B, L_rank, H, 64] Q/K/V into the
        send buffer (``pack_qkv``, ``qkv_packing.py:31-48``)."""
        batch, lme, heads, dim = query.shape
        if heads != self.layer.heads or dim != HEAD_DIM:
            raise ValueError("query must be [B, L_rank, heads, 64]")
        bufs = self._usp_buffers(batch, length, query.device, query.dtype)
        lengths, send1 = bufs[0], bufs[2]
        if lme != lengths[self.rank]:
            raise ValueError("local sequence length must match the rank's partition")
        n, hl = self.degree, self.local_heads
        for i, x in enumerate((query, key, value)):
            # send1[i][dest][token][b][head][d] <- x[b][token][dest * hl + head][d]
            send1[i].view(n, lme, batch, hl, dim).copy_(
                x.view(batch, lme, n, hl, dim).permute(2, 1, 0, 3, 4))
        return self._step(batch, length, bufs)

    def ulysses_in(self, step: _Step) -> list[tuple[list, list]]:
        """(outputs, inputs) of the three Ulysses exchanges (Q, K, V)."""
        n = self.degree
        slot = self._exchange_slot()
        targets = (step.recv1, step.kbuf[slot], step.vbuf[slot])
        return [([targets[i][s, :step.lengths[s]] for s in range(n)],
                 [step.send1[i, d] for d in range(n)]) for i in range(3)]

    def owner(self, hop: int) -> int:
        """Ring index whose piece this rank holds after ``hop`` rotations."""
        return (self.ring_rank - hop) % self.ring_degree

    def ring_pairs(self, step: _Step, hop: int) -> tuple[list, list]:
        """(sends, receives) of rotation ``hop`` (0-based)."""
        if self.mode == "reference":
            src, dst = self.owner(hop), self.owner(hop + 1)
        else:
            src, dst = hop % 2, (hop + 1) % 2
        return [step.kbuf[src], step.vbuf[src]], [step.kbuf[dst], step.vbuf[dst]]

    def _ring_attend(self, step: _Step, hop: int | None) -> None:
        """Attention of the local queries: over every piece (``hop`` None,
        reference mode) or over the piece held after ``hop`` rotations."""
        n, b, hl = self.degree, step.batch, self.local_heads
        row, lmax = b * hl * HEAD_DIM, step.lmax
        strides = (row, HEAD_DIM, hl * HEAD_DIM, lmax * row)
        seg_out = getattr(step, "seg_out", None)
        if seg_out is not None:
            # peer transport: rows straight into the owners' output-projection
            # input, recv2[b][token slot][src][head][d]
            o = None
            o_strides = (n * hl * HEAD_DIM, HEAD_DIM, lmax * n * hl * HEAD_DIM, 0)
        else:
            o = step.send2[0].view(-1)[FLAG:]
            o_strides = (row, HEAD_DIM, hl * HEAD_DIM, FLAG + lmax * row)
        common = dict(batch=b, heads=hl, seg_len=lmax, q_seg_lens=step.lengths, kv_seg_len=lmax,
                      q_strides=strides, k_strides=strides, v_strides=strides,
                      o_strides=o_strides, seg_out=seg_out)
        if hop is None:
            kv_lens = floor_lengths(step.length, self.sp_degree)
            ring_attention_into(step.recv1, step.kbuf, step.vbuf, o, self.layer.softmax_scale,
                                kv_seg_lens=kv_lens, **common)
            return
        last = hop == self.ring_degree - 1
        mode = (STATE_READ if hop > 0 else 0) | (0 if last else STATE_WRITE)
        slot = hop % 2
        ring_attention_into(step.recv1, step.kbuf[slot], step.vbuf[slot], o if last else None,
                            self.layer.softmax_scale,
                            kv_seg_lens=self.piece_lengths(step.length, self.owner(hop)),
                            state=step.state if mode else None, state_mode=mode, **common)

    def ring_attention(self, step: _Step) -> None:
        """The ring phase: rotations and attention launches, every collective
        entered on every rank even after a local failure."""
        events = self.attention_events
        error = None

        def attend(hop):
            nonlocal error
            if error is not None:
                return
            try:
                if events is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                self._ring_attend(step, hop)
                if events is not None:
                    e1.record()
                    events.append((e0, e1))
            except Exception as exc:
                error = exc

        R = self.ring_degree
        if self.mode == "reference":
            self.effective_attention = "b200_ring_gather"
            for hop in range(R - 1):
                self.rotate(*self.ring_pairs(step, hop))
                self.calls_ring += 1
            attend(None)
        elif not step.recv1.is_cuda or R == 1:
            self.effective_attention = "b200_ring_fp32_state"
            self.partial_attention_dtype = "float32_carried_state"
            for hop in range(R):
                attend(hop)
                if hop + 1 < R:
                    self.rotate(*self.ring_pairs(step, hop))
                    self.calls_ring += 1
        else:
            self.effective_attention = "b200_ring_fp32_state"
            self.partial_attention_dtype = "float32_carried_state"
            self._streaming_overlapped(step, attend)
        self.calls += 1
        if error is not None:
            step.failed = True
            raise error

    def _streaming_overlapped(self, step: _Step, attend) -> None:
        """Piece ``hop`` attends on the current stream while piece ``hop + 1``
        rotates on a communication stream; a slot is received into only after
        the attention that read it has finished."""
        device = step.recv1.device
        current = torch.cuda.current_stream(device)
        if self._comm_stream is None:
            self._comm_stream = torch.cuda.Stream(device=device)
        comm = self._comm_stream
        comm.wait_stream(current)  # piece 0 from the Ulysses exchange
        R = self.ring_degree
        done = None
        try:
            for hop in range(R):
                if hop + 1 < R:
                    with torch.cuda.stream(comm):
                        if done is not None:
                            comm.wait_event(done)  # the receive slot was read by hop - 1
                        self.rotate(*self.ring_pairs(step, hop))
                        self.calls_ring += 1
                        arrived = torch.cuda.Event()
                        arrived.record(comm)
                attend(hop)
                done = torch.cuda.Event()
                done.record(current)
                if hop + 1 < R:
                    current.wait_event(arrived)
        finally:
            current.wait_stream(comm)

    # -------------------------------------------------------------- forward
    def _exchange_in(self, step: _Step) -> None:
        for outputs, inputs in self.ulysses_in(step):
            self.exchange(outputs, inputs)

    def _run(self, step: _Step) -> None:
        self._exchange_in(step)
        error = None
        try:
            self.ring_attention(step)
        except Exception as exc:  # every rank still enters the inverse exchange
            error = exc
        step.send2[0, :, :FLAG].fill_(0.0 if error is None else 1.0)
        self.exchange(*self.send_recv_2(step))
        if error is not None:
            raise error

    def forward(self, x_local: torch.Tensor, rope, length: int) -> torch.Tensor:
        """Layer output for this rank's tokens [B, L_rank, 2048]."""
        if self.transport == "peer":
            self.drain(keep=max(self.status_lag, 1) - 1)  # earlier calls' status
            step = self.usp_peer_pre(x_local, rope, length)
            self.usp_peer_wait_in(step)
            ok = True
            try:
                self.ring_attention(step)
            except Exception:  # every rank still signals and waits
                ok = False
            self.usp_peer_signal_out(step, ok)
            return self.usp_peer_post(step, ok)
        step = self.pre(x_local, rope, length)
        self._run(step)
        return self.post(step)

    # ----------------------------------------------------- peer transport
    # The Ulysses exchanges become stores over NVLink (CUDA IPC mappings inside
    # the Ulysses group): the prologue stores Q, K and V into the group peers'
    # recv1 (``recv_q``, and the K / V piece slot this ring index fills), the
    # last attention launch stores rows into the owners' recv2, and the epoch
    # flags of ``peer_exchange`` order the two phases.  The rotation stays a
    # batch of NCCL sends and receives over the ring group.  A rank passes the
    # second wait of call k only after every group peer's rotations and
    # attention of call k (which read and receive into its recv1) are done.

    def peer_buffers(self, batch: int, length: int, device, connect=True):
        from .peer_exchange import PeerBuffers
        key = (batch, length, str(device))
        bufs = self._peer.get(key)
        if bufs is None:
            n, hl = self.degree, self.local_heads
            lmax = max(floor_lengths(length, self.sp_degree))
            row = batch * hl * HEAD_DIM
            # recv1 = recv_q [src][slot token][row] | kbuf [slot][src][...] | vbuf [...];
            # recv2 = [b][token slot][src][head][d], the output projection's input
            sizes = {"recv1": 2 * (1 + 2 * self._slots()) * n * lmax * row,
                     "recv2": 2 * batch * lmax * n * hl * HEAD_DIM}
            bufs = PeerBuffers(sizes, torch.device(device))  # zero-filled
            if connect and self.degree == 1:
                bufs.connect_local([bufs])  # a one-rank Ulysses group stores locally
            elif connect:
                bufs.connect_group(self.group, self.rank, self.degree)
            self._peer[key] = bufs
        return bufs

    def _peer_step(self, bufs, batch: int, length: int) -> _Step:
        n, hl = self.degree, self.local_heads
        lengths = self._lengths(length)
        lmax = max(floor_lengths(length, self.sp_degree))
        row = batch * hl * HEAD_DIM
        slots = self._slots()
        region = bufs.view("recv1", (1 + 2 * slots) * n * lmax * row, torch.bfloat16)
        recv_q = region[:n * lmax * row].view(n, lmax, row)
        kbuf = region[n * lmax * row:(1 + slots) * n * lmax * row].view(slots, n, lmax, row)
        vbuf = region[(1 + slots) * n * lmax * row:].view(slots, n, lmax, row)
        state = self._peer_state.get((batch, length))
        if state is None and self.mode != "reference" and self.ring_degree > 1:
            state = self._peer_state[(batch, length)] = RingState(batch, hl, lmax, n, bufs.device)
        start, _ = self._bounds(length, self.rank)
        step = _Step(batch, length, lengths, start, None, recv_q, None, None)
        step.kbuf, step.vbuf, step.state, step.lmax = kbuf, vbuf, state, lmax
        step.bufs = bufs
        step.seg_out = [bufs.peers["recv2"][s] + 2 * self.rank * hl * HEAD_DIM for s in range(n)]
        return step

    def usp_peer_pre(self, x_local: torch.Tensor, rope, length: int) -> _Step:
        """QKV projection, then the prologue stores Q/K/V into the group peers' recv1."""
        from .operator_fusion import qk_norm_rope_peer_into
        from .peer_exchange import PHASE_IN, signal
        batch = x_local.shape[0]
        n, hl = self.degree, self.local_heads
        start, end = self._bounds(length, self.rank)
        if x_local.shape[1] != end - start:
            raise ValueError("local sequence length must match the rank's partition")
        bufs = self.peer_buffers(batch, length, x_local.device)
        step = self._peer_step(bufs, batch, length)
        self._epoch += 1
        qkv = self.layer.project_qkv(x_local)
        q, k, v = qkv[..., :HIDDEN], qkv[..., HIDDEN:2 * HIDDEN], qkv[..., 2 * HIDDEN:]
        row, lmax, slots = batch * hl * HEAD_DIM, step.lmax, self._slots()
        piece = n * lmax * row  # elements of one Q block or one K/V slot
        slot = self._exchange_slot()
        # our rows in destination d: recv_q[src = this rank], K / V in slot `slot`
        dest = [bufs.peers["recv1"][d] + 2 * self.rank * lmax * row for d in range(n)]
        qk_norm_rope_peer_into(q, k, v, self.layer.norm_q, self.layer.norm_k, self.layer.eps,
                               rope, dest, piece * (1 + slot), piece * (1 + slots + slot),
                               token_offset=start, out_token_stride=row,
                               out_batch_stride=hl * HEAD_DIM, out_head_stride=HEAD_DIM,
                               heads_per_dest=hl)
        signal(bufs, PHASE_IN, self.rank, n, self._epoch, _native.stream_handle(x_local.device))
        return step

    def usp_peer_wait_in(self, step: _Step) -> None:
        from .peer_exchange import PHASE_IN, wait
        device = step.bufs.device
        wait(step.bufs, PHASE_IN, self.degree, self._epoch, _native.status_word(device),
             _native.stream_handle(device))

    def usp_peer_signal_out(self, step: _Step, ok: bool) -> None:
        from .peer_exchange import PHASE_OUT, signal
        signal(step.bufs, PHASE_OUT, self.rank, self.degree, self._epoch if ok else -self._epoch,
               _native.stream_handle(step.bufs.device))

    def usp_peer_post(self, step: _Step, ok: bool) -> torch.Tensor:
        """Wait for every group peer's rows, keep the status for drain(), project."""
        from .peer_exchange import PHASE_OUT, wait
        bufs, n, hl = step.bufs, self.degree, self.local_heads
        device = bufs.device
        word = _native.status_word(device)
        wait(bufs, PHASE_OUT, n, self._epoch, word, _native.stream_handle(device))
        if not ok:
            raise RuntimeError("local sequence-parallel attention failed")
        self._status_to_host(word, bufs, n)
        lme, lmax = step.lengths[self.rank], step.lmax
        heads = bufs.view("recv2", step.batch * lmax * n * hl * HEAD_DIM, torch.bfloat16)
        return self.layer.project_out(heads.view(step.batch, lmax, n * hl * HEAD_DIM)[:, :lme])

    def attention(self, query, key, value, impl=None, metadata=None) -> torch.Tensor:
        """The reference's SP hook with the ring axis (``nccl_sequence.py:235-332``)."""
        if impl is not None and (getattr(impl, "causal", False) or getattr(impl, "dropout", 0)):
            raise ValueError("distributed DiT self-attention requires noncausal SDPA, dropout 0")
        if metadata is not None and getattr(metadata, "attn_mask", None) is not None:
            raise ValueError("distributed DiT self-attention requires an unmasked SDPA")
        length = getattr(self, "length", None)
        if length is None:
            raise RuntimeError("call partition(length) before attention()")
        step = self.attention_pre(query, key, value, length)
        self._run(step)
        return self.gather_heads(step).view(query.shape)

    __call__ = forward


def emulate_usp_ranks(layer: EraserDiTSelfAttention, ulysses: int, ring: int, x: torch.Tensor,
                      rope, mode: str = "reference", transport: str = "nccl"
                      ) -> list[torch.Tensor]:
    """All U x R ranks of the USP layer in one process on one device
    (exchanges and rotations by copies, the same buffers and kernels as the
    NCCL path).  Returns each sequence-parallel rank's output, in rank order
    u + U * r."""
    length = x.shape[1]
    ranks = [UspSelfAttention(layer, ulysses, u, None, ring, r, None, mode=mode,
                              transport=transport)
             for r in range(ring) for u in range(ulysses)]
    at = lambda u, r: ranks[u + ulysses * r]
    if transport == "peer":
        bufs = [usp.peer_buffers(x.shape[0], length, x.device, connect=False) for usp in ranks]
        for r in range(ring):  # IPC-style mappings inside every Ulysses group
            group = bufs[r * ulysses:(r + 1) * ulysses]
            for b in group:
                b.connect_local(group)
        steps = [usp.usp_peer_pre(x[:, usp.partition(length)].contiguous(), rope, length)
                 for usp in ranks]
        for usp, s in zip(ranks, steps):
            usp.usp_peer_wait_in(s)
    else:
        steps = [usp.pre(x[:, usp.partition(length)].contiguous(), rope, length)
                 for usp in ranks]
    for r in range(ring if transport != "peer" else 0):  # Ulysses exchanges per ring index
        for u in range(ulysses):
            for i, (outputs, _) in enumerate(at(u, r).ulysses_in(steps[u + ulysses * r])):
                for src in range(ulysses):
                    outputs[src].copy_(at(src, r).ulysses_in(steps[src + ulysses * r])[i][1][u])

    def rotate_all(hop):
        pairs = [usp.ring_pairs(s, hop) for usp, s in zip(ranks, steps)]
        for idx, usp in enumerate(ranks):
            prev = (usp.ring_rank - 1) % ring
            sends, _ = pairs[usp.rank + ulysses * prev]
            for dst, src in zip(pairs[idx][1], sends):
                dst.copy_(src)

    label = "b200_ring_gather" if mode == "reference" else "b200_ring_fp32_state"
    for usp in ranks:
        usp.effective_attention = label
    if mode == "reference":
        for hop in range(ring - 1):
            rotate_all(hop)
        for usp, s in zip(ranks, steps):
            usp._ring_attend(s, None)
    else:
        for hop in range(ring):
            for usp, s in zip(ranks, steps):
                usp._ring_attend(s, hop)
            if hop + 1 < ring:
                rotate_all(hop)
    if transport == "peer":
        for usp, s in zip(ranks, steps):
            usp.usp_peer_signal_out(s, True)
        outs = [usp.usp_peer_post(s, True) for usp, s in zip(ranks, steps)]
        torch.cuda.synchronize(x.device)
        for usp in ranks:
            usp.close()  # raises a failed peer's error
        return outs
    for usp, s in zip(ranks, steps):
        s.send2[0, :, :FLAG].zero_()
    for r in range(ring):  # inverse Ulysses exchanges
        for u in range(ulysses):
            outputs, _ = at(u, r).send_recv_2(steps[u + ulysses * r])
            for src in range(ulysses):
                outputs[src].copy_(at(src, r).send_recv_2(steps[src + ulysses * r])[1][u])
    return [usp.post(s) for usp, s in zip(ranks, steps)]
