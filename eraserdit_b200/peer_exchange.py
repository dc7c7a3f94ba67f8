"""Peer-memory buffers for the Ulysses exchanges over NVLink.

The reference moves Q/K/V and the attention output with two NCCL
all-to-alls (``nccl_sequence.py:43-103``).  Here each rank owns its receive
buffers (allocated with ``erd_peer_alloc``) and maps every peer's with CUDA
IPC (``erd_peer_ipc_handle`` / ``erd_peer_ipc_open``; the handles travel once
through the process group).  The prologue and the attention epilogue then
store straight into the peers' buffers, and ``erd_peer_signal`` /
``erd_peer_wait`` order each phase with one epoch flag per (rank, phase):
flags live in the receiver's memory, ``[phase][source rank]`` int32.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native

FLAG_BYTES = 256  # [2 phases][up to 16 ranks] int32, padded
PHASE_IN, PHASE_OUT = 0, 1


class _CudaArray:
    """Zero-copy view of raw device memory for ``torch.as_tensor``."""

    def __init__(self, ptr: int, numel: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def tensor_at(ptr: int, numel: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A 1-D tensor over ``numel`` elements at device address ``ptr`` (not owned)."""
    typestr = {torch.bfloat16: "<u2", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    t = torch.as_tensor(_CudaArray(ptr, numel, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _alloc(nbytes: int) -> int:
    out = ctypes.c_void_p()
    _native.check(_native.load().erd_peer_alloc(nbytes, ctypes.byref(out)), "erd_peer_alloc")
    return int(out.value)


class PeerBuffers:
    """One rank's receive buffers (``recv1``, ``recv2``, ``flags``) and the
    device addresses of every rank's copies of them."""

    NAMES = ("recv1", "recv2", "flags")

    def __init__(self, sizes: dict, device: torch.device) -> None:
        self.device = device
        self.sizes = dict(sizes, flags=FLAG_BYTES)
        with torch.cuda.device(device):
            self.local = {name: _alloc(self.sizes[name]) for name in self.NAMES}
        self.peers: dict[str, list[int]] = {}
        self._opened: list[int] = []

    def handles(self) -> dict:
        lib = _native.load()
        out = {}
        for name in self.NAMES:
            h = ctypes.create_string_buffer(64)
            _native.check(lib.erd_peer_ipc_handle(self.local[name], h), "erd_peer_ipc_handle")
            out[name] = h.raw
        return out

    def connect_group(self, group, index: int, size: int) -> None:
        """Exchange IPC handles over ``group`` (collective) and map the peers'."""
        mine = self.handles()
        gathered = [None] * size
        dist.all_gather_object(gathered, mine, group=group)
        lib = _native.load()
        self.peers = {name: [] for name in self.NAMES}
        with torch.cuda.device(self.device):
            for r, theirs in enumerate(gathered):
                for name in self.NAMES:
                    if r == index:
                        self.peers[name].append(self.local[name])
                        continue
                    ptr = ctypes.c_void_p()
                    h = ctypes.create_string_buffer(theirs[name], 64)
                    _native.check(lib.erd_peer_ipc_open(h, ctypes.byref(ptr)), "erd_peer_ipc_open")
                    self.peers[name].append(int(ptr.value))
                    self._opened.append(int(ptr.value))

    def connect_local(self, all_buffers: list["PeerBuffers"]) -> None:
        """Single-process emulation: the 'peers' are other objects' local buffers."""
        self.peers = {name: [b.local[name] for b in all_buffers] for name in self.NAMES}

    def view(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        return tensor_at(self.local[name], numel, dtype, self.device)

    def close(self) -> None:
        """Unmap peers and free this rank's buffers.  Every rank of the group
        must have finished its exchanges (callers synchronise first)."""
        lib = _native.load()
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                lib.erd_peer_ipc_close(ptr)
            self._opened = []
            for name in self.NAMES:
                if self.local.get(name):
                    lib.erd_peer_free(self.local[name])
            self.local = {}
        self.peers = {}


def signal(bufs: PeerBuffers, phase: int, index: int, n: int, epoch: int, stream: int) -> None:
    """Store ``epoch`` in every rank's flag slot [phase][index]."""
    lib = _native.load()
    slots = (ctypes.c_void_p * n)(*[bufs.peers["flags"][r] + 4 * (phase * 16 + index)
                                    for r in range(n)])
    _native.check(lib.erd_peer_signal(slots, n, epoch, stream), "erd_peer_signal")


def wait(bufs: PeerBuffers, phase: int, n: int, epoch: int, status: torch.Tensor, stream: int,
         timeout_ns: int = 2_000_000_000) -> None:
    """Enqueue the bounded wait for every rank's ``epoch`` in our flags [phase]."""
    lib = _native.load()
    _native.check(lib.erd_peer_wait(bufs.local["flags"] + 4 * phase * 16, n, epoch, timeout_ns,
                                    status.data_ptr(), stream), "erd_peer_wait")
