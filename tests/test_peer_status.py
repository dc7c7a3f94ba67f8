"""Host logic of the peer transport's deferred status checks (no GPU).

A peer-transport call copies its device status word to pinned host memory on
the stream and queues it; ``drain(keep)`` waits for all but the newest
``keep`` queued calls, oldest first, and raises ``SequenceParallelPeerError``
for the first that failed.  The real events, pinned buffers and peer flags are
replaced by stand-ins here.
"""
import pytest
import torch

from eraserdit_b200.ulysses import SequenceParallelPeerError, UlyssesSelfAttention


class _Event:
    def __init__(self, log, name):
        self.log, self.name = log, name

    def synchronize(self):
        self.log.append(self.name)


class _Bufs:
    def __init__(self, flags):
        self.flags = flags

    def view(self, name, count, dtype):
        assert name == "flags"
        t = torch.zeros(count, dtype=dtype)
        t[16:16 + len(self.flags)] = torch.tensor(self.flags, dtype=dtype)
        return t


def _rank(group_ranks=(4, 5, 6, 7)):
    sp = UlyssesSelfAttention.__new__(UlyssesSelfAttention)
    sp.group_ranks = group_ranks
    sp.status_lag = 2
    sp._pending = []
    sp._status_pool = []
    return sp


def _queue(sp, log, name, status, epoch, flags):
    host = torch.tensor([status], dtype=torch.int32)
    sp._pending.append((_Event(log, name), host, _Bufs(flags), epoch, len(flags)))


def test_drain_keeps_the_newest_calls_and_waits_oldest_first():
    sp, log = _rank(), []
    for k in range(1, 4):
        _queue(sp, log, f"call{k}", 0, k, [k] * 4)
    sp.drain(keep=1)
    assert log == ["call1", "call2"]
    assert len(sp._pending) == 1 and len(sp._status_pool) == 2
    sp.drain()
    assert log == ["call1", "call2", "call3"] and not sp._pending


def test_drain_raises_for_the_first_failed_call_and_names_its_ranks():
    sp, log = _rank(), []
    _queue(sp, log, "call1", 0, 1, [1, 1, 1, 1])
    _queue(sp, log, "call2", 0x20, 2, [2, -2, 2, 2])  # group index 1 (rank 5) failed
    _queue(sp, log, "call3", 0, 3, [3, 3, 3, 3])
    with pytest.raises(SequenceParallelPeerError) as info:
        sp.drain(keep=1)
    assert info.value.peer_ranks == (5,)
    assert log == ["call1", "call2"]
    assert len(sp._pending) == 1  # call 3 is still queued for the next drain


def test_drain_names_the_whole_group_when_the_flags_have_moved_on():
    sp, log = _rank((0, 1)), []
    _queue(sp, log, "call1", 0x10, 1, [2, 2])  # flags already hold a later epoch
    with pytest.raises(SequenceParallelPeerError) as info:
        sp.drain()
    assert info.value.peer_ranks == (0, 1)
