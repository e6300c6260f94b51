"""Host logic of the peer gradient exchange (``switchyard.sharding.PeerExchange``)
on the CPU: the tag sequence the kernel relies on and the failure bookkeeping.
The kernel call is replaced by a recorder; nothing touches a GPU.
"""

from __future__ import annotations

import pytest
import torch

from switchyard import sharding


def _peer(monkeypatch, calls):
    peer = sharding.PeerExchange.__new__(sharding.PeerExchange)
    peer.world, peer.rank, peer.length = 2, 0, 8
    peer.bases = torch.zeros(2, dtype=torch.int64)
    peer.calls, peer.tag, peer.wait_limit_ns = 0, 0, 1000
    peer.fail = torch.zeros(1, dtype=torch.int32)
    peer.timing, peer.broken = None, None

    def record(part, bases, world, rank, buf_off, tag, out, limit, timing, fail):
        calls.append(tag)

    monkeypatch.setattr(sharding._native, "dw_exchange", record)
    return peer


def test_tags_start_at_one_alternate_parity_and_skip_zero_on_wrap(monkeypatch):
    calls = []
    peer = _peer(monkeypatch, calls)
    part, out = torch.zeros(1, 8), torch.zeros(8)
    for _ in range(4):
        peer.reduce_exchange(part, out)
    assert calls == [1, 2, 3, 4]
    # jump to the end of the 32-bit range: ..., 2**32 - 3, 2**32 - 2, then 1 again
    peer.calls = 2**32 - 5
    for _ in range(4):
        peer.reduce_exchange(part, out)
    assert calls[4:] == [2**32 - 4, 2**32 - 3, 2**32 - 2, 1]
    assert 0 not in calls
    # the slot (tag parity) alternates on every call, across the wrap too
    parities = [t & 1 for t in calls[4:]]
    assert all(a != b for a, b in zip(parities, parities[1:]))


def test_a_recorded_timeout_raises_and_the_exchange_stays_broken(monkeypatch):
    calls = []
    peer = _peer(monkeypatch, calls)
    part, out = torch.zeros(1, 8), torch.zeros(8)
    peer.reduce_exchange(part, out)
    peer.fail[0] = 1  # what the kernel stores when a wait ran out at tag 1
    with pytest.raises(sharding.PeerExchangeError, match="call 1"):
        peer.reduce_exchange(part, out)
    peer.fail[0] = 0
    with pytest.raises(sharding.PeerExchangeError):
        peer.reduce_exchange(part, out)  # no later call goes out
    assert calls == [1]


def test_single_rank_and_cpu_groups_take_no_peer_exchange(monkeypatch):
    monkeypatch.setattr(sharding.dist, "get_world_size", lambda group=None: 1)
    assert sharding.peer_exchange(None, 8, torch.device("cuda", 0)) is None
    assert sharding.peer_exchange(None, 8, torch.device("cpu")) is None
    monkeypatch.setenv("SWITCHYARD_DW_EXCHANGE", "collective")
    monkeypatch.setattr(sharding.dist, "get_world_size", lambda group=None: 2)
    assert sharding.peer_exchange(None, 8, torch.device("cuda", 0)) is None
