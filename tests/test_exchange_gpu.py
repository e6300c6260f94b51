"""The peer gradient exchange (``sy_dw_exchange``) on one GPU: its result, its
bounded wait running out, and what the host sees afterwards.

Two "ranks" are emulated on one GPU by giving the kernel two local buffers as
the ranks' buffers. Only one kernel runs at a time and none waits on a kernel
that has not finished: a call either finds every word it needs already there
(stored by an earlier, completed call or by the test itself) or waits for a
word that nothing will store, which must run out after the short limit the
test passes. Nothing faults and nothing hangs.

Buffer layout (per rank): two slots (tag parity) of ``world * L`` 8-byte words,
word (src, col) = fp32 value of rank ``src`` in the low half, the call's tag in
the high half.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

L, P = 96, 5  # three 32-column blocks, five partial rows
LIMIT_NS = 10_000_000  # 10 ms


@pytest.fixture()
def native():
    from switchyard import _native

    torch.cuda.set_device(0)
    _native.device_error()  # start from a clear error word
    yield _native
    torch.cuda.synchronize()
    _native.device_error()


def _buffers(native, world=2):
    words = native.dw_exchange_bytes(L, world) // 8
    bufs = [torch.zeros(words, dtype=torch.int64, device="cuda") for _ in range(world)]
    bases = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    return bufs, bases


def _slot(buf, tag, world=2):
    """The words of the slot a tag uses, as [world, L] int64."""
    return buf.view(2, world, L)[tag & 1]


def _words(values: torch.Tensor, tag: int) -> torch.Tensor:
    """(value, tag) words for fp32 values."""
    bits = values.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (tag << 32)


def _rows(native, part):
    dw = torch.empty(part.shape[1], dtype=torch.float32, device="cuda")
    native.dw_reduce(part, dw)
    return dw


def test_wait_runs_out_then_the_exchange_recovers(native):
    bufs, bases = _buffers(native)
    g = torch.Generator(device="cuda").manual_seed(5)
    part0 = torch.randn(P, L, device="cuda", generator=g)
    part1 = torch.randn(P, L, device="cuda", generator=g)
    out = torch.empty(L, dtype=torch.float32, device="cuda")
    fail = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    timing = torch.zeros(8, dtype=torch.int64, device="cuda")

    # rank 0, tag 1: rank 1 never stores its words, so every block's wait runs out
    t0 = time.perf_counter()
    native.dw_exchange(part0, bases, 2, 0, 0, 1, out, LIMIT_NS, timing, fail)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 2.0, f"the bounded wait took {elapsed:.3f} s"
    assert torch.isnan(out).all(), "a timed-out exchange must poison its output"
    assert int(fail[0]) == 1, "the fail word must hold the tag of the call that timed out"
    calls, _, wait_max = timing.tolist()[:3]
    assert calls == 1 and wait_max >= LIMIT_NS
    assert native.device_error() & 1, "bit 1 of the device error word: a wait ran out"
    assert native.device_error() == 0  # reading cleared it
    # rank 0 pushed its rows, tagged 1, into rank 1's buffer (row src = 0)
    assert torch.equal(_slot(bufs[1], 1)[0], _words(_rows(native, part0), 1))

    # rank 1, tag 1: rank 0's words are already there, so it completes at once
    # with rank 0's rows added first
    out1 = torch.empty(L, dtype=torch.bfloat16, device="cuda")
    native.dw_exchange(part1, bases, 2, 1, 0, 1, out1, LIMIT_NS)
    torch.cuda.synchronize()
    want = (_rows(native, part0) + _rows(native, part1)).to(torch.bfloat16)
    assert torch.equal(out1, want)
    assert native.device_error() == 0
    assert torch.equal(_slot(bufs[0], 1)[1], _words(_rows(native, part1), 1))

    # rank 0, tag 2, after the error word was cleared: rank 1's words of tag 2
    # are stored by the test, so the call finds them and sums both ranks in
    # rank order
    rows1 = _rows(native, part1) * 3
    _slot(bufs[0], 2)[1].copy_(_words(rows1, 2))
    out2 = torch.empty(L, dtype=torch.float32, device="cuda")
    native.dw_exchange(part0, bases, 2, 0, 0, 2, out2, LIMIT_NS, timing, fail)
    torch.cuda.synchronize()
    assert torch.equal(out2, _rows(native, part0) + rows1)
    assert native.device_error() == 0
    assert timing.tolist()[0] == 2


def test_stale_words_of_another_tag_are_not_taken(native):
    """A word left from two calls earlier (same slot, older tag) is not this
    call's: the wait runs out instead of adding it."""
    bufs, bases = _buffers(native)
    part = torch.ones(P, L, device="cuda")
    _slot(bufs[0], 3)[1].copy_(_words(torch.full((L,), 7.0, device="cuda"), 1))
    out = torch.empty(L, dtype=torch.float32, device="cuda")
    native.dw_exchange(part, bases, 2, 0, 0, 3, out, LIMIT_NS)
    torch.cuda.synchronize()
    assert torch.isnan(out).all()
    assert native.device_error() & 1


def test_sharded_backward_raises_after_a_timeout(native, monkeypatch):
    """The sharded op's backward on a peer exchange whose peer never arrives:
    the first backward's dw is NaN, and the exchange refuses the next call."""
    from switchyard import sharding

    bufs, bases = _buffers(native)
    d = L
    peer = sharding.PeerExchange.__new__(sharding.PeerExchange)
    peer.world, peer.rank, peer.length = 2, 0, d
    peer.buf, peer.bases = bufs[0], bases
    peer.calls, peer.tag, peer.wait_limit_ns = 0, 0, LIMIT_NS
    peer.fail = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    peer.timing, peer.broken = None, None
    monkeypatch.setattr(sharding, "peer_exchange", lambda group, length, device: peer)

    g = torch.Generator(device="cuda").manual_seed(9)
    v = torch.randn(3, 1, 40, d, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(d, device="cuda", generator=g) / d**0.5).to(torch.bfloat16)
    dout = torch.randn(1, 40, d, device="cuda", generator=g).to(torch.bfloat16)

    def step():
        vv = v.detach().requires_grad_(True)
        ww = w.detach().requires_grad_(True)
        sharding.block_attn_res_sharded(vv, ww).backward(dout)
        return vv.grad, ww.grad

    dv, dw = step()
    torch.cuda.synchronize()
    assert torch.isnan(dw.float()).all()
    assert torch.isfinite(dv.float()).all()  # the local gradient is unaffected
    with pytest.raises(sharding.PeerExchangeError, match="timed out"):
        step()
    with pytest.raises(sharding.PeerExchangeError):
        peer.check()  # stays broken
    assert native.device_error() & 1
