"""Token-axis sharding of Block AttnRes across GPUs (one process per GPU).

Every token ``(b, t)`` is independent for ``out``, ``dv`` and the softmax
(the reference: ``src/switchyard/reference.py:55-57``), so the flattened
``B*T`` axis is split into contiguous ranges, one per rank, and each rank holds
its own ``v[:, range]`` as a ``[N, B_local*T_local, D]`` allocation: no input
exchange and no exchange for ``out`` or ``dv``. The only quantity that crosses
GPUs is the query gradient ``dw = sum over all tokens``: each rank reduces its
own fp32 partial and every rank adds all ranks' partials in rank order
0..world-1, so all ranks hold the bitwise-same ``dw`` and the result is
deterministic for a given partition.

On CUDA ranks the partials cross NVLink as peer stores: one kernel
(``sy_dw_exchange``), launched as a programmatic dependent of the backward,
sums the rank's partial rows and stores each column, with the call's tag in
the same 8-byte word, into every other rank's buffer (torch symmetric memory,
allocated once per group and D); each rank waits, bounded, for the others'
words in its own memory and adds all ranks' rows in rank order -- no NCCL call
and no second launch on the step.
Elsewhere (gloo on CPU, or if peer memory is not available, or with
``SWITCHYARD_DW_EXCHANGE=collective``) the rows are all-gathered with the
process group and summed in the same order, which gives the same bits.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import _native
from .triton_op import DEFAULT_EPS, _backward, _backward_partials, _forward, _validate

__all__ = ["token_range", "exchange_dw", "block_attn_res_sharded", "block_attn_res_batched_sharded",
           "PeerExchange", "PeerExchangeError", "peer_exchange", "device_barrier"]


def token_range(bt: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced ``[start, stop)`` of the flattened token axis owned
    by ``rank``: the first ``bt % world`` ranks get one extra token."""
    if world < 1 or not 0 <= rank < world or bt < 0:
        raise ValueError(f"bad partition request bt={bt} world={world} rank={rank}")
    base, rem = divmod(bt, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def exchange_dw(dw_local: torch.Tensor, group=None) -> torch.Tensor:
    """Sum the ranks' fp32 ``dw`` partials in rank order; identical on every rank."""
    if dw_local.dtype != torch.float32 or dw_local.ndim != 1:
        raise ValueError("dw partial must be a 1-D float32 tensor")
    world = dist.get_world_size(group)
    flat = torch.empty(world * dw_local.numel(), dtype=torch.float32, device=dw_local.device)
    dist.all_gather_into_tensor(flat, dw_local.contiguous(), group=group)
    gathered = flat.view(world, dw_local.numel())
    total = gathered[0].clone()
    for r in range(1, world):
        total += gathered[r]
    return total


#: Bounded wait of the peer exchange, in nanoseconds. A legitimate wait lasts
#: microseconds (the slowest rank's backward tail plus an NVLink round trip);
#: after this long the kernel stops waiting, writes NaN into the gradient,
#: records the device error word and stores the call's tag into the host-visible
#: fail word that the next call checks. ``SWITCHYARD_EXCHANGE_WAIT_S`` overrides
#: the default of 2 s.
EXCHANGE_WAIT_LIMIT_NS = int(float(os.environ.get("SWITCHYARD_EXCHANGE_WAIT_S", "2")) * 1e9)


class PeerExchangeError(RuntimeError):
    """A peer exchange's bounded wait ran out: a rank did not reach the step.
    The gradient of that call is NaN; the exchange is unusable afterwards."""


class PeerExchange:
    """The peer-memory gradient exchange of one (process group, length L,
    device): a buffer every rank can address -- two slots, used alternately, of
    one 8-byte (value, tag) word per (source rank, column) -- and the device
    array of all ranks' addresses of it. Built collectively on first use
    (:func:`peer_exchange`).

    :meth:`reduce_exchange` is one launch (``sy_dw_exchange``): it sums this
    rank's partial rows in ``sy_dw_reduce``'s order, stores them into every
    other rank's buffer, waits in its own buffer for every rank's words
    (bounded) and adds all ranks' sums in rank order.

    Failure handling: if a wait runs out, that call's output is NaN and its tag
    lands in :attr:`fail` (pinned host memory the kernel writes, read by the
    host without a synchronisation). Every call first checks it -- the host
    queues work ahead of the GPU, so a timeout is seen by a later call, and at
    the latest after the next synchronisation -- and then raises
    :class:`PeerExchangeError`; the exchange stays broken, so no later call can
    reuse a slot that a late peer may still be writing into.
    """

    def __init__(self, group, length: int, device: torch.device):
        import torch.distributed._symmetric_memory as symm

        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.length = length
        nbytes = _native.dw_exchange_bytes(length, self.world)
        self.buf = symm.empty(nbytes // 8, dtype=torch.int64, device=device)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, group)
        ptrs = list(self.handle.buffer_ptrs)
        delta = self.buf.data_ptr() - ptrs[self.rank]
        self.bases = torch.tensor([p + delta for p in ptrs], dtype=torch.int64, device=device)
        self.calls = 0
        self.tag = 0
        self.wait_limit_ns = EXCHANGE_WAIT_LIMIT_NS
        self.fail = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.timing = None
        self.broken = None
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every rank's buffer is zero before the first words arrive

    def check(self) -> None:
        """Raise if an earlier call of this exchange timed out (host read of the
        fail word; no synchronisation)."""
        if self.broken is None:
            tag = int(self.fail[0])
            if tag:
                self.broken = (f"switchyard: peer gradient exchange (rank {self.rank} of "
                               f"{self.world}) timed out waiting for a rank at call {tag}; that "
                               "gradient is NaN and the exchange is no longer usable")
        if self.broken is not None:
            raise PeerExchangeError(self.broken)

    def reduce_exchange(self, part: torch.Tensor, out: torch.Tensor) -> None:
        """``out`` [L] (any of the three dtypes) = sum over ranks, in rank
        order, of each rank's fp32 sum of its partial rows ``part`` [P, L]."""
        self.check()
        self.calls += 1
        # 1, 2, ..., 2**32 - 2, 1, ...: never 0 (the zeroed buffer's tag), and
        # the parity, which picks the slot, alternates across the wrap too
        self.tag = (self.calls - 1) % (2**32 - 2) + 1
        _native.dw_exchange(part, self.bases, self.world, self.rank, 0, self.tag, out,
                            self.wait_limit_ns, self.timing, self.fail)

    def start_timing(self) -> None:
        """Count calls and phase nanoseconds from now on (device counters)."""
        self.timing = torch.zeros(8, dtype=torch.int64, device=self.bases.device)

    def read_timing(self) -> dict:
        """Counters since :meth:`start_timing` (synchronises), per call of the
        kernel's first block: mean and largest wait from the end of this
        rank's stores into its peers' buffers until every peer's word of this
        call has arrived in its own; mean time from the kernel's start to the
        end of its sum, and of its phases: the partial-row sum
        (``reduce_mean_us``), the tagged stores into the peers' buffers
        (``announce_mean_us``), and the rank-order sum with the output store
        (``peer_sum_mean_us``)."""
        c = [int(x) for x in self.timing.tolist()]
        k = max(c[0], 1)
        return {"calls": c[0], "wait_mean_us": c[1] / k / 1e3, "wait_max_us": c[2] / 1e3,
                "kernel_mean_us": c[3] / k / 1e3, "reduce_mean_us": c[4] / k / 1e3,
                "announce_mean_us": c[5] / k / 1e3, "peer_sum_mean_us": c[6] / k / 1e3}


_PEER: dict = {}
_PEER_UNAVAILABLE: set = set()


def peer_exchange(group, length: int, device: torch.device):
    """The group's peer exchange for ``length`` columns on ``device`` (built
    collectively on first use), or None where the collective path is used: CPU
    or single-rank groups, ``SWITCHYARD_DW_EXCHANGE=collective``, or no peer
    memory on this system."""
    if device.type != "cuda" or os.environ.get("SWITCHYARD_DW_EXCHANGE") == "collective":
        return None
    world = dist.get_world_size(group)
    if world < 2:
        return None
    gname = (group or dist.group.WORLD).group_name
    key = (gname, length, device.index)
    if key in _PEER_UNAVAILABLE:
        return None
    peer = _PEER.get(key)
    if peer is None:
        try:
            peer = _PEER[key] = PeerExchange(group, length, device)
        except (RuntimeError, ImportError, AttributeError):
            # every rank takes the same branch: the allocation or the
            # rendezvous is unsupported on this system
            _PEER_UNAVAILABLE.add(key)
            return None
    return peer


_BARRIER_LEN = 1  # the barrier's exchange is keyed by this length on its own group key


def device_barrier(group=None, device: torch.device | None = None) -> None:
    """Queue a barrier across the ranks' current CUDA streams: work queued after
    it on any rank starts only once every rank's stream has reached it (one
    single-value peer exchange; bounded wait). The host does not block. Used to
    start ranks' timed regions together."""
    device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    world = dist.get_world_size(group)
    if world < 2:
        return
    gname = (group or dist.group.WORLD).group_name
    key = ("barrier", gname, device.index)
    peer = _PEER.get(key)
    if peer is None:
        peer = _PEER[key] = PeerExchange(group, _BARRIER_LEN, device)
        peer.zero = torch.zeros(1, _BARRIER_LEN, dtype=torch.float32, device=device)
        peer.sink = torch.empty(_BARRIER_LEN, dtype=torch.float32, device=device)
    peer.reduce_exchange(peer.zero, peer.sink)


class _ShardedBlockAttnRes(torch.autograd.Function):
    """Local forward on this rank's tokens; backward adds the ranks' dw."""

    @staticmethod
    def forward(ctx, v_local, w, eps, group):
        _validate(v_local, w)
        v_local, w, out, stats, strategy = _forward(v_local, w, eps)
        ctx.save_for_backward(v_local, w, stats)
        ctx.eps, ctx.group, ctx.strategy = eps, group, strategy
        return out

    @staticmethod
    def backward(ctx, grad_out):
        v, w, stats = ctx.saved_tensors
        peer = peer_exchange(ctx.group, w.shape[0], w.device)
        if peer is not None:
            dv, part = _backward_partials(v, w, stats, grad_out, ctx.eps)
            dw = torch.empty_like(w)
            if part is not None:
                with torch.cuda.device(v.device):
                    peer.reduce_exchange(part, dw)
        else:
            dv, dw32 = _backward(v, w, stats, grad_out, ctx.eps, torch.float32)
            dw = exchange_dw(dw32, ctx.group).to(w.dtype)
        return dv, dw, None, None


def block_attn_res_sharded(v_local: torch.Tensor, w: torch.Tensor, eps: float = DEFAULT_EPS,
                           group=None) -> torch.Tensor:
    """Block AttnRes over this rank's token shard ``v_local [N, B, T_local, D]``.

    Forward is purely local. In backward, ``dv`` stays local and ``w.grad`` is
    the gradient of the full (all-rank) batch, the same on every rank -- what
    data parallelism over the token axis needs. Every rank must call it, in the
    same order, with the same ``w``.
    """
    return _ShardedBlockAttnRes.apply(v_local, w, eps, group)


class _ShardedBatched(torch.autograd.Function):
    """The batched operator on this rank's tokens; backward adds the ranks'
    fp32 query-gradient rows ``[S*D]`` in rank order, through the same
    exchange as ``dw`` (its length is S*D)."""

    @staticmethod
    def forward(ctx, v_local, queries, eps, group):
        from .two_phase import _check_batched

        _check_batched(v_local, queries)
        v_local = v_local.contiguous()
        queries = queries.contiguous()
        n, b, t, d = v_local.shape
        s = queries.shape[0]
        out = torch.empty(s, b, t, d, device=v_local.device, dtype=v_local.dtype)
        if b * t > 0:
            with torch.cuda.device(v_local.device):
                _native.fwd_batched(v_local, queries, out, n, b * t, d, s, eps)
        ctx.save_for_backward(v_local, queries)
        ctx.eps, ctx.group = eps, group
        return out

    @staticmethod
    def backward(ctx, grad_out):
        v, q = ctx.saved_tensors
        n, b, t, d = v.shape
        s = q.shape[0]
        bt = b * t
        g = grad_out.to(v.dtype).contiguous()
        dv = torch.empty_like(v)
        dq = torch.empty_like(q)
        with torch.cuda.device(v.device):
            p = _native.bwd_batched_partials(n, bt, d, s, v.dtype)
            part = torch.empty(p, s * d, device=v.device, dtype=torch.float32)
            _native.bwd_batched(v, q, g, dv, part, n, bt, d, s, ctx.eps)
            peer = peer_exchange(ctx.group, s * d, q.device)
            if peer is not None:
                peer.reduce_exchange(part, dq.view(s * d))
            else:
                dq32 = torch.empty(s * d, device=v.device, dtype=torch.float32)
                _native.dw_reduce(part, dq32)
                dq = exchange_dw(dq32, ctx.group).to(q.dtype).view(s, d)
        return dv, dq, None, None


def block_attn_res_batched_sharded(v_local: torch.Tensor, queries: torch.Tensor,
                                   eps: float = DEFAULT_EPS, group=None) -> torch.Tensor:
    """``S`` queries against this rank's token shard ``v_local [N, B, T_local, D]``
    (the batched training contract, ``switchyard.block_attn_res_batched_train``,
    sharded like :func:`block_attn_res_sharded`): output and ``dv`` stay local,
    ``queries.grad`` is the full-batch gradient, bitwise the same on every rank.
    Every rank must call it, in the same order, with the same ``queries``."""
    from .two_phase import _check_batched, _check_trainable

    _check_batched(v_local, queries)
    _check_trainable(v_local, queries)
    return _ShardedBatched.apply(v_local, queries, eps, group)
