"""Token-axis sharding of Block AttnRes across GPUs (one process per GPU).

Every token ``(b, t)`` is independent for ``out``, ``dv`` and the softmax
(the reference: ``src/switchyard/reference.py:55-57``), so the flattened
``B*T`` axis is split into contiguous ranges, one per rank, and each rank holds
its own ``v[:, range]`` as a ``[N, B_local*T_local, D]`` allocation: no input
exchange and no exchange for ``out`` or ``dv``. The only quantity that crosses
GPUs is the query gradient ``dw = sum over all tokens``: each rank reduces its
own fp32 partial, the D-length rows are all-gathered (8 KiB at D=2048, NCCL
over NVLink on GPUs, gloo in the CPU tests) and every rank adds them in rank
order 0..world-1, so all ranks hold the bitwise-same ``dw`` and the result is
deterministic for a given partition.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .triton_op import DEFAULT_EPS, _backward, _forward, _validate

__all__ = ["token_range", "exchange_dw", "block_attn_res_sharded"]


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
