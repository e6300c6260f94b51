"""The decoder's arena staging step, fused.

After every sublayer the reference decoder adds the sublayer's output to the
block's running partial and copies the result into the source arena that the
next Block AttnRes site reads (``src/switchyard/model.py:532-535``)::

    partial = out if partial is None else partial + out
    arena[len(blocks)].copy_(partial)          # under torch.no_grad()

:func:`stage_partial` does the add and the arena write in one kernel
(``sy_stage_partial``): two slabs read and two written in one launch, instead
of three plus two in two launches. The returned partial carries autograd like
``partial + out`` (the add's gradient passes to both inputs unchanged); the
arena write is not part of the graph, as in the reference.
"""

from __future__ import annotations

import torch

from . import _native

__all__ = ["stage_partial"]


class _StagePartial(torch.autograd.Function):
    @staticmethod
    def forward(ctx, partial: torch.Tensor, out: torch.Tensor, arena_slot: torch.Tensor):
        partial = partial.contiguous()
        out = out.contiguous()
        new = torch.empty_like(partial)
        if partial.numel():
            with torch.cuda.device(partial.device):
                _native.stage_partial(partial, out, new, arena_slot)
        ctx.mark_non_differentiable(arena_slot)
        return new

    @staticmethod
    def backward(ctx, grad):
        return grad, grad, None


def stage_partial(partial: torch.Tensor, out: torch.Tensor, arena_slot: torch.Tensor) -> torch.Tensor:
    """Return ``partial + out`` and write it into ``arena_slot`` in the same pass.

    ``partial``, ``out`` and ``arena_slot`` must be CUDA tensors of one shape,
    dtype (bf16, fp16 or fp32) and device; ``arena_slot`` must be contiguous
    (it is written in place, e.g. ``arena[k]`` of a contiguous arena) and must
    not overlap the inputs.
    """
    if partial.shape != out.shape or partial.shape != arena_slot.shape:
        raise ValueError(
            f"partial, out and arena_slot must have one shape, got {tuple(partial.shape)}, "
            f"{tuple(out.shape)}, {tuple(arena_slot.shape)}")
    if not (partial.dtype == out.dtype == arena_slot.dtype):
        raise ValueError("partial, out and arena_slot must have the same dtype")
    if not (partial.is_cuda and out.is_cuda and arena_slot.is_cuda):
        raise ValueError("partial, out and arena_slot must be CUDA tensors")
    if not (partial.device == out.device == arena_slot.device):
        raise ValueError("partial, out and arena_slot must be on the same CUDA device")
    if not arena_slot.is_contiguous():
        raise ValueError("arena_slot must be contiguous")
    _native.dtype_code(partial.dtype)
    return _StagePartial.apply(partial, out, arena_slot)
