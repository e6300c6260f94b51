"""The batched training contract and the two-phase schedule on the GPU.

The reference's batched API is output-only: it returns no merge statistics and
raises on ``requires_grad`` (``src/switchyard/triton_op.py:438-501``,
``README.md:63-70``); completing it is the reference's own next item
(``PROJECT_STATE.md:74-75``). The paper's two-phase schedule needs both: each
phase returns ``(o, m, ell)`` (``attn_with_stats``,
``src/switchyard/reference.py:195-216``) and the phases are combined by an
exact online-softmax merge (``merge_online_softmax``, ``reference.py:219-233``).

This module provides, through the C ABI:

* :func:`attn_with_stats` -- ``(o, m, ell)`` for one query ``w`` ``[D]`` or for
  ``S`` queries ``[S, D]``, from one read of ``v`` (``sy_fwd_batched_stats``
  with ``raw = 1``: the kernel skips the division by ``ell``);
* :func:`merge_online_softmax` -- the merge of two triples in one pass
  (``sy_merge_stats``), optionally finishing with ``o / ell``;
* :func:`block_attn_res_batched_train` -- the batched operator with autograd
  (the ``sy_fwd_batched`` forward; ``sy_bwd_batched`` recomputes the dot
  products and softmax from ``v``, and the fixed-order ``sy_dw_reduce`` sums
  the queries' gradient).

``block_attn_res_batched`` itself keeps the reference's behaviour (output only,
``RuntimeError`` on ``requires_grad``) so the reference's tests pass unchanged.
The statistics functions are forward-only; gradients of a merged result are
those of the single-pass operator over the union of the sources, which
``block_attn_res_triton`` and :func:`block_attn_res_batched_train` compute.
"""

from __future__ import annotations

import math

import torch

from . import _native
from .triton_op import DEFAULT_EPS
from .triton_op import _BlockAttnResTriton as _BlockAttnResTritonFn

__all__ = ["attn_with_stats", "merge_online_softmax", "block_attn_res_batched_train"]


def _check_batched(v: torch.Tensor, queries: torch.Tensor) -> None:
    # Same checks and messages as block_attn_res_batched
    # (src/switchyard/triton_op.py:463-474).
    if v.ndim != 4:
        raise ValueError(f"v must be [N, B, T, D], got {tuple(v.shape)}")
    if queries.ndim != 2 or queries.shape[1] != v.shape[-1]:
        raise ValueError(f"queries must be [S, {v.shape[-1]}], got {tuple(queries.shape)}")
    if not v.is_cuda or not queries.is_cuda:
        raise ValueError("v and queries must be CUDA tensors")
    if v.device != queries.device:
        raise ValueError("v and queries must be on the same CUDA device")
    if v.dtype != queries.dtype:
        raise ValueError("v and queries must have the same dtype")
    if v.shape[0] == 0 or queries.shape[0] == 0 or v.shape[-1] == 0:
        raise ValueError("N, S, and D must be positive")
    _native.dtype_code(v.dtype)


#: Queries the batched backward takes (``sy_bwd_batched``); the forward takes any number.
BATCHED_TRAIN_MAX_QUERIES = 16


def _check_trainable(v: torch.Tensor, queries: torch.Tensor) -> None:
    """Refuse, before the forward runs, a batched call whose backward could not
    run: more than BATCHED_TRAIN_MAX_QUERIES queries while a gradient is wanted."""
    wants_grad = torch.is_grad_enabled() and (v.requires_grad or queries.requires_grad)
    if wants_grad and queries.shape[0] > BATCHED_TRAIN_MAX_QUERIES:
        raise ValueError(
            f"the batched backward takes at most {BATCHED_TRAIN_MAX_QUERIES} queries, got "
            f"{queries.shape[0]}; split the queries, or run the forward under torch.no_grad()")


def _forward_stats(v: torch.Tensor, queries: torch.Tensor, eps: float, raw: bool):
    """One launch: out ``[S, B, T, D]`` (normalised, or unnormalised when
    ``raw``) and the fp32 statistics ``[S, B*T, 2]`` = (max logit, sum of
    exponentials)."""
    n, b, t, d = v.shape
    s = queries.shape[0]
    out = torch.empty(s, b, t, d, device=v.device, dtype=v.dtype)
    mstats = torch.empty(s, b * t, 2, device=v.device, dtype=torch.float32)
    if b * t > 0:
        with torch.cuda.device(v.device):
            _native.fwd_batched_stats(v, queries, out, mstats, raw, n, b * t, d, s, eps)
    return out, mstats


def attn_with_stats(v: torch.Tensor, w: torch.Tensor, eps: float = DEFAULT_EPS):
    """``ATTNWITHSTATS`` of the paper's Algorithm 1 on the GPU.

    Same contract as ``attn_with_stats`` (``src/switchyard/reference.py:195-216``):
    for ``w`` of shape ``[D]`` returns ``(o [B, T, D], m [B, T], ell [B, T])``
    with ``m`` the max logit, ``ell = sum_n exp(logit_n - m)`` and the
    unnormalised ``o = sum_n exp(logit_n - m) v_n`` in ``v``'s dtype, so that
    ``o / ell`` is the operator's output. For ``w`` of shape ``[S, D]`` (S
    queries) every output gains a leading ``S`` axis. ``m`` and ``ell`` are
    fp32. Forward only.
    """
    if v.requires_grad or w.requires_grad:
        raise RuntimeError(
            "attn_with_stats has no backward; train through block_attn_res_triton or "
            "block_attn_res_batched_train, or run this under torch.no_grad()"
        )
    single = w.ndim == 1
    queries = w.unsqueeze(0) if single else w
    _check_batched(v, queries)
    v = v.contiguous()
    queries = queries.contiguous()
    _, b, t, _ = v.shape
    o, mstats = _forward_stats(v, queries, eps, raw=True)
    s = queries.shape[0]
    m = mstats[..., 0].reshape(s, b, t)
    ell = mstats[..., 1].reshape(s, b, t)
    if single:
        return o[0], m[0], ell[0]
    return o, m, ell


def _contiguous_strides(shape) -> tuple:
    strides, acc = [], 1
    for n in reversed(shape):
        strides.append(acc)
        acc *= n
    return tuple(reversed(strides))


def _pairs(m: torch.Tensor, ell: torch.Tensor, rows: int) -> torch.Tensor:
    """The statistics as one fp32 ``[rows, 2]`` tensor of (m, ell) pairs. The
    views :func:`attn_with_stats` returns already are that buffer (ell one
    float after m, both with every stride doubled): it is used in place, with
    no copy kernel; any other pair of tensors is stacked."""
    if (m.dtype == ell.dtype == torch.float32 and m.device == ell.device
            and ell.data_ptr() == m.data_ptr() + 4 and m.stride() == ell.stride()
            and m.stride() == tuple(2 * x for x in _contiguous_strides(m.shape))):
        return m.as_strided((rows, 2), (2, 1))
    return torch.stack((m.float(), ell.float()), -1).reshape(rows, 2)


def merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize: bool = False):
    """Combine two ``(o, m, ell)`` triples over disjoint source groups, exactly.

    Same contract as ``merge_online_softmax`` (``src/switchyard/reference.py:219-233``):
    ``m = max(m1, m2)``, ``s_i = exp(m_i - m)``, ``o = o1 s1 + o2 s2``,
    ``ell = l1 s1 + l2 s2``, with ``o`` in ``o1``'s dtype and ``m``, ``ell`` in
    fp32, one kernel pass over the two ``o`` slabs. With ``normalize=True`` the
    returned ``o`` is already divided by ``ell`` (the finished output of the
    two-phase schedule, one pass fewer). Forward only.
    """
    if any(x.requires_grad for x in (o1, m1, l1, o2, m2, l2)):
        raise RuntimeError("merge_online_softmax has no backward; run it under torch.no_grad()")
    if o1.shape != o2.shape or o1.dtype != o2.dtype:
        raise ValueError("o1 and o2 must have the same shape and dtype")
    lead = o1.shape[:-1]
    for x in (m1, l1, m2, l2):
        if x.shape != lead:
            raise ValueError(f"statistics must have shape {tuple(lead)}, got {tuple(x.shape)}")
    if not all(x.is_cuda and x.device == o1.device for x in (o1, m1, l1, o2, m2, l2)):
        raise ValueError("every input must be a CUDA tensor on the same device")
    _native.dtype_code(o1.dtype)
    d = o1.shape[-1]
    rows = math.prod(lead)
    ms1 = _pairs(m1, l1, rows)
    ms2 = _pairs(m2, l2, rows)
    o1c = o1.contiguous()
    o2c = o2.contiguous()
    o = torch.empty_like(o1c)
    ms = torch.empty(rows, 2, device=o1.device, dtype=torch.float32)
    with torch.cuda.device(o1.device):
        _native.merge_stats(o1c, ms1, o2c, ms2, o, ms, normalize, rows, d)
    return o, ms[:, 0].reshape(lead), ms[:, 1].reshape(lead)


class _BlockAttnResBatched(torch.autograd.Function):
    """Autograd for ``S`` queries against shared sources: forward saves
    ``(v, queries)`` only; backward recomputes the dot products and softmax
    from ``v`` and writes ``dv`` and per-CTA fp32 partial rows of
    ``dqueries``, summed in a fixed order."""

    @staticmethod
    def forward(ctx, v: torch.Tensor, queries: torch.Tensor, eps: float):
        _check_batched(v, queries)
        v = v.contiguous()
        queries = queries.contiguous()
        n, b, t, d = v.shape
        s = queries.shape[0]
        out = torch.empty(s, b, t, d, device=v.device, dtype=v.dtype)
        if b * t > 0:
            with torch.cuda.device(v.device):
                _native.fwd_batched(v, queries, out, n, b * t, d, s, eps)
        ctx.save_for_backward(v, queries)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, grad_out):
        v, queries = ctx.saved_tensors
        n, b, t, d = v.shape
        s = queries.shape[0]
        bt = b * t
        g = grad_out.to(v.dtype).contiguous()
        dv = torch.empty_like(v)
        dq = torch.empty_like(queries)
        with torch.cuda.device(v.device):
            p = _native.bwd_batched_partials(n, bt, d, s, v.dtype)
            part = torch.empty(p, s * d, device=v.device, dtype=torch.float32)
            _native.bwd_batched(v, queries, g, dv, part, n, bt, d, s, ctx.eps)
            _native.dw_reduce(part, dq.view(s * d))
        return dv, dq, None


def block_attn_res_batched_train(
    v: torch.Tensor, queries: torch.Tensor, eps: float = DEFAULT_EPS
) -> torch.Tensor:
    """``block_attn_res_batched`` with a backward: output ``[S, B, T, D]``,
    entry ``s`` equal to ``block_attn_res_triton(v, queries[s], eps)``, and
    gradients for ``v`` and ``queries`` (``S <= 16``: more queries with a
    gradient wanted are refused before the forward). Same validation and
    messages as the reference's batched API (``triton_op.py:463-474``)."""
    if queries.ndim == 2 and queries.shape[0] == 1:
        # one query: the single-query operator's kernels (the same forward
        # kernel block_attn_res_batched runs for S = 1, and its backward from
        # saved statistics), queries' gradient through the index
        _check_batched(v, queries)
        return _BlockAttnResTritonFn.apply(v, queries[0], eps).unsqueeze(0)
    _check_batched(v, queries)
    _check_trainable(v, queries)
    return _BlockAttnResBatched.apply(v, queries, eps)
