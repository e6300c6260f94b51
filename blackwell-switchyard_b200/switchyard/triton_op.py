"""Block AttnRes operator on B200: the drop-in for ``switchyard.triton_op``.

Same module path, names, argument meaning and error behaviour as the
reference's Triton module (``src/switchyard/triton_op.py``), so callers such as
the reference's ``model.py`` (``_IMPLS["switchyard"] = block_attn_res_triton``,
``model.py:140-143``) and its tests run unchanged. The name is kept for that
reason only: nothing here uses Triton. Every call goes through the C ABI of
``libswitchyard_b200.so`` into hand-written sm_100a CUDA kernels; there is no
eager or CPU fallback, and a missing library fails at import.

Per token, over the N sources ``v[:, b, t, :]`` and the query ``w``::

    logit_n = dot(w, v_n) * rsqrt(mean(v_n ** 2) + eps)     # no 1/sqrt(D)
    alpha   = softmax_n(logit)
    out     = sum_n alpha_n * v_n                          # raw sources

Forward saves ``v``, ``w`` and a small fp32 statistics tensor ``[B*T, SW]``
(``SW = round_up(2N+2, 4)``: the N logits, the N inverse RMS values, the max
logit and the log-sum-exp). The backward reads them instead of recomputing the
two full-D reductions, writes ``dv`` and one fp32 ``dw`` partial row per
consumer group, and a second small kernel sums the rows in a fixed order into
``dw`` in ``w``'s dtype -- deterministic, no atomics, no zero-fill launch.

The autograd functions here keep the reference's names and checks; each of
their forward and backward passes is one call into the PyTorch C++ extension
``_sy_torch`` (``csrc/torch_ext/sy_torch.cpp``), which allocates the outputs
with torch's caching allocator on the current stream and launches through the
C ABI. The remaining entry points go through the ctypes binding ``_native``.
"""

from __future__ import annotations

import torch

from . import _native

try:
    from . import _sy_torch  # the PyTorch C++ extension over the same C ABI
except ImportError as exc:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "switchyard: the C++ extension _sy_torch is missing or stale; build it with "
        "`python blackwell-switchyard_b200/csrc/build.py` (or __graft_entry__.build())"
    ) from exc

__all__ = [
    "DEFAULT_EPS",
    "block_attn_res_triton",
    "block_attn_res_batched",
    "BlockAttnResTriton",
    "speed_of_light",
]

#: RMSNorm epsilon, as in the reference (``src/switchyard/reference.py:95``).
DEFAULT_EPS = 1e-6

#: Kernel families reported by :func:`_plan` (``sy_plan_kind``): the generic
#: any-shape kernels, the register-tile kernels (exact N <= 16) and the
#: shared-memory tile kernels (run-time N <= 64), both TMA-pipelined, and the
#: row-stream forward (one warp per token, online softmax over the sources).
PLAN_GENERIC, PLAN_TILE, PLAN_SMEM_TILE, PLAN_STREAM = 0, 1, 2, 3


def _plan(op: str, n: int, bt: int, d: int, dtype: torch.dtype, s: int = 1) -> int:
    """Which kernel family a shape dispatches to (the reference's
    ``_launch_config`` / ``_bwd_launch`` / ``_batched_launch`` counterpart).

    ``op`` is ``"fwd"``, ``"bwd"`` or ``"batched"``. Returns :data:`PLAN_STREAM`,
    :data:`PLAN_TILE`, :data:`PLAN_SMEM_TILE` or :data:`PLAN_GENERIC`.
    """
    code = {"fwd": 0, "bwd": 1, "batched": 2}[op]
    k = _native.plan_kind(code, n, bt, d, s, dtype)
    if k < 0:
        raise _native.NativeError("sy_plan_kind", -k)
    return k


_STRATEGY = {PLAN_GENERIC: "generic", PLAN_TILE: "register-tile", PLAN_SMEM_TILE: "smem-tile",
             PLAN_STREAM: "row-stream"}


def _validate(v: torch.Tensor, w: torch.Tensor) -> None:
    """Argument checks of the reference forward (triton_op.py:507-513), plus
    the device of ``w`` and a positive source count, which it left unchecked."""
    if v.ndim != 4:
        raise ValueError(f"v must be [N, B, T, D], got {tuple(v.shape)}")
    n, b, t, d = v.shape
    if w.shape != (d,):
        raise ValueError(f"w must be [{d}], got {tuple(w.shape)}")
    if not v.is_cuda:
        raise ValueError("v must be on a CUDA device")
    if not w.is_cuda or w.device != v.device:
        raise ValueError("w must be on the same CUDA device as v")
    if n == 0:
        raise ValueError("N must be positive")
    _native.dtype_code(v.dtype)
    _native.dtype_code(w.dtype)


def _forward(v: torch.Tensor, w: torch.Tensor, eps: float):
    """Launch the forward (one call into the C++ extension: allocations on
    the current stream, ``sy_fwd``). Returns ``(v, w, out, stats, strategy)``
    with ``v`` and ``w`` contiguous (the kernels walk tokens with one stride,
    so B and T are flattened; a contiguous input -- the model's arena alias
    included -- is used in place, never copied)."""
    v = v.contiguous()
    w = w.contiguous()
    out, stats, kind = _sy_torch.forward(v, w, float(eps))
    return v, w, out, stats, _STRATEGY.get(kind, "empty")


def _backward_partials(v, w, stats, grad_out, eps: float):
    """Launch the backward. Returns ``(dv, dw_partial)``: the fp32 partial
    rows of dw, one per CTA (None when D == 0)."""
    dv, part = _sy_torch.backward_partials(v, w, stats, grad_out, float(eps))
    return dv, part


def _backward(v, w, stats, grad_out, eps: float, dw_dtype: torch.dtype):
    """Launch the backward and the fixed-order dw reduction. Returns
    ``(dv, dw)`` with ``dw`` in ``dw_dtype`` (float32 for the sharded path's
    collective exchange, which still adds the other ranks' rows)."""
    return _sy_torch.backward(v, w, stats, grad_out, float(eps), dw_dtype)


class _BlockAttnResTriton(torch.autograd.Function):
    """Autograd boundary (``src/switchyard/triton_op.py:504-589``).

    The class name is kept: the reference's profiler attribution keys on the
    autograd node name ``_BlockAttnResTritonBackward``.
    """

    @staticmethod
    def forward(ctx, v: torch.Tensor, w: torch.Tensor, eps: float, gain=None):
        # With the module's gain the query is q = w * gain (one elementwise
        # kernel, as the reference computes it) and the backward's dw
        # reduction also splits dq into dw = dq * gain and dgain = dq * w
        # (sy_dw_reduce_gain) instead of leaving two products to autograd.
        q = w if gain is None else (w * gain).contiguous()
        _validate(v, q)
        v, q, out, stats, strategy = _forward(v, q, eps)
        if gain is None:
            ctx.save_for_backward(v, q, stats)
        else:
            ctx.save_for_backward(v, q, stats, w.contiguous(), gain.contiguous())
        ctx.gain = gain is not None
        ctx.eps = eps
        ctx.strategy = strategy
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if not ctx.gain:
            v, w, stats = ctx.saved_tensors
            dv, dw = _backward(v, w, stats, grad_out, ctx.eps, w.dtype)
            return dv, dw, None, None
        v, q, stats, w, gain = ctx.saved_tensors
        dv, dw, dg = _sy_torch.backward_gain(v, q, stats, grad_out, w, gain, float(ctx.eps),
                                             ctx.needs_input_grad[1], ctx.needs_input_grad[3])
        return dv, dw, None, dg


def block_attn_res_triton(v: torch.Tensor, w: torch.Tensor, eps: float = DEFAULT_EPS):
    """Fused Block AttnRes. Same contract as ``block_attn_res_reference``
    (``src/switchyard/triton_op.py:592-594``)."""
    return _BlockAttnResTriton.apply(v, w, eps)


def block_attn_res_batched(
    v: torch.Tensor, queries: torch.Tensor, eps: float = DEFAULT_EPS
) -> torch.Tensor:
    """Answer ``S`` pseudo-queries against one shared source tensor, forward only.

    Mirrors ``src/switchyard/triton_op.py:438-501``: same validation and error
    messages, output ``[S, B, T, D]`` with entry ``s`` equal to
    ``block_attn_res_triton(v, queries[s], eps)``. Unlike the reference there
    is no per-query fallback loop: every shape runs as one kernel launch that
    reads ``v`` once for all queries.
    """
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
    if v.requires_grad or queries.requires_grad:
        raise RuntimeError(
            "block_attn_res_batched has no backward; use block_attn_res_triton per query "
            "for training, or run this under torch.no_grad() for inference"
        )
    _native.dtype_code(v.dtype)

    n, b, t, d = v.shape
    s = queries.shape[0]
    v = v.contiguous()
    queries = queries.contiguous()
    out = torch.empty(s, b, t, d, device=v.device, dtype=v.dtype)
    if b * t == 0:
        return out
    with torch.cuda.device(v.device):
        _native.fwd_batched(v, queries, out, n, b * t, d, s, eps)
    return out


def speed_of_light(v: torch.Tensor) -> torch.Tensor:
    """Read every source element and write ``sum_n v_n``: the traffic ceiling
    for the forward, with its exact bytes and access pattern
    (``src/switchyard/triton_op.py:153-191``). Used by the benchmark."""
    if v.ndim != 4 or not v.is_cuda:
        raise ValueError("v must be a CUDA tensor [N, B, T, D]")
    n, b, t, d = v.shape
    v = v.contiguous()
    out = torch.empty(b, t, d, device=v.device, dtype=v.dtype)
    if b * t > 0 and d > 0:
        with torch.cuda.device(v.device):
            _native.speed_of_light(v, out, n, b * t, d)
    return out


class BlockAttnResTriton(torch.nn.Module):
    """Drop-in replacement for ``switchyard.reference.BlockAttnRes``
    (``src/switchyard/triton_op.py:597-609``): zero-initialised query ``w``,
    optional RMSNorm gain ``g`` folded as ``w * g`` before the call."""

    def __init__(self, d_model: int, norm_affine: bool = True, eps: float = DEFAULT_EPS) -> None:
        super().__init__()
        self.d_model = d_model
        self.eps = eps
        self.w = torch.nn.Parameter(torch.zeros(d_model))
        self.g = torch.nn.Parameter(torch.ones(d_model)) if norm_affine else None

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, norm_affine={self.g is not None}, eps={self.eps}"

    def forward(self, v: torch.Tensor) -> torch.Tensor:
        if self.g is None:
            return block_attn_res_triton(v, self.w, self.eps)
        if self.w.dtype == self.g.dtype and self.w.device == self.g.device:
            # q = w * g, with dq split into dw and dg inside the dw reduction
            return _BlockAttnResTriton.apply(v, self.w, self.eps, self.g)
        return block_attn_res_triton(v, self.w * self.g, self.eps)
