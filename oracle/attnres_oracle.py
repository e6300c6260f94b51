"""CPU oracle for the Block AttnRes operator -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The operator itself (``switchyard.triton_op``) never calls it and has no CPU
path.

It restates, in float64 numpy, the mathematics of the reference
(``sabdulmajid/blackwell-switchyard``), one function per reference function,
each citing the file and lines it follows. Parity is pinned: the golden
fixtures under ``tests/golden/`` were produced by importing the reference's own
``src/switchyard/reference.py`` / ``baselines.py`` (script:
``tests/golden/make_golden.py``), and ``tests/test_oracle.py`` checks every
function here against them.

Shapes follow the reference: ``v [N, B, T, D]``, ``w [D]``, output ``[B, T, D]``.
All arrays are converted to float64 on entry.
"""

from __future__ import annotations

import numpy as np

#: reference.py:95
DEFAULT_EPS = 1e-6


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


def inv_rms(v, eps: float = DEFAULT_EPS) -> np.ndarray:
    """``1 / sqrt(mean(v**2, -1) + eps)`` per row (reference.py:98-104, the
    scale that ``rms_norm`` multiplies by). Returns ``[N, B, T]``."""
    v = _f64(v)
    return 1.0 / np.sqrt(np.mean(v * v, axis=-1) + eps)


def rms_norm(v, eps: float = DEFAULT_EPS) -> np.ndarray:
    """RMSNorm without gain over the last axis (reference.py:98-104)."""
    v = _f64(v)
    return v * inv_rms(v, eps)[..., None]


def logits(v, w, eps: float = DEFAULT_EPS) -> np.ndarray:
    """``dot(w, rms_norm(v_n))`` per source and token, no 1/sqrt(D)
    (reference.py:44-45, :130-131). Returns ``[N, B, T]``."""
    v, w = _f64(v), _f64(w)
    return np.einsum("d,nbtd->nbt", w, rms_norm(v, eps))


def softmax0(x) -> np.ndarray:
    """Softmax over the source axis 0 (reference.py:46, :132)."""
    x = _f64(x)
    e = np.exp(x - x.max(axis=0, keepdims=True))
    return e / e.sum(axis=0, keepdims=True)


def forward(v, w, eps: float = DEFAULT_EPS) -> np.ndarray:
    """Block AttnRes forward (reference.py:107-133; oracle reference.py:136-146).

    out[b,t] = sum_n softmax_n(logit)[n,b,t] * v[n,b,t]  -- the RAW sources.
    """
    v, w = _f64(v), _f64(w)
    if v.ndim != 4:
        raise ValueError(f"v must be [N, B, T, D], got shape {tuple(v.shape)}")
    if w.ndim != 1:
        raise ValueError(f"w must be [D], got shape {tuple(w.shape)}")
    if w.shape[0] != v.shape[-1]:
        raise ValueError(f"w has D={w.shape[0]} but v has D={v.shape[-1]}")
    alpha = softmax0(logits(v, w, eps))
    return np.einsum("nbt,nbtd->btd", alpha, v)


def forward_stats(v, w, eps: float = DEFAULT_EPS):
    """The per-token statistics the B200 forward saves for its backward.

    Returns ``(logit [N,B,T], r [N,B,T], m [B,T], lse [B,T])`` with
    ``r = inv_rms``, ``m = max_n logit`` and ``lse = m + log(sum_n exp(logit-m))``.
    (``m`` and ``sum exp`` are the quantities of reference.py:195-216.)
    """
    lg = logits(v, w, eps)
    r = inv_rms(v, eps)
    m = lg.max(axis=0)
    lse = m + np.log(np.exp(lg - m).sum(axis=0))
    return lg, r, m, lse


def backward(v, w, g, eps: float = DEFAULT_EPS):
    """Analytic gradients ``(dv, dw)`` of ``sum(forward(v, w) * g)``.

    Follows the derivation in the reference's backward kernel docstring
    (src/switchyard/triton_op.py:205-214) with ``r_n = inv_rms``,
    ``a_n = w.v_n``, ``logit_n = a_n r_n``, ``alpha = softmax(logit)``::

        G_n      = g . v_n
        S        = sum_n alpha_n G_n
        dlogit_n = alpha_n (G_n - S)
        da_n     = dlogit_n r_n
        dssq_n   = -dlogit_n a_n r_n^3 / (2D)
        dv_n     = alpha_n g + da_n w + 2 dssq_n v_n
        dw       = sum_{tokens} sum_n da_n v_n

    ``tests/test_oracle.py`` also pins it to autograd through the reference
    forward in float64 (the reference's own check, tests/test_triton_op.py:151-182).
    """
    v, w, g = _f64(v), _f64(w), _f64(g)
    d = v.shape[-1]
    r = inv_rms(v, eps)
    a = np.einsum("d,nbtd->nbt", w, v)
    alpha = softmax0(a * r)
    G = np.einsum("btd,nbtd->nbt", g, v)
    S = (alpha * G).sum(axis=0)
    dlogit = alpha * (G - S)
    da = dlogit * r
    dssq = -dlogit * a * r**3 / (2.0 * d)
    dv = alpha[..., None] * g[None] + da[..., None] * w + 2.0 * dssq[..., None] * v
    dw = np.einsum("nbt,nbtd->d", da, v)
    return dv, dw


def attn_with_stats(v, w, eps: float = DEFAULT_EPS):
    """``(o, m, ell)`` of the paper's ATTNWITHSTATS (reference.py:195-216):
    ``o = sum_n exp(logit_n - m) v_n`` unnormalised, ``ell = sum_n exp(logit_n - m)``."""
    v = _f64(v)
    lg = logits(v, w, eps)
    m = lg.max(axis=0)
    p = np.exp(lg - m)
    return np.einsum("nbt,nbtd->btd", p, v), m, p.sum(axis=0)


def merge_online_softmax(o1, m1, l1, o2, m2, l2):
    """Exact merge of two partial ``(o, m, ell)`` triples (reference.py:219-233)."""
    o1, m1, l1, o2, m2, l2 = map(_f64, (o1, m1, l1, o2, m2, l2))
    m = np.maximum(m1, m2)
    s1 = np.exp(m1 - m)
    s2 = np.exp(m2 - m)
    return o1 * s1[..., None] + o2 * s2[..., None], m, l1 * s1 + l2 * s2


def batched(v, queries, eps: float = DEFAULT_EPS) -> np.ndarray:
    """``S`` queries against one source tensor, ``[S, B, T, D]``
    (baselines.py:76-81; triton_op.py:460-461: entry s == forward(v, q_s))."""
    v, q = _f64(v), _f64(queries)
    dots = np.einsum("sd,nbtd->snbt", q, v)
    alpha = softmax0(np.moveaxis(dots * inv_rms(v, eps)[None], 1, 0))  # softmax over n
    alpha = np.moveaxis(alpha, 0, 1)  # back to [S, N, B, T]
    return np.einsum("snbt,nbtd->sbtd", alpha, v)


def batched_stats(v, queries, eps: float = DEFAULT_EPS):
    """Per-query ``(o, m, ell)`` triples, each with a leading ``S`` axis:
    ``attn_with_stats`` (reference.py:195-216) applied to every query."""
    res = [attn_with_stats(v, q, eps) for q in _f64(queries)]
    return tuple(np.stack(x) for x in zip(*res))


def batched_backward(v, queries, g, eps: float = DEFAULT_EPS):
    """Gradients ``(dv, dqueries)`` of ``sum(batched(v, queries) * g)``, ``g``
    of shape ``[S, B, T, D]``. Output ``s`` is ``forward(v, queries[s])``
    (triton_op.py:460-461), so the loss is a sum of single-query losses and
    ``dv = sum_s backward(v, q_s, g_s).dv``, ``dq_s = backward(v, q_s, g_s).dw``."""
    v, q, g = _f64(v), _f64(queries), _f64(g)
    dv = np.zeros_like(v)
    dq = np.zeros_like(q)
    for s in range(q.shape[0]):
        dvs, dqs = backward(v, q[s], g[s], eps)
        dv += dvs
        dq[s] = dqs
    return dv, dq


def speed_of_light(v) -> np.ndarray:
    """``sum_n v_n``: the bytes of the forward without its softmax
    (triton_op.py:153-176)."""
    return _f64(v).sum(axis=0)


def attn_res_flops(n: int, b: int, t: int, d: int) -> int:
    """Three multiply-adds per source element (reference.py:236-244)."""
    return 2 * n * b * t * d * 3


def attn_res_min_bytes(n: int, b: int, t: int, d: int, itemsize: int = 2) -> int:
    """Read every source once, write the output once (reference.py:247-255)."""
    return (n * b * t * d + b * t * d) * itemsize


def fwd_bwd_min_bytes(n: int, b: int, t: int, d: int, itemsize: int = 2) -> int:
    """Forward bytes plus the backward's minimum: read v and g, write dv
    (``(3N+2) * BTD * itemsize``; dw and the statistics are excluded)."""
    return (3 * n + 2) * b * t * d * itemsize


def batched_min_bytes(n: int, b: int, t: int, d: int, s: int, itemsize: int = 2) -> int:
    """Read v once and the S queries, write S outputs."""
    return ((n + s) * b * t * d + s * d) * itemsize


# ---------------------------------------------------------------------------
# Metrics (tests/test_triton_op.py:35-44; bench/harness.py:331-345)
# ---------------------------------------------------------------------------


def round_to(x, dtype: str) -> np.ndarray:
    """Round float64 values to ``dtype`` and back, the way torch's
    ``tensor.to(dtype)`` does from float64: through float32 first, then (for
    bf16) round-to-nearest-even on the top 16 bits."""
    x32 = _f64(x).astype(np.float32)
    if dtype == "float32":
        return x32.astype(np.float64)
    if dtype == "float16":
        return x32.astype(np.float16).astype(np.float64)
    if dtype == "bfloat16":
        u = x32.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x32)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        out = rounded.astype(np.uint32).view(np.float32).astype(np.float64)
        out[nan] = np.nan
        return out
    raise ValueError(f"unknown dtype {dtype}")


def rel_l2(got, oracle) -> float:
    got, oracle = _f64(got), _f64(oracle)
    return float(np.linalg.norm(got - oracle) / np.linalg.norm(oracle))


def dtype_floor(oracle, dtype: str) -> float:
    """Relative L2 error of merely rounding the exact answer to ``dtype``."""
    o = _f64(oracle)
    return float(np.linalg.norm(round_to(o, dtype) - o) / np.linalg.norm(o))
