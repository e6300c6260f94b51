"""The batched training contract and the two-phase schedule on the GPU.

Parity of ``attn_with_stats`` / ``merge_online_softmax`` (the paper's
Algorithm 1, ``src/switchyard/reference.py:195-233``) and of the batched
operator's backward with the float64 oracle on the same rounded inputs, at the
bounds of ``test_parity_gpu.py`` (bf16/fp16: 1.005x the dtype's rounding floor;
fp32: max(1.6x floor, 1e-6)). The reference's own two-phase test
(``tests/test_reference.py:140-150``) is reproduced with the GPU pieces: the
merged result of two source groups equals the single-pass operator.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attnres_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU runs deselect this module
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import (  # noqa: E402
    attn_with_stats,
    block_attn_res_batched,
    block_attn_res_batched_train,
    block_attn_res_triton,
    merge_online_softmax,
)
from switchyard.triton_op import DEFAULT_EPS  # noqa: E402

DEV = "cuda"
NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}

# Shapes that reach each batched kernel: the register tile (N <= 16, rows of
# 16-byte chunks that fit it), the row stream (N = 17, 8 KiB rows), the generic
# kernel (D = 777: rows not a multiple of 16 bytes) and small odd shapes.
# The backward: its register-tile kernel (N <= 9, rows of at most 4 KiB in
# whole 16-byte chunks, including rows of fewer chunks than threads: D = 1000)
# and its generic kernel (N = 17, D = 777, fp32 rows of 8 KiB).
CASES = [((9, 1, 16, 2048), 8), ((9, 1, 24, 2048), 16), ((17, 1, 8, 4096), 8),
         ((5, 1, 17, 777), 3), ((3, 2, 5, 64), 5), ((9, 1, 32, 2048), 1), ((4, 1, 9, 512), 2),
         ((6, 1, 40, 1000), 4)]


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float64).cpu().numpy()


def bound(floor: float, dtype: torch.dtype) -> float:
    return max(floor * 1.6, 1e-6) if dtype == torch.float32 else floor * 1.005


def check(got, want, dtype, what, factor=None):
    assert torch.isfinite(got).all(), what
    err = O.rel_l2(np64(got), want)
    floor = O.dtype_floor(want, NAMES[dtype])
    lim = bound(floor, dtype) if factor is None else factor * floor
    assert err <= lim, f"{what}: rel_l2 {err:.4e} vs floor {floor:.4e} ({err / max(floor, 1e-30):.4f}x)"


def make(shape, s, dtype, seed=0, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    v = torch.randn(*shape, generator=gen).to(dtype)
    q = torch.randn(s, shape[-1], generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True) * scale).to(dtype)
    g = torch.randn(s, *shape[1:], generator=gen).to(dtype)
    return v.to(DEV), q.to(DEV), g.to(DEV)


@pytest.mark.parametrize(("shape", "s"), CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_attn_with_stats_matches_oracle(shape, s, dtype):
    v, q, _ = make(shape, s, dtype)
    o, m, ell = attn_with_stats(v, q, DEFAULT_EPS)
    assert o.shape == (s,) + shape[1:] and o.dtype == dtype
    assert m.shape == ell.shape == (s,) + shape[1:3] and m.dtype == torch.float32
    o_w, m_w, l_w = O.batched_stats(np64(v), np64(q), DEFAULT_EPS)
    check(o, o_w, dtype, f"o {shape} S={s}")
    np.testing.assert_allclose(np64(m), m_w, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(np64(ell), l_w, rtol=2e-5, atol=2e-5)
    # one query as a vector: the reference's signature, outputs without the S axis
    o1, m1, l1 = attn_with_stats(v, q[0], DEFAULT_EPS)
    assert o1.shape == shape[1:] and m1.shape == shape[1:3]
    check(o1, o_w[0], dtype, f"o {shape} single query")


@pytest.mark.parametrize("split", [1, 2, 4])
def test_two_phase_merge_equals_single_pass(split):
    """tests/test_reference.py:140-150 on the GPU: attn_with_stats on two
    source groups, merged, equals the operator over all sources. The partial
    o's are rounded to bf16 before the merge, so the bound is 1.5x the floor
    (two roundings); the merge itself, against the oracle merge of the same
    rounded partials, is at the single-rounding bound."""
    v, q, _ = make((8, 1, 64, 1024), 1, torch.bfloat16, seed=3)
    w = q[0]
    o1, m1, l1 = attn_with_stats(v[:split], w)
    o2, m2, l2 = attn_with_stats(v[split:], w)
    out, m, ell = merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize=True)
    want = O.forward(np64(v), np64(w), DEFAULT_EPS)
    check(out, want, torch.bfloat16, f"two-phase split={split}", factor=1.5)
    o_m, m_m, l_m = O.merge_online_softmax(np64(o1), np64(m1), np64(l1), np64(o2), np64(m2), np64(l2))
    check(out, o_m / l_m[..., None], torch.bfloat16, "merge normalised")
    raw, m_r, l_r = merge_online_softmax(o1, m1, l1, o2, m2, l2)
    check(raw, o_m, torch.bfloat16, "merge raw")
    np.testing.assert_allclose(np64(m_r), m_m, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(np64(l_r), l_m, rtol=2e-6)
    assert torch.equal(m, m_r) and torch.equal(ell, l_r)


def test_merge_survives_extreme_logit_separation():
    """tests/test_reference.py:153-163: logits 200x apart stay finite."""
    v, q, _ = make((6, 1, 32, 512), 1, torch.bfloat16, seed=4, scale=200.0)
    w = q[0]
    o1, m1, l1 = attn_with_stats(v[:3], w)
    o2, m2, l2 = attn_with_stats(v[3:], w)
    out, _, _ = merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize=True)
    assert torch.isfinite(out).all()
    check(out, O.forward(np64(v), np64(w), DEFAULT_EPS), torch.bfloat16, "extreme", factor=1.5)


@pytest.mark.parametrize(("shape", "s"), CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_batched_backward_matches_oracle(shape, s, dtype):
    v, q, g = make(shape, s, dtype, seed=5)
    vt = v.clone().requires_grad_(True)
    qt = q.clone().requires_grad_(True)
    out = block_attn_res_batched_train(vt, qt, DEFAULT_EPS)
    with torch.no_grad():
        plain = block_attn_res_batched(v, q, DEFAULT_EPS)
    assert torch.equal(out.detach(), plain)  # same forward kernel as the output-only API
    check(out, O.batched(np64(v), np64(q), DEFAULT_EPS), dtype, f"out {shape} S={s}")
    out.backward(g)
    assert vt.grad.dtype == dtype and qt.grad.dtype == dtype
    dv_w, dq_w = O.batched_backward(np64(v), np64(q), np64(g), DEFAULT_EPS)
    check(vt.grad, dv_w, dtype, f"dv {shape} S={s}")
    check(qt.grad, dq_w, dtype, f"dq {shape} S={s}")


def test_batched_backward_is_bit_stable_and_sums_single_queries():
    """Two runs give identical gradients (fixed-order dq reduction, no
    atomics); dq_s equals the single-query operator's dw for the same query
    within the bf16 floor."""
    v, q, g = make((9, 1, 96, 2048), 4, torch.bfloat16, seed=6)
    grads = []
    for _ in range(2):
        vt = v.clone().requires_grad_(True)
        qt = q.clone().requires_grad_(True)
        block_attn_res_batched_train(vt, qt).backward(g)
        grads.append((vt.grad, qt.grad))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])
    for s in range(4):
        ws = q[s].clone().requires_grad_(True)
        block_attn_res_triton(v, ws).backward(g[s])
        dq_w = O.backward(np64(v), np64(q[s]), np64(g[s]), DEFAULT_EPS)[1]
        check(ws.grad, dq_w, torch.bfloat16, f"single dw {s}")
        check(grads[0][1][s], dq_w, torch.bfloat16, f"batched dq {s}")


def test_batched_backward_single_source_and_empty():
    # N = 1: softmax is identically 1, so dq is exactly zero and dv_0 = sum_s g_s
    v, q, g = make((1, 1, 16, 256), 3, torch.float32, seed=7)
    vt = v.clone().requires_grad_(True)
    qt = q.clone().requires_grad_(True)
    block_attn_res_batched_train(vt, qt).backward(g)
    assert qt.grad.abs().max().item() == 0.0
    torch.testing.assert_close(vt.grad[0], g.sum(0), rtol=1e-6, atol=1e-6)
    # no tokens: empty outputs, zero dq
    v0 = torch.zeros(3, 1, 0, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    q0 = torch.randn(2, 64, device=DEV).to(torch.bfloat16).requires_grad_(True)
    out = block_attn_res_batched_train(v0, q0)
    assert out.shape == (2, 1, 0, 64)
    out.sum().backward()
    assert q0.grad.abs().max().item() == 0.0


def test_two_phase_api_errors():
    v, q, _ = make((3, 1, 4, 64), 2, torch.bfloat16)
    with pytest.raises(RuntimeError, match="no backward"):
        attn_with_stats(v.clone().requires_grad_(True), q)
    with pytest.raises(ValueError, match="same dtype"):
        block_attn_res_batched_train(v, q.float())
    with pytest.raises(ValueError, match="positive"):
        block_attn_res_batched_train(v, q[:0])
    o, m, ell = attn_with_stats(v, q)
    with pytest.raises(ValueError, match="same shape"):
        merge_online_softmax(o, m, ell, o[:1], m[:1], ell[:1])


def test_more_than_16_queries_refused_before_the_forward_when_training():
    """The batched backward takes at most 16 queries: with a gradient wanted, a
    larger S is refused before anything runs (single-GPU and sharded ops);
    without one the forward runs for any S."""
    from switchyard.sharding import block_attn_res_batched_sharded

    v, q, _ = make((3, 1, 8, 64), 17, torch.bfloat16, seed=3)
    with pytest.raises(ValueError, match="at most 16 queries"):
        block_attn_res_batched_train(v.clone().requires_grad_(True), q)
    with pytest.raises(ValueError, match="at most 16 queries"):
        block_attn_res_batched_train(v, q.clone().requires_grad_(True))
    with pytest.raises(ValueError, match="at most 16 queries"):
        block_attn_res_batched_sharded(v.clone().requires_grad_(True), q)
    with torch.no_grad():
        out = block_attn_res_batched_train(v.clone().requires_grad_(True), q)
    assert out.shape == (17, 1, 8, 64)
    out = block_attn_res_batched_train(v, q)  # nothing requires a gradient
    assert out.shape == (17, 1, 8, 64) and not out.requires_grad
