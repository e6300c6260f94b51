"""The CPU oracle, pinned to the reference (CPU only).

Every oracle function is compared with the golden fixtures the reference's own
code produced (``tests/golden/make_golden.py``), then with float64 autograd,
and then with the semantic properties the reference's ``tests/test_reference.py``
asserts. A deliberately wrong oracle (planted here, on the CPU) must fail the
golden comparison, which shows the comparison has teeth.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases, load_golden

from oracle import attnres_oracle as O
from oracle import eager_port as E

EPS = O.DEFAULT_EPS
CASES = golden_cases()


def _close(got, want, rtol=1e-10, atol=1e-12, msg=""):
    np.testing.assert_allclose(np.asarray(got), np.asarray(want), rtol=rtol, atol=atol, err_msg=msg)


def test_golden_fixtures_present():
    assert len(CASES) >= 10
    assert "c1_4_1_256_512" in CASES  # the small fp32 case N=4 T=256 D=512


@pytest.mark.parametrize("name", CASES)
def test_forward_matches_reference(name):
    z, (v, w, _, _) = load_golden(name)
    sub = int(z["meta_sub"])
    _close(O.forward(v, w, EPS)[..., ::sub], z["out"], msg=name)


@pytest.mark.parametrize("name", CASES)
def test_statistics_match_reference(name):
    z, (v, w, _, _) = load_golden(name)
    lg, r, m, lse = O.forward_stats(v, w, EPS)
    _close(lg, z["logits"], msg=name)
    _close(r, z["r"], msg=name)
    _close(m, z["m"], msg=name)
    _close(lse, z["lse"], msg=name)


@pytest.mark.parametrize("name", CASES)
def test_backward_matches_reference_autograd(name):
    z, (v, w, g, _) = load_golden(name)
    dv, dw = O.backward(v, w, g, EPS)
    want_dv = z["dv"]
    got_dv = dv[:, :, :16] if name.startswith("c1_") else dv[..., :: int(z["meta_sub"])]
    _close(got_dv, want_dv, rtol=1e-9, atol=1e-11, msg=name)
    _close(dw, z["dw"], rtol=1e-9, atol=1e-11, msg=name)


@pytest.mark.parametrize("name", CASES)
def test_attn_with_stats_and_merge_match_reference(name):
    z, (v, w, _, _) = load_golden(name)
    sub, split = int(z["meta_sub"]), int(z["split"])
    o1, m1, l1 = O.attn_with_stats(v[:split], w, EPS)
    cut = (lambda a: a[:, :16]) if name.startswith("c1_") else (lambda a: a[..., ::sub])
    _close(cut(o1), z["aws1_o"], msg=name)
    _close(m1, z["aws1_m"], msg=name)
    _close(l1, z["aws1_l"], msg=name)
    if "merged" in z:
        o2, m2, l2 = O.attn_with_stats(v[split:], w, EPS)
        o, _, ell = O.merge_online_softmax(o1, m1, l1, o2, m2, l2)
        _close(cut(o / ell[..., None]), z["merged"], msg=name)


@pytest.mark.parametrize("name", [c for c in CASES])
def test_batched_matches_reference(name):
    z, (v, _, _, q) = load_golden(name)
    if "batched" not in z:
        pytest.skip("case has no queries")
    _close(O.batched(v, q, EPS)[..., :: int(z["meta_sub"])], z["batched"], msg=name)
    # entry s is the single-query forward (triton_op.py:460-461)
    for s in range(q.shape[0]):
        _close(O.batched(v, q, EPS)[s], O.forward(v, q[s], EPS))


@pytest.mark.parametrize("name", CASES)
def test_byte_and_flop_models_match_reference(name):
    z, _ = load_golden(name)
    n, b, t, d = (int(x) for x in z["meta_shape"])
    assert O.attn_res_min_bytes(n, b, t, d, 2) == int(z["min_bytes_bf16"])
    assert O.attn_res_flops(n, b, t, d) == int(z["flops"])


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("s_")])
def test_eager_port_matches_reference(name):
    """The timed CPU baseline computes what the reference computes."""
    z, (v, w, g, _) = load_golden(name)
    vt, wt, gt = (torch.from_numpy(x) for x in (v, w, g))
    out, dv, dw = E.fwd_bwd(vt, wt, gt, EPS)
    _close(out.numpy(), z["out"], msg=name)
    _close(dv.numpy(), z["dv"], rtol=1e-9, atol=1e-11, msg=name)
    _close(dw.numpy(), z["dw"], rtol=1e-9, atol=1e-11, msg=name)
    if "folded" in z:
        _close(E.folded_eager(vt, wt, EPS).numpy(), z["folded"], msg=name)


def test_round_to_matches_torch():
    x = np.concatenate([np.random.default_rng(0).standard_normal(20000) * 10.0 ** k for k in range(-3, 4)])
    for dt in ("bfloat16", "float16", "float32"):
        want = torch.from_numpy(x).to(getattr(torch, dt)).to(torch.float64).numpy()
        np.testing.assert_array_equal(O.round_to(x, dt), want, err_msg=dt)


def test_planted_mistake_is_caught():
    """A 1/sqrt(D) temperature (the mistake reference.py:58-59 warns about)
    must fail the golden comparison."""
    z, (v, w, _, _) = load_golden("b_9_1_4_2048")
    d = v.shape[-1]
    wrong = O.forward(v, w / np.sqrt(d), EPS)[..., :: int(z["meta_sub"])]
    assert O.rel_l2(wrong, z["out"]) > 1e-3
    # ...and so must a weighted sum over the normalised instead of the raw sources
    alpha = O.softmax0(O.logits(v, w, EPS))
    wrong2 = np.einsum("nbt,nbtd->btd", alpha, O.rms_norm(v, EPS))[..., :: int(z["meta_sub"])]
    assert O.rel_l2(wrong2, z["out"]) > 1e-3


# ---- semantics, as the reference's tests/test_reference.py asserts them ----


def _inp(n=5, b=2, t=7, d=16, seed=0, scale=1.0):
    rng = np.random.default_rng(seed)
    v = rng.standard_normal((n, b, t, d))
    w = rng.standard_normal(d)
    return v, w / np.linalg.norm(w) * scale


def test_zero_query_gives_mean():
    v, _ = _inp()
    _close(O.forward(v, np.zeros(v.shape[-1])), v.mean(0))


def test_single_source_is_identity():
    v, w = _inp(n=1)
    _close(O.forward(v, w), v[0])


def test_output_is_convex_combination():
    v, w = _inp(scale=3.0)
    out = O.forward(v, w)
    assert (out <= v.max(0) + 1e-12).all() and (out >= v.min(0) - 1e-12).all()


def test_softmax_is_per_token():
    v, w = _inp()
    v2 = v.copy()
    v2[:, 0, 3, :] += 10.0
    changed = np.abs(O.forward(v, w) - O.forward(v2, w)).sum(-1) > 1e-9
    assert changed[0, 3] and changed.sum() == 1


def test_backward_matches_float64_autograd():
    """The oracle's closed-form gradient equals autograd through the
    forward, the reference's own check (tests/test_triton_op.py:151-182)."""
    v, w = _inp(n=6, b=2, t=5, d=24, seed=3)
    g = np.random.default_rng(4).standard_normal((2, 5, 24))
    vv = torch.from_numpy(v).requires_grad_(True)
    ww = torch.from_numpy(w).requires_grad_(True)
    E.block_attn_res_eager(vv, ww, EPS).backward(torch.from_numpy(g))
    dv, dw = O.backward(v, w, g, EPS)
    _close(dv, vv.grad.numpy(), rtol=1e-10, atol=1e-12)
    _close(dw, ww.grad.numpy(), rtol=1e-10, atol=1e-12)


def test_batched_backward_matches_float64_autograd():
    """The batched gradient (dv summed over queries, one dq row per query)
    equals autograd through the eager forward applied per query and stacked,
    which is the batched output's definition (triton_op.py:460-461)."""
    v, _ = _inp(n=5, b=2, t=3, d=16, seed=7)
    rng = np.random.default_rng(8)
    q = rng.standard_normal((3, 16)) / 4.0
    g = rng.standard_normal((3, 2, 3, 16))
    vv = torch.from_numpy(v).requires_grad_(True)
    qq = torch.from_numpy(q).requires_grad_(True)
    out = torch.stack([E.block_attn_res_eager(vv, qq[s], EPS) for s in range(3)])
    out.backward(torch.from_numpy(g))
    dv, dq = O.batched_backward(v, q, g, EPS)
    _close(dv, vv.grad.numpy(), rtol=1e-10, atol=1e-12)
    _close(dq, qq.grad.numpy(), rtol=1e-10, atol=1e-12)
    o, m, ell = O.batched_stats(v, q, EPS)
    _close(o / ell[..., None], O.batched(v, q, EPS), rtol=1e-12, atol=1e-12)
    _close(m[1], O.logits(v, q[1], EPS).max(axis=0), rtol=1e-12)


def test_single_source_gives_zero_query_gradient():
    v, w = _inp(n=1)
    g = np.random.default_rng(1).standard_normal(v.shape[1:])
    dv, dw = O.backward(v, w, g)
    assert np.abs(dw).max() == 0.0
    _close(dv[0], g)


@pytest.mark.parametrize("split", [1, 2, 4])
def test_online_softmax_merge_is_exact(split):
    v, w = _inp(n=8)
    o1, m1, l1 = O.attn_with_stats(v[:split], w)
    o2, m2, l2 = O.attn_with_stats(v[split:], w)
    o, _, ell = O.merge_online_softmax(o1, m1, l1, o2, m2, l2)
    _close(o / ell[..., None], O.forward(v, w), rtol=1e-12, atol=1e-12)


def test_rejects_bad_shapes():
    with pytest.raises(ValueError, match=r"\[N, B, T, D\]"):
        O.forward(np.zeros((3, 4)), np.zeros(4))
    with pytest.raises(ValueError, match="D="):
        O.forward(np.zeros((2, 1, 3, 8)), np.zeros(7))
