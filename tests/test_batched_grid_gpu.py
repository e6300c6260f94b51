"""The batched-query forward over every source count its register-tile kernel
is compiled for (N = 1..16) and a spread of query counts, against the float64
oracle (GPU).

The kernel is instantiated per (N, chunks per thread, query slots): the slots
are S rounded up to 4, 8 or 16, the queries go through the 32-value reductions
in blocks of QB = min(4, 32 / N), and the N sums of squares ride in the last
block's spare lanes or in a block of their own. Each combination below lands on
a different one of those layouts (and D = 1024 gives 4, 2 and 1 chunks per
thread as N grows); T = 37 leaves most CTAs with one token and some with none.
Outputs are checked at the dtype's rounding floor as in ``test_parity_gpu``;
with statistics (``attn_with_stats``) the (m, l) pairs too; and the batched
backward's dv and dq at every N up to 12.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attnres_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU runs deselect this module
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import attn_with_stats, block_attn_res_batched  # noqa: E402
from switchyard.triton_op import DEFAULT_EPS  # noqa: E402

DEV = "cuda"
T, D = 37, 1024
NAMES = {torch.bfloat16: "bfloat16", torch.float32: "float32"}


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float64).cpu().numpy()


def inputs(n, s, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(n, 1, T, D, generator=g).to(dtype)
    q = torch.randn(s, D, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True) * 4.0).to(dtype)  # logits of a few units
    return v.to(DEV), q.to(DEV)


def check(got, want, dtype, what):
    assert torch.isfinite(got).all(), what
    err = O.rel_l2(np64(got), want)
    floor = O.dtype_floor(want, NAMES[dtype])
    lim = max(floor * 1.6, 1e-6) if dtype == torch.float32 else floor * 1.005
    assert err <= lim, f"{what}: rel_l2 {err:.4e} vs floor {floor:.4e} ({err / max(floor, 1e-30):.4f}x)"


@pytest.mark.parametrize("s", [2, 3, 4, 5, 7, 8, 9, 12, 16])
@pytest.mark.parametrize("n", list(range(1, 17)))
def test_every_source_count_and_query_layout_bf16(n, s):
    v, q = inputs(n, s, torch.bfloat16, seed=100 * n + s)
    with torch.no_grad():
        got = block_attn_res_batched(v, q, DEFAULT_EPS)
    assert got.shape == (s, 1, T, D)
    check(got, O.batched(np64(v), np64(q), DEFAULT_EPS), torch.bfloat16, f"N={n} S={s}")


@pytest.mark.parametrize("s", [3, 8, 16])
@pytest.mark.parametrize("n", list(range(1, 17)))
def test_every_source_count_fp32(n, s):
    v, q = inputs(n, s, torch.float32, seed=200 * n + s)
    with torch.no_grad():
        got = block_attn_res_batched(v, q, DEFAULT_EPS)
    check(got, O.batched(np64(v), np64(q), DEFAULT_EPS), torch.float32, f"N={n} S={s} fp32")


@pytest.mark.parametrize("s", [3, 9])
@pytest.mark.parametrize("n", list(range(1, 17)))
def test_statistics_for_every_source_count(n, s):
    """The raw output and (m, l) of attn_with_stats: the statistics are stored
    by the first lane of each query's N lanes, for real queries only."""
    v, q = inputs(n, s, torch.bfloat16, seed=300 * n + s)
    o, m, ell = attn_with_stats(v, q, DEFAULT_EPS)
    o_w, m_w, l_w = O.batched_stats(np64(v), np64(q), DEFAULT_EPS)
    check(o, o_w, torch.bfloat16, f"o N={n} S={s}")
    np.testing.assert_allclose(np64(m), m_w, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(np64(ell), l_w, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("s", [1, 2, 5, 8, 16])
@pytest.mark.parametrize("n", list(range(1, 13)))
def test_batched_backward_for_every_source_count(n, s):
    """block_attn_res_batched_train's dv and dq: the register-tile backward for
    N <= 9 (one CTA per token, every dot product of a token in one pass), the
    generic kernel beyond."""
    from switchyard import block_attn_res_batched_train

    dd = 512
    g = torch.Generator().manual_seed(400 * n + s)
    v = torch.randn(n, 1, T, dd, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(s, dd, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True) * 4.0).to(torch.bfloat16).to(DEV)
    gout = torch.randn(s, 1, T, dd, generator=g).to(torch.bfloat16).to(DEV)
    vt = v.clone().requires_grad_(True)
    qt = q.clone().requires_grad_(True)
    block_attn_res_batched_train(vt, qt, DEFAULT_EPS).backward(gout)
    dv_w, dq_w = O.batched_backward(np64(v), np64(q), np64(gout), DEFAULT_EPS)
    check(vt.grad, dv_w, torch.bfloat16, f"dv N={n} S={s}")
    if n == 1:  # one source: the softmax is identically 1 and dq exactly zero
        assert qt.grad.abs().max().item() == 0.0
    else:
        check(qt.grad, dq_w, torch.bfloat16, f"dq N={n} S={s}")
