"""The single-query operator, forward and backward through autograd, at every
source count from 1 to 20 (GPU).

The register-tile kernels are compiled per N (1..16) and chunks per thread; the
row-stream kernels take larger N and 4 KiB rows. D = 512 and 2048 put each N on
both sides of those boundaries, and T = 37 leaves most CTAs with one token and
some with none. out, dv and dw are checked against the float64 oracle at the
dtype's rounding floor, as in ``test_parity_gpu``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attnres_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU runs deselect this module
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import block_attn_res_triton  # noqa: E402
from switchyard.triton_op import DEFAULT_EPS  # noqa: E402

DEV = "cuda"
T = 37
NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float64).cpu().numpy()


def check(got, want, dtype, what):
    assert torch.isfinite(got).all(), what
    err = O.rel_l2(np64(got), want)
    floor = O.dtype_floor(want, NAMES[dtype])
    lim = max(floor * 1.6, 1e-6) if dtype == torch.float32 else floor * 1.005
    assert err <= lim, f"{what}: rel_l2 {err:.4e} vs floor {floor:.4e} ({err / max(floor, 1e-30):.4f}x)"


def run(n, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(n, 1, T, d, generator=g).to(dtype).to(DEV)
    w = (torch.randn(d, generator=g) / d**0.5).to(dtype).to(DEV)
    dout = torch.randn(1, T, d, generator=g).to(dtype).to(DEV)
    vt = v.clone().requires_grad_(True)
    wt = w.clone().requires_grad_(True)
    out = block_attn_res_triton(vt, wt, DEFAULT_EPS)
    out.backward(dout)
    check(out, O.forward(np64(v), np64(w), DEFAULT_EPS), dtype, f"out N={n} D={d}")
    dv_w, dw_w = O.backward(np64(v), np64(w), np64(dout), DEFAULT_EPS)
    check(vt.grad, dv_w, dtype, f"dv N={n} D={d}")
    if n == 1:  # one source: the softmax is identically 1 and dw exactly zero
        assert wt.grad.abs().max().item() == 0.0
    else:
        check(wt.grad, dw_w, dtype, f"dw N={n} D={d}")


@pytest.mark.parametrize("d", [512, 2048])
@pytest.mark.parametrize("n", list(range(1, 21)))
def test_every_source_count_bf16(n, d):
    run(n, d, torch.bfloat16, seed=10 * n + d)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("n", [1, 3, 6, 9, 12, 16, 17, 20])
def test_other_dtypes(n, dtype):
    run(n, 1024, dtype, seed=7 * n)
