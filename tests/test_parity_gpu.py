"""Parity of the sm_100a kernels with the float64 oracle (GPU).

The metric is the reference's (tests/test_triton_op.py:35-44): relative L2
against float64, next to the dtype's own rounding floor -- the error of merely
rounding the exact answer to the output dtype. A kernel that accumulates in
fp32 and rounds once sits at that floor. Bounds used here:

* bf16 / fp16 outputs: ``err <= 1.005 * floor`` ("prints as 1.00x"), tighter
  than the reference's 1.6x (forward) and 1.05x (batched);
* fp32 outputs: the reference's own ``max(1.6 * floor, 1e-6)``, because the
  fp32 floor (~3e-8) is below fp32 arithmetic noise.

The oracle is ``oracle/attnres_oracle.py`` evaluated on the same rounded
inputs; it is pinned to the reference by ``tests/test_oracle.py``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import golden_cases, load_golden

from oracle import attnres_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU runs deselect this module
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import block_attn_res_batched, block_attn_res_triton  # noqa: E402
from switchyard.triton_op import DEFAULT_EPS, _BlockAttnResTriton  # noqa: E402

DEV = "cuda"
NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}

# The reference's 16 shapes (tests/test_triton_op.py:57-62): both of its
# dispatch paths, non-power-of-two N, D and T, N up to 33, D up to 8192.
SHAPES = [
    (1, 1, 32, 256), (2, 1, 64, 128), (4, 2, 128, 512), (8, 1, 256, 2048),
    (9, 1, 512, 1024), (9, 1, 256, 2048), (9, 1, 128, 4096), (9, 1, 64, 8192),
    (16, 1, 128, 1024), (17, 1, 64, 2048), (32, 1, 64, 1024), (33, 1, 64, 512),
    (3, 1, 64, 777), (5, 1, 17, 63), (8, 3, 101, 1536), (7, 2, 1, 320),
]


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float64).cpu().numpy()


def bound(floor: float, dtype: torch.dtype) -> float:
    if dtype == torch.float32:
        return max(floor * 1.6, 1e-6)
    return floor * 1.005


def make(n, b, t, d, dtype, seed=0, scale=1.0):
    """The reference's generator (tests/test_triton_op.py:47-52), on the CPU
    for reproducibility, then moved to the GPU."""
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(n, b, t, d, generator=g, dtype=torch.float32).to(dtype)
    w = torch.randn(d, generator=g, dtype=torch.float32)
    w = (w / w.norm() * scale).to(dtype)
    return v.to(DEV), w.to(DEV)


def check(got: torch.Tensor, want: np.ndarray, dtype: torch.dtype, what: str):
    assert torch.isfinite(got).all(), what
    err = O.rel_l2(np64(got), want)
    floor = O.dtype_floor(want, NAMES[dtype])
    assert err <= bound(floor, dtype), f"{what}: rel_l2 {err:.4e} vs floor {floor:.4e} ({err / max(floor, 1e-30):.4f}x)"
    return err, floor


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_forward_is_at_the_dtype_floor(shape, dtype):
    v, w = make(*shape, dtype)
    got = block_attn_res_triton(v, w, DEFAULT_EPS)
    assert got.shape == shape[1:] and got.dtype == dtype
    check(got, O.forward(np64(v), np64(w), DEFAULT_EPS), dtype, f"fwd {shape} {dtype}")


@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_oracle(shape):
    """The reference's backward test (tests/test_triton_op.py:151-182): f64
    inputs rounded to bf16, gradients against f64 autograd of the unrounded
    inputs (dv rel-L2 < 0.03, dw < 0.06) -- and, tighter, against the oracle on
    the rounded inputs at the bf16 floor."""
    n, b, t, d = shape
    gen = torch.Generator().manual_seed(1)
    v64 = torch.randn(n, b, t, d, generator=gen, dtype=torch.float64)
    w64 = torch.randn(d, generator=gen, dtype=torch.float64)
    w64 = w64 / w64.norm()
    g64 = torch.randn(b, t, d, generator=gen, dtype=torch.float64)

    vt = v64.to(torch.bfloat16).to(DEV).requires_grad_(True)
    wt = w64.to(torch.bfloat16).to(DEV).requires_grad_(True)
    gt = g64.to(torch.bfloat16).to(DEV)
    block_attn_res_triton(vt, wt, DEFAULT_EPS).backward(gt)
    assert torch.isfinite(vt.grad).all() and torch.isfinite(wt.grad).all()
    assert vt.grad.dtype == torch.bfloat16 and wt.grad.dtype == torch.bfloat16

    dv_ref, dw_ref = O.backward(v64.numpy(), w64.numpy(), g64.numpy(), DEFAULT_EPS)
    assert O.rel_l2(np64(vt.grad), dv_ref) < 0.03

    dv_o, dw_o = O.backward(np64(vt), np64(wt), np64(gt), DEFAULT_EPS)
    check(vt.grad, dv_o, torch.bfloat16, f"dv {shape}")
    if n == 1:
        # one source: softmax is identically 1, so dw is exactly zero
        assert wt.grad.abs().max().item() == 0.0
        assert torch.equal(vt.grad[0], gt)
    else:
        assert O.rel_l2(np64(wt.grad), dw_ref) < 0.06
        check(wt.grad, dw_o, torch.bfloat16, f"dw {shape}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(4, 2, 128, 512), (9, 1, 64, 2048), (3, 1, 64, 777), (33, 1, 16, 512),
                                   (17, 1, 48, 4096)])
def test_backward_other_dtypes(shape, dtype):
    v, w = make(*shape, dtype, seed=5)
    g = torch.randn(shape[1:], generator=torch.Generator().manual_seed(6)).to(dtype).to(DEV)
    v.requires_grad_(True)
    w.requires_grad_(True)
    block_attn_res_triton(v, w, DEFAULT_EPS).backward(g)
    dv_o, dw_o = O.backward(np64(v), np64(w), np64(g), DEFAULT_EPS)
    check(v.grad, dv_o, dtype, f"dv {shape} {dtype}")
    check(w.grad, dw_o, dtype, f"dw {shape} {dtype}")


@pytest.mark.parametrize(
    ("shape", "n_queries"),
    [((2, 1, 7, 32), 2), ((5, 1, 17, 777), 3), ((9, 1, 16, 2048), 8), ((9, 1, 4, 4096), 4),
     ((9, 1, 32, 2048), 16), ((17, 1, 8, 4096), 8), ((9, 1, 8, 2048), 1), ((3, 2, 5, 64), 5),
     # the row-stream batched kernel: several tokens per stream, S = 16 (32-wide
     # reduce-scatter), S = 9 (two sweeps of pass B), N up to 32
     ((20, 1, 300, 2048), 16), ((17, 1, 200, 4096), 3), ((24, 1, 160, 1024), 9),
     ((32, 2, 80, 1024), 2),
     # the register-tile batched kernel at its edges: one source, N = 8 and 16,
     # 9 to 16 queries (three and six query blocks), 128-column rows, several
     # tokens per group around the ring, 8 KiB rows
     ((1, 1, 9, 64), 3), ((8, 1, 40, 128), 16), ((16, 1, 30, 1024), 9),
     ((16, 1, 200, 2048), 16), ((12, 2, 150, 1024), 12), ((9, 1, 300, 4096), 8),
     ((9, 2, 700, 2048), 8)],
)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_batched_forward_is_at_the_dtype_floor(shape, n_queries, dtype):
    """tests/test_triton_op.py:95-118, plus Q=16 and the off-resident N=17 D=4096 shape."""
    v, _ = make(*shape, dtype)
    q = torch.randn(n_queries, shape[-1], generator=torch.Generator().manual_seed(7))
    q = (q / q.norm(dim=-1, keepdim=True)).to(dtype).to(DEV)
    with torch.no_grad():
        got = block_attn_res_batched(v, q, DEFAULT_EPS)
    assert got.shape == (n_queries, *shape[1:]) and got.dtype == dtype
    want = O.batched(np64(v), np64(q), DEFAULT_EPS)
    check(got, want, dtype, f"batched {shape} Q={n_queries}")
    for i in range(n_queries):
        check(got[i], want[i], dtype, f"batched {shape} q{i}")


@pytest.mark.parametrize("name", golden_cases())
def test_kernels_match_reference_golden_vectors(name):
    """Direct comparison with the reference's own outputs (fixtures made by
    tests/golden/make_golden.py from the reference's reference.py/baselines.py)."""
    z, (v, w, g, q) = load_golden(name)
    dt = str(z["meta_dtype"])
    if dt == "float64":
        pytest.skip("float64-input fixture: oracle-only")
    dtype = getattr(torch, dt)
    sub = int(z["meta_sub"])
    vt = torch.from_numpy(v).to(dtype).to(DEV).requires_grad_(True)
    wt = torch.from_numpy(w).to(dtype).to(DEV).requires_grad_(True)
    gt = torch.from_numpy(g).to(dtype).to(DEV)
    out = block_attn_res_triton(vt, wt, DEFAULT_EPS)
    out.backward(gt)
    check(out[..., ::sub], z["out"], dtype, f"{name} out")
    dv = vt.grad[:, :, :16] if name.startswith("c1_") else vt.grad[..., ::sub]
    check(dv, z["dv"], dtype, f"{name} dv")
    check(wt.grad, z["dw"], dtype, f"{name} dw")
    if "batched" in z:
        with torch.no_grad():
            bo = block_attn_res_batched(vt.detach(), torch.from_numpy(q).to(dtype).to(DEV))
        check(bo[..., ::sub], z["batched"], dtype, f"{name} batched")


@pytest.mark.parametrize("shape", [(9, 1, 64, 2048), (3, 1, 16, 777), (33, 2, 8, 512), (1, 1, 8, 256)])
def test_saved_statistics_match_oracle(shape):
    """The statistics the backward consumes: logits, inverse RMS, max, lse."""
    v, w = make(*shape, torch.bfloat16, seed=3)
    v.requires_grad_(True)
    out = block_attn_res_triton(v, w, DEFAULT_EPS)
    stats = out.grad_fn.saved_tensors[2]
    n, b, t, _ = shape
    lg, r, m, lse = O.forward_stats(np64(v), np64(w), DEFAULT_EPS)
    s = stats.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(s[:, :n], lg.reshape(n, b * t).T, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s[:, n:2 * n], r.reshape(n, b * t).T, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s[:, 2 * n], m.reshape(-1), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(s[:, 2 * n + 1], lse.reshape(-1), rtol=1e-5, atol=1e-5)
    assert out.grad_fn.name() == "_BlockAttnResTritonBackward"
    assert isinstance(out.grad_fn, _BlockAttnResTriton._backward_cls)
