"""Behaviour of the drop-in operator on the GPU: the reference's semantic and
rejection tests (tests/test_triton_op.py:210-288), dispatch pins, edge cases,
bit-stability, the model-arena calling pattern, and full-size property checks
at the representative shape (N=9 B=1 T=4096 D=2048 bf16)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attnres_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import (  # noqa: E402
    BlockAttnResTriton,
    block_attn_res_batched,
    block_attn_res_triton,
    speed_of_light,
)
from switchyard import _native  # noqa: E402
from switchyard.triton_op import (  # noqa: E402
    DEFAULT_EPS,
    PLAN_GENERIC,
    PLAN_SMEM_TILE,
    PLAN_STREAM,
    PLAN_TILE,
    _plan,
)

DEV = "cuda"


def np64(t):
    return t.detach().to(torch.float64).cpu().numpy()


def randn(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


def fwd_bwd(v, w, g):
    v = v.detach().requires_grad_(True)
    w = w.detach().requires_grad_(True)
    out = block_attn_res_triton(v, w, DEFAULT_EPS)
    out.backward(g)
    return out.detach(), v.grad, w.grad


# ---------------------------------------------------------------- semantics


def test_zero_query_averages():
    v = randn(6, 2, 64, 512)
    w = torch.zeros(512, device=DEV)
    torch.testing.assert_close(block_attn_res_triton(v, w), v.mean(0), rtol=1e-5, atol=1e-5)


def test_extreme_logits_do_not_overflow():
    """tests/test_triton_op.py:218-225: a query of norm 500 saturates the
    softmax; the max is subtracted before exponentiating."""
    v = randn(8, 1, 128, 1024)
    w = randn(1024, seed=1)
    w = w / w.norm() * 500.0
    got = block_attn_res_triton(v, w)
    assert torch.isfinite(got).all()
    assert O.rel_l2(np64(got), O.forward(np64(v), np64(w))) < 1e-5
    g = randn(1, 128, 1024, seed=2)
    _, dv, dw = fwd_bwd(v, w, g)
    assert torch.isfinite(dv).all() and torch.isfinite(dw).all()


def test_handles_non_contiguous_input():
    base = randn(4, 9, 64, 512, dtype=torch.bfloat16)
    v = base.transpose(0, 1)
    assert not v.is_contiguous()
    w = randn(512, dtype=torch.bfloat16, seed=1) / 22.6
    torch.testing.assert_close(block_attn_res_triton(v, w), block_attn_res_triton(v.contiguous(), w))


def test_batched_handles_non_contiguous_inputs():
    base = randn(2, 5, 11, 63, dtype=torch.bfloat16)
    v = base.transpose(0, 1)
    q = randn(63, 3, dtype=torch.bfloat16, seed=1).T
    torch.testing.assert_close(block_attn_res_batched(v, q), block_attn_res_batched(v.contiguous(), q.contiguous()))


def test_module_matches_functional():
    m = BlockAttnResTriton(256).to(DEV)
    with torch.no_grad():
        m.w.normal_(0, 0.05)
        m.g.normal_(1, 0.05)
    v = randn(5, 1, 64, 256)
    torch.testing.assert_close(m(v), block_attn_res_triton(v, m.w * m.g, m.eps))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("which", ["both", "w", "g"])
def test_module_gain_split_matches_autograd_bitwise(dtype, which):
    """The module folds dq -> (dw = dq * g, dg = dq * w) into the dw reduction
    (sy_dw_reduce_gain); autograd through w * g gives the same bits."""
    m = BlockAttnResTriton(2048).to(DEV).to(dtype)
    with torch.no_grad():
        m.w.copy_(randn(2048, seed=31) / 2048**0.5)
        m.g.copy_(1 + 0.1 * randn(2048, seed=32))
    m.w.requires_grad_(which in ("both", "w"))
    m.g.requires_grad_(which in ("both", "g"))
    v = randn(9, 1, 300, 2048, dtype=torch.bfloat16, seed=33).requires_grad_(True)
    gout = randn(1, 300, 2048, dtype=torch.bfloat16, seed=34)
    out = m(v)
    out.backward(gout)
    w2 = m.w.detach().clone().requires_grad_(m.w.requires_grad)
    g2 = m.g.detach().clone().requires_grad_(m.g.requires_grad)
    v2 = v.detach().clone().requires_grad_(True)
    out2 = block_attn_res_triton(v2, w2 * g2, m.eps)
    out2.backward(gout)
    assert torch.equal(out, out2) and torch.equal(v.grad, v2.grad)
    for p1, p2 in ((m.w, w2), (m.g, g2)):
        if p1.requires_grad:
            assert p1.grad.dtype == dtype and torch.equal(p1.grad, p2.grad)
        else:
            assert p1.grad is None


def test_module_starts_from_uniform_attention():
    m = BlockAttnResTriton(128).to(DEV)
    v = randn(7, 1, 32, 128)
    torch.testing.assert_close(m(v), v.mean(0), rtol=1e-5, atol=1e-5)


def test_query_dtype_may_differ_from_sources():
    """The reference loads w in any dtype and returns dw in w's dtype
    (triton_op.py:67, :563)."""
    v = randn(5, 1, 32, 512, dtype=torch.bfloat16)
    w = randn(512, seed=3) / 22.6  # fp32 query, bf16 sources
    g = randn(1, 32, 512, dtype=torch.bfloat16, seed=4)
    out, dv, dw = fwd_bwd(v, w, g)
    assert out.dtype == torch.bfloat16 and dv.dtype == torch.bfloat16 and dw.dtype == torch.float32
    dv_o, dw_o = O.backward(np64(v), np64(w), np64(g))
    assert O.rel_l2(np64(dw), dw_o) < 1e-5
    assert O.rel_l2(np64(dv), dv_o) <= 1.005 * O.dtype_floor(dv_o, "bfloat16")


# ---------------------------------------------------------------- rejections


@pytest.mark.parametrize("bad", ["rank", "query", "cpu"])
def test_rejects_bad_input(bad):
    v = randn(4, 1, 8, 32)
    w = randn(32)
    if bad == "rank":
        with pytest.raises(ValueError, match=r"\[N, B, T, D\]"):
            block_attn_res_triton(v[0], w)
    elif bad == "query":
        with pytest.raises(ValueError, match="w must be"):
            block_attn_res_triton(v, randn(31))
    else:
        with pytest.raises(ValueError, match="CUDA"):
            block_attn_res_triton(v.cpu(), w.cpu())


def test_batched_rejects_gradients_and_bad_inputs():
    v = randn(4, 1, 8, 32)
    q = randn(3, 32)
    with pytest.raises(RuntimeError, match="no backward"):
        block_attn_res_batched(v.clone().requires_grad_(), q)
    with pytest.raises(ValueError, match="same dtype"):
        block_attn_res_batched(v, q.half())
    with pytest.raises(ValueError, match="CUDA"):
        block_attn_res_batched(v.cpu(), q.cpu())
    with pytest.raises(ValueError, match="positive"):
        block_attn_res_batched(v[:0], q)


# ---------------------------------------------------------------- dispatch


def test_dispatch_sends_the_representative_shape_to_the_tile_kernels():
    """tests/test_triton_op.py:271-288: N=9, D=2048 is the shape a Block
    AttnRes model spends most of its time in; pin its path."""
    # 4 KiB rows: the re-read row-stream forward, the register-tile backward
    assert _plan("fwd", 9, 4096, 2048, torch.bfloat16) == PLAN_STREAM
    assert _plan("bwd", 9, 4096, 2048, torch.bfloat16) == PLAN_TILE
    for n in range(1, 10):  # every source count the 24-layer 8-block model uses
        assert _plan("fwd", n, 8192, 2048, torch.bfloat16) == PLAN_STREAM
        assert _plan("bwd", n, 8192, 2048, torch.bfloat16) == PLAN_TILE
    # shorter rows: the register-tile forward
    assert _plan("fwd", 9, 4096, 512, torch.bfloat16) == PLAN_TILE
    # more sources than the register tile holds: the row-stream forward
    assert _plan("fwd", 17, 4096, 2048, torch.bfloat16) == PLAN_STREAM
    # rows or source counts the register-tile backward cannot hold: the
    # row-stream backward (K warps per token, rows read twice)
    for n, d in ((9, 8192), (17, 4096), (17, 2048), (32, 4096)):
        assert _plan("bwd", n, 4096, d, torch.bfloat16) == PLAN_STREAM
    # batched queries: the register tile reused across queries; tiles that do
    # not fit registers (N=17, D=4096) take the row-stream batched kernel
    for s in (2, 4, 8, 16):
        assert _plan("batched", 9, 4096, 2048, torch.bfloat16, s) == PLAN_TILE
    assert _plan("batched", 17, 4096, 4096, torch.bfloat16, 8) == PLAN_STREAM
    assert _plan("batched", 33, 4096, 4096, torch.bfloat16, 8) == PLAN_GENERIC  # N > 32
    # rows that are not a multiple of 16 bytes take the generic kernels
    assert _plan("fwd", 3, 64, 777, torch.bfloat16) == PLAN_GENERIC
    assert _plan("bwd", 5, 17, 63, torch.float32) == PLAN_GENERIC


# ---------------------------------------------------------------- edge cases


EPS_SHAPES = [  # fp32 shapes that reach every kernel family
    ((9, 1, 64, 1024), PLAN_STREAM, PLAN_TILE),  # 4 KiB rows: re-read row stream
    ((7, 2, 16, 512), PLAN_STREAM, PLAN_TILE),  # 2 KiB rows: re-read row stream, 4 chunks/lane
    ((7, 2, 16, 256), PLAN_TILE, PLAN_TILE),
    ((9, 1, 48, 256), PLAN_TILE, PLAN_TILE),
    ((17, 1, 40, 1024), PLAN_STREAM, PLAN_STREAM),  # backward: 2 warps per token
    ((10, 1, 24, 2048), PLAN_STREAM, PLAN_STREAM),  # 8 KiB rows: split row streams
    ((10, 1, 24, 1536), PLAN_SMEM_TILE, PLAN_STREAM),  # backward: 3 warps per token
    ((33, 1, 24, 512), PLAN_STREAM, PLAN_STREAM),  # backward: 1 warp per token, N > 32
    ((33, 1, 24, 768), PLAN_STREAM, PLAN_STREAM),  # 3 KiB rows: 2 chunks per lane, 3 warps
    ((33, 1, 24, 648), PLAN_STREAM, PLAN_SMEM_TILE),  # 162 chunks a row: the shared-memory tile
    ((3, 1, 16, 777), PLAN_GENERIC, PLAN_GENERIC),
]


@pytest.mark.parametrize("eps", [DEFAULT_EPS, 0.25])
@pytest.mark.parametrize("shape,fwd_kind,bwd_kind", EPS_SHAPES)
def test_eps_reaches_every_kernel(shape, fwd_kind, bwd_kind, eps):
    """eps is an argument of every kernel, not a constant: a source row of
    zeros gets r = eps**-1/2 and logit 0 (not NaN), and a large eps changes
    every logit (reference.py:98-104)."""
    n, b, t, d = shape
    assert _plan("fwd", n, b * t, d, torch.float32) == fwd_kind
    assert _plan("bwd", n, b * t, d, torch.float32) == bwd_kind
    v = randn(*shape, seed=21)
    v[2, :, ::3] = 0.0  # every third token has an all-zero source 2
    w = randn(d, seed=22) / d**0.5
    g = randn(b, t, d, seed=23)
    v = v.detach().requires_grad_(True)
    w = w.detach().requires_grad_(True)
    out = block_attn_res_triton(v, w, eps)
    out.backward(g)
    assert torch.isfinite(out).all() and torch.isfinite(v.grad).all()
    np.testing.assert_allclose(np64(out), O.forward(np64(v), np64(w), eps), rtol=2e-5, atol=2e-6)
    dv_o, dw_o = O.backward(np64(v), np64(w), np64(g), eps)
    np.testing.assert_allclose(np64(v.grad), dv_o, rtol=2e-4, atol=2e-5)
    # dw sums B*T tokens: absolute error scales with its largest entries
    np.testing.assert_allclose(np64(w.grad), dw_o, rtol=2e-4, atol=2e-6 * np.abs(dw_o).max())


def test_empty_token_axis():
    v = randn(3, 2, 0, 64).requires_grad_(True)
    w = randn(64).requires_grad_(True)
    out = block_attn_res_triton(v, w)
    assert out.shape == (2, 0, 64)
    out.sum().backward()
    assert v.grad.shape == v.shape and torch.equal(w.grad, torch.zeros_like(w))


@pytest.mark.parametrize("shape", [(1, 1, 1, 8), (2, 1, 1, 3), (4, 1, 3, 1), (3, 1, 2, 9), (64, 1, 4, 64), (65, 1, 2, 40)])
def test_tiny_and_ragged_shapes(shape):
    v = randn(*shape, seed=9)
    w = randn(shape[-1], seed=10) / max(1.0, shape[-1] ** 0.5)
    g = randn(*shape[1:], seed=11)
    out, dv, dw = fwd_bwd(v, w, g)
    np.testing.assert_allclose(np64(out), O.forward(np64(v), np64(w)), rtol=2e-5, atol=2e-6)
    dv_o, dw_o = O.backward(np64(v), np64(w), np64(g))
    np.testing.assert_allclose(np64(dv), dv_o, rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(np64(dw), dw_o, rtol=2e-4, atol=2e-5)


def test_misaligned_views_take_the_generic_path_and_agree():
    """A view starting 2 bytes into its storage cannot be bulk-copied; it must
    still be right."""
    base = randn(2 * 9 * 64 * 256 + 1, dtype=torch.bfloat16)
    v = base[1:].view(9, 2, 64, 256)
    assert v.is_contiguous() and v.data_ptr() % 16 != 0
    w = randn(256, dtype=torch.bfloat16, seed=1) / 16
    want = O.forward(np64(v), np64(w))
    floor = O.dtype_floor(want, "bfloat16")
    for x in (v, v.clone()):  # generic kernel, then the tile kernel on an aligned copy
        assert O.rel_l2(np64(block_attn_res_triton(x, w)), want) <= 1.005 * floor


def test_arena_alias_pattern():
    """model.py:325-369: the op runs on a `set_` alias of an arena slice under
    enable_grad inside a custom Function, and its backward runs through
    autograd.grad. The alias must be used in place (no copy) and gradients
    must match a plain call."""
    n_src, b, t, d = 5, 2, 32, 256
    arena = randn(n_src + 3, b, t, d, dtype=torch.bfloat16)
    alias = torch.empty(0, dtype=arena.dtype, device=DEV)
    alias.set_(arena.untyped_storage(), arena.storage_offset(), (n_src, b, t, d), arena.stride())
    w = (randn(d, dtype=torch.bfloat16, seed=1) / 16).requires_grad_(True)
    with torch.enable_grad():
        va = alias.requires_grad_(True)
        out = block_attn_res_triton(va, w)
    assert out.grad_fn.saved_tensors[0].data_ptr() == arena.data_ptr()  # no copy
    g = randn(b, t, d, dtype=torch.bfloat16, seed=2)
    dv, dw = torch.autograd.grad(out, (va, w), g)
    ref_v = arena[:n_src].clone().requires_grad_(True)
    ref_w = w.detach().clone().requires_grad_(True)
    block_attn_res_triton(ref_v, ref_w).backward(g)
    assert torch.equal(dv, ref_v.grad) and torch.equal(dw, ref_w.grad)


# ---------------------------------------------------------------- determinism


def test_row_stream_batched_is_bit_stable():
    v = randn(17, 1, 700, 4096, dtype=torch.bfloat16, seed=3)
    q = randn(8, 4096, dtype=torch.bfloat16, seed=4, scale=4096 ** -0.5)
    assert _plan("batched", 17, 700, 4096, torch.bfloat16, 8) == PLAN_STREAM
    with torch.no_grad():
        a = block_attn_res_batched(v, q)
        b = block_attn_res_batched(v, q)
    assert torch.equal(a, b)
    toks = torch.arange(0, 700, 37)
    want = O.batched(np64(v[:, :, toks]), np64(q))
    assert O.rel_l2(np64(a[:, :, toks]), want) <= 1.005 * O.dtype_floor(want, "bfloat16")


@pytest.mark.parametrize("shape", [(9, 1, 4096, 2048), (4, 2, 128, 512), (17, 1, 64, 2048), (3, 1, 64, 777)])
def test_bit_stable_across_runs(shape):
    v = randn(*shape, dtype=torch.bfloat16)
    w = randn(shape[-1], dtype=torch.bfloat16, seed=1) / shape[-1] ** 0.5
    g = randn(*shape[1:], dtype=torch.bfloat16, seed=2)
    a = fwd_bwd(v, w, g)
    b = fwd_bwd(v, w, g)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


# ---------------------------------------------------------------- full size


def test_representative_shape_full_size_properties():
    """The representative shape (N=9 B=1 T=4096 D=2048 bf16, v~N(0,1), w~N(0,1/D),
    dout~N(0,1)). Tokens are independent, so out and dv are checked exactly
    against the oracle on a sample of tokens; dw (a sum over every token) is
    checked against a chunked float64 sum over all of them."""
    n, b, t, d = 9, 1, 4096, 2048
    v = randn(n, b, t, d, dtype=torch.bfloat16, seed=0)
    w = randn(d, dtype=torch.bfloat16, seed=1, scale=d ** -0.5)
    g = randn(b, t, d, dtype=torch.bfloat16, seed=2)
    out, dv, dw = fwd_bwd(v, w, g)
    toks = torch.randperm(t, generator=torch.Generator().manual_seed(5))[:96].sort().values
    vs, gs = np64(v[:, :, toks]), np64(g[:, toks])
    ww = np64(w)
    o_ref = O.forward(vs, ww)
    dv_ref, _ = O.backward(vs, ww, gs)
    assert O.rel_l2(np64(out[:, toks]), o_ref) <= 1.005 * O.dtype_floor(o_ref, "bfloat16")
    assert O.rel_l2(np64(dv[:, :, toks]), dv_ref) <= 1.005 * O.dtype_floor(dv_ref, "bfloat16")
    v64, g64 = np64(v), np64(g)
    dw_ref = np.zeros(d)
    for c in range(0, t, 512):
        dw_ref += O.backward(v64[:, :, c:c + 512], ww, g64[:, c:c + 512])[1]
    assert O.rel_l2(np64(dw), dw_ref) <= 1.005 * O.dtype_floor(dw_ref, "bfloat16")
    sol = speed_of_light(v)
    s_ref = O.speed_of_light(np64(v[:, :, toks]))
    assert O.rel_l2(np64(sol[:, toks]), s_ref) <= 1.005 * O.dtype_floor(s_ref, "bfloat16")


@pytest.mark.parametrize("shape", [(9, 1, 600, 2048), (9, 1, 300, 4096), (9, 1, 150, 8192),
                                   (3, 1, 60, 16384), (9, 1, 600, 1024), (4, 2, 100, 1800)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_forward_same_bits_for_16bit_and_fp32_queries(shape, dtype):
    """A query of the sources' own 16-bit type takes the packed mixed-precision
    dot product (fma.rn.f32.{bf16,f16} on the 16-bit halves); the same values
    as an fp32 query take the unpacked path. Products are exact and the
    accumulation order is the same, so out and the statistics agree bitwise."""
    n, b, t, d = shape
    v = randn(*shape, dtype=dtype, seed=7)
    w = randn(d, dtype=dtype, seed=8, scale=d ** -0.5)
    out16 = block_attn_res_triton(v, w)
    out32 = block_attn_res_triton(v, w.float())
    assert torch.equal(out16, out32)
    stats = [torch.empty(b * t, _native.stats_stride(n), device=DEV) for _ in range(2)]
    o = [torch.empty(b, t, d, dtype=dtype, device=DEV) for _ in range(2)]
    _native.fwd(v, w, o[0], stats[0], n, b * t, d, DEFAULT_EPS)
    _native.fwd(v, w.float(), o[1], stats[1], n, b * t, d, DEFAULT_EPS)
    assert torch.equal(o[0], o[1]) and torch.equal(stats[0], stats[1])


@pytest.mark.parametrize("shape", [(40, 1, 64, 2048), (36, 1, 48, 1024), (40, 1, 24, 4096)])
def test_statistics_of_more_than_32_sources(shape):
    """The row-stream forwards keep row n's statistics in lane n for n < 32 and
    write later rows directly; the backward reads them back (re-read stream at
    4 and 2 KiB rows, split stream at 8 KiB rows)."""
    n, b, t, d = shape
    assert _plan("fwd", n, b * t, d, torch.bfloat16) == PLAN_STREAM
    v = randn(*shape, dtype=torch.bfloat16, seed=41)
    w = randn(d, dtype=torch.bfloat16, seed=42, scale=d ** -0.5)
    g = randn(b, t, d, dtype=torch.bfloat16, seed=43)
    out, dv, dw = fwd_bwd(v, w, g)
    o_ref = O.forward(np64(v), np64(w))
    dv_ref, dw_ref = O.backward(np64(v), np64(w), np64(g))
    assert O.rel_l2(np64(out), o_ref) <= 1.005 * O.dtype_floor(o_ref, "bfloat16")
    assert O.rel_l2(np64(dv), dv_ref) <= 1.005 * O.dtype_floor(dv_ref, "bfloat16")
    assert O.rel_l2(np64(dw), dw_ref) <= 1.005 * O.dtype_floor(dw_ref, "bfloat16")


@pytest.mark.parametrize("shape,dtype", [
    ((9, 1, 1024, 8192), torch.bfloat16),   # 16 KiB rows: 8 warps per token, 4 tokens per stream
    ((17, 1, 1024, 4096), torch.bfloat16),  # N > 16: 4 warps per token
    ((24, 1, 1200, 2048), torch.float16),   # 2 warps per token, 6-7 rows in each ring
])
def test_row_stream_backward_many_tokens_per_stream(shape, dtype):
    """The row-stream backward with several tokens per token stream (the ring
    wraps many times, the G exchange alternates its two buffers): dv on a
    sample of tokens against the oracle, dw against a chunked float64 sum over
    every token, both at the dtype's rounding floor, and bitwise stable."""
    n, b, t, d = shape
    assert _plan("bwd", n, b * t, d, dtype) == PLAN_STREAM
    name = {torch.bfloat16: "bfloat16", torch.float16: "float16"}[dtype]
    v = randn(*shape, dtype=dtype, seed=3)
    w = randn(d, dtype=dtype, seed=4, scale=d ** -0.5)
    g = randn(b, t, d, dtype=dtype, seed=5)
    out, dv, dw = fwd_bwd(v, w, g)
    out2, dv2, dw2 = fwd_bwd(v, w, g)
    assert torch.equal(out, out2) and torch.equal(dv, dv2) and torch.equal(dw, dw2)
    toks = torch.randperm(t, generator=torch.Generator().manual_seed(6))[:64].sort().values
    ww = np64(w)
    dv_ref, _ = O.backward(np64(v[:, :, toks]), ww, np64(g[:, toks]))
    assert O.rel_l2(np64(dv[:, :, toks]), dv_ref) <= 1.005 * O.dtype_floor(dv_ref, name)
    dw_ref = np.zeros(d)
    for c in range(0, t, 256):
        dw_ref += O.backward(np64(v[:, :, c:c + 256]), ww, np64(g[:, c:c + 256]))[1]
    assert O.rel_l2(np64(dw), dw_ref) <= 1.005 * O.dtype_floor(dw_ref, name)


@pytest.mark.parametrize("shape,dtype", [
    ((33, 1, 600, 2048), torch.bfloat16),   # N > 32: two coefficient slots per lane, K = 2
    ((64, 1, 300, 4096), torch.bfloat16),   # N = 64, the row stream's maximum, K = 4
    ((33, 1, 900, 1024), torch.bfloat16),   # 2 KiB rows: one warp per token (K = 1)
    ((17, 2, 700, 1024), torch.float16),    # K = 1 with N <= 32
    ((40, 1, 500, 512), torch.float32),     # fp32 2 KiB rows, K = 1, two slots
    ((17, 1, 400, 1536), torch.bfloat16),   # 3 KiB rows: 2 chunks per lane, K = 3
    ((20, 1, 300, 1280), torch.bfloat16),   # 2.5 KiB rows: 1 chunk per lane, K = 5
])
def test_row_stream_backward_beyond_32_sources_and_2kib_rows(shape, dtype):
    """The row-stream backward with the per-source coefficients in two
    register slots per lane (N = 33..64) and with one warp per token (2 KiB
    rows): dv on sampled tokens and dw over every token against the float64
    oracle at the dtype's rounding floor, bitwise stable."""
    n, b, t, d = shape
    assert _plan("bwd", n, b * t, d, dtype) == PLAN_STREAM
    name = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}[dtype]
    v = randn(*shape, dtype=dtype, seed=13)
    w = randn(d, dtype=dtype, seed=14, scale=d ** -0.5)
    g = randn(b, t, d, dtype=dtype, seed=15)
    out, dv, dw = fwd_bwd(v, w, g)
    _, dv2, dw2 = fwd_bwd(v, w, g)
    assert torch.equal(dv, dv2) and torch.equal(dw, dw2)
    toks = torch.randperm(t, generator=torch.Generator().manual_seed(16))[:32].sort().values
    ww = np64(w)
    dv_ref, _ = O.backward(np64(v[:, :, toks]), ww, np64(g[:, toks]))
    floor = (lambda ref: O.dtype_floor(ref, name)) if dtype != torch.float32 else (
        lambda ref: max(1.6 * O.dtype_floor(ref, name), 1e-6) / 1.005)
    assert O.rel_l2(np64(dv[:, :, toks]), dv_ref) <= 1.005 * floor(dv_ref)
    dw_ref = np.zeros(d)
    for c in range(0, t, 128):
        dw_ref += O.backward(np64(v[:, :, c:c + 128]), ww, np64(g[:, c:c + 128]))[1]
    assert O.rel_l2(np64(dw), dw_ref) <= 1.005 * floor(dw_ref)


def test_backward_accumulates_dw_in_fp32():
    """tests/test_triton_op.py:185-207: dw over 8192 tokens stays accurate."""
    n, b, t, d = 9, 1, 8192, 512
    gen = torch.Generator().manual_seed(2)
    v64 = torch.randn(n, b, t, d, generator=gen, dtype=torch.float64)
    w64 = torch.randn(d, generator=gen, dtype=torch.float64)
    w64 = w64 / w64.norm()
    g64 = torch.randn(b, t, d, generator=gen, dtype=torch.float64)
    _, _, dw = fwd_bwd(v64.to(torch.bfloat16).to(DEV), w64.to(torch.bfloat16).to(DEV),
                       g64.to(torch.bfloat16).to(DEV))
    _, dw_ref = O.backward(v64.numpy(), w64.numpy(), g64.numpy())
    assert O.rel_l2(np64(dw), dw_ref) < 0.06


def test_no_device_error_recorded():
    """No kernel's bounded wait ran out during this session's tests."""
    torch.cuda.synchronize()
    assert _native.device_error() == 0
