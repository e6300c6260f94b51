"""sy_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers cannot hand the library a scratch buffer -- code inside a host
framework that owns all device memory and allows no raw allocation, or a
latency-critical loop that must not allocate. For them sy_bwd_noalloc keeps the
backward's fp32 dw partial rows in a fixed array inside the library. This test
calls it through the C ABI and checks that dv and dw equal what the regular
entry points (sy_bwd with a caller buffer, then sy_dw_reduce) produce, for two
calls in a row with different inputs (the shared array keeps the previous
call's contents, which must not leak into the next result). This file is named
to be collected last.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import _native  # noqa: E402

DEV = "cuda"
EPS = 1e-6


def _inputs(n, bt, d, seed):
    gen = torch.Generator().manual_seed(seed)
    v = torch.randn(n, bt, d, generator=gen).to(torch.bfloat16).to(DEV)
    w = (torch.randn(d, generator=gen) / d**0.5).to(torch.bfloat16).to(DEV)
    g = torch.randn(bt, d, generator=gen).to(torch.bfloat16).to(DEV)
    stats = torch.empty(bt, _native.stats_stride(n), device=DEV)
    out = torch.empty(bt, d, device=DEV, dtype=torch.bfloat16)
    _native.fwd(v, w, out, stats, n, bt, d, EPS)
    return v, w, g, stats


def _regular(v, w, g, stats):
    n, bt, d = v.shape
    dv = torch.empty_like(v)
    part = torch.empty(_native.bwd_partials(n, bt, d, v.dtype), d, device=DEV)
    dw = torch.empty(d, device=DEV, dtype=w.dtype)
    _native.bwd(v, w, g, stats, dv, part, n, bt, d, EPS)
    _native.dw_reduce(part, dw)
    return dv, dw


def _noalloc(v, w, g, stats):
    n, bt, d = v.shape
    dv = torch.empty_like(v)
    dw = torch.empty(d, device=DEV, dtype=w.dtype)
    st = _native.lib.sy_bwd_noalloc(
        v.data_ptr(), w.data_ptr(), g.data_ptr(), stats.data_ptr(), dv.data_ptr(), dw.data_ptr(),
        n, bt, d, _native.dtype_code(v.dtype), _native.dtype_code(w.dtype), EPS,
        _native.stream_of(v))
    _native.check(st, "sy_bwd_noalloc")
    return dv, dw


@pytest.mark.parametrize("shape", [(9, 4096, 2048), (4, 1000, 512), (3, 64, 777)])
def test_noalloc_backward_matches_the_regular_entry_points(shape):
    n, bt, d = shape
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        v, w, g, stats = _inputs(n, bt, d, seed)
        dv_ref, dw_ref = _regular(v, w, g, stats)
        dv, dw = _noalloc(v, w, g, stats)
        torch.cuda.synchronize()
        # Same kernels and the same partial-row partition: equal bit for bit,
        # which is tighter than the 1.005x-floor tolerance the parity tests use.
        assert torch.equal(dv, dv_ref), f"dv differs on call {call}"
        assert torch.equal(dw, dw_ref), f"dw differs on call {call}"


def test_noalloc_rejects_shapes_beyond_its_scratch():
    cap = int(_native.lib.sy_bwd_noalloc_max_floats())
    n, d = 2, 65536  # partial rows x D far beyond the fixed array
    bt = 4096
    assert _native.bwd_partials(n, bt, d, torch.bfloat16) * d > cap
    st = _native.lib.sy_bwd_noalloc(1, 1, 1, 1, 1, 1, n, bt, d, _native.SY_BF16, _native.SY_BF16,
                                    EPS, None)
    assert st == _native.SY_ERR_SCRATCH
    assert b"sy_bwd_noalloc" in _native.lib.sy_status_string(st)
