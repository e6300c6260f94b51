"""The benchmark's own checkers and bookkeeping, on the CPU.

``bench.py --grid`` checks every shape of the benchmark grid with a float64
evaluation on the GPU (``f64_tokens`` / ``f64_dw``); here those functions are
pinned to the oracle, and the byte model and the summary statistics to their
definitions.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import bench  # noqa: E402
from oracle import attnres_oracle as O  # noqa: E402


def test_float64_checker_matches_the_oracle():
    g = torch.Generator().manual_seed(3)
    n, k, d = 7, 11, 96
    v = torch.randn(n, k, d, generator=g, dtype=torch.float64)
    w = torch.randn(d, generator=g, dtype=torch.float64) / d**0.5
    dout = torch.randn(k, d, generator=g, dtype=torch.float64)
    out, dv, dw = bench.f64_tokens(v, w, dout)
    vo, go = v.numpy()[:, None], dout.numpy()[None]
    np.testing.assert_allclose(out.numpy(), O.forward(vo, w.numpy())[0], rtol=1e-12, atol=1e-14)
    dv_o, dw_o = O.backward(vo, w.numpy(), go)
    np.testing.assert_allclose(dv.numpy(), dv_o[:, 0], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(dw.numpy(), dw_o, rtol=1e-12, atol=1e-13)
    np.testing.assert_allclose(bench.f64_dw(v, w, dout).numpy(), dw_o, rtol=1e-12, atol=1e-13)
    # the eps argument reaches the checker
    out_e, _, _ = bench.f64_tokens(v, w, dout, eps=0.5)
    np.testing.assert_allclose(out_e.numpy(), O.forward(vo, w.numpy(), 0.5)[0], rtol=1e-12, atol=1e-14)


def test_checker_metrics_match_the_oracles():
    g = torch.Generator().manual_seed(4)
    want = torch.randn(4096, generator=g, dtype=torch.float64)
    got = want.to(torch.bfloat16)
    assert abs(bench.rel_l2_t(got, want) - O.rel_l2(got.double().numpy(), want.numpy())) < 1e-15
    assert abs(bench.bf16_floor(want) - O.dtype_floor(want.numpy(), "bfloat16")) < 1e-12


def test_byte_model_and_summary():
    fwd, bwd, tot = bench.alg_bytes(9, 1, 4096, 2048)
    assert fwd == 167_772_160 == O.attn_res_min_bytes(9, 1, 4096, 2048, 2)
    assert tot == 486_539_264 and bwd == tot - fwd
    s = bench.summarize([1.0, 2.0, 3.0, 10.0])
    assert s["median_ms"] == 3.0 and s["min_ms"] == 1.0 and s["max_ms"] == 10.0
    assert s["slow_steps"]["count"] == 1 and s["slow_steps"]["first_indices"] == [3]


def test_grid_covers_baseline_config_4():
    assert bench.GRID_N == (2, 3, 5, 9, 17, 33)
    assert bench.GRID_B == (1, 4)
    assert bench.GRID_T == (4096, 16384, 65536)
    assert bench.GRID_D == (1024, 2048, 4096, 8192)
