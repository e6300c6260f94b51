"""The Python drop-in API's argument checks, on CPU tensors (no GPU needed).

Mirrors the rejection tests of the reference (tests/test_triton_op.py:256-268,
:132-142): same exception types and the same message fragments, raised before
anything reaches the native library.
"""

from __future__ import annotations

import pytest
import torch

from switchyard import BlockAttnResTriton, block_attn_res_batched, block_attn_res_triton
from switchyard.triton_op import DEFAULT_EPS


def test_rejects_wrong_rank():
    with pytest.raises(ValueError, match=r"\[N, B, T, D\]"):
        block_attn_res_triton(torch.randn(1, 8, 32), torch.randn(32), DEFAULT_EPS)


def test_rejects_wrong_query_shape():
    with pytest.raises(ValueError, match="w must be"):
        block_attn_res_triton(torch.randn(4, 1, 8, 32), torch.randn(31), DEFAULT_EPS)


def test_rejects_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        block_attn_res_triton(torch.randn(4, 1, 8, 32), torch.randn(32), DEFAULT_EPS)


def test_batched_rejects_bad_shapes_and_cpu():
    v = torch.randn(4, 1, 8, 32)
    with pytest.raises(ValueError, match=r"\[N, B, T, D\]"):
        block_attn_res_batched(v[0], torch.randn(3, 32))
    with pytest.raises(ValueError, match="queries must be"):
        block_attn_res_batched(v, torch.randn(3, 31))
    with pytest.raises(ValueError, match="CUDA"):
        block_attn_res_batched(v, torch.randn(3, 32))


def test_module_initialisation_matches_reference():
    """Zero query, unit gain (reference.py:167-172; triton_op.py:600-605)."""
    m = BlockAttnResTriton(64)
    assert torch.equal(m.w, torch.zeros(64)) and torch.equal(m.g, torch.ones(64))
    assert BlockAttnResTriton(64, norm_affine=False).g is None
    assert "d_model=64" in repr(m)


def test_public_names_match_the_reference_module():
    import switchyard.triton_op as op

    for name in ("block_attn_res_triton", "block_attn_res_batched", "BlockAttnResTriton",
                 "speed_of_light", "_BlockAttnResTriton"):
        assert hasattr(op, name)


def test_stage_partial_rejects_cpu_tensors():
    from switchyard import stage_partial

    a = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="CUDA"):
        stage_partial(a, a, torch.zeros(4, 8))
