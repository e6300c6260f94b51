"""The fused arena staging step (``sy_stage_partial``) on the GPU.

``stage_partial(partial, out, arena_slot)`` must equal the reference decoder's
``partial + out`` followed by ``arena[len(blocks)].copy_(partial)``
(``src/switchyard/model.py:532-535``) bit for bit: both add in fp32 and round
once to the tensor's dtype. Covers the 16-byte vector path, the element path
(odd lengths, unaligned slots), autograd, and a decoder-style loop whose Block
AttnRes sites read the staged arena.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU runs deselect this module
    pytest.skip("needs a CUDA device", allow_module_level=True)

from switchyard import block_attn_res_triton, stage_partial  # noqa: E402

DEV = "cuda"


def _pair(shape, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    a = torch.randn(*shape, generator=gen).to(dtype).to(DEV)
    b = torch.randn(*shape, generator=gen).to(dtype).to(DEV)
    return a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 4096, 2048), (2, 33, 512), (1, 7, 63), (3, 1, 5)])
def test_stage_partial_equals_add_then_copy(shape, dtype):
    a, b = _pair(shape, dtype, 1)
    arena = torch.full((3,) + shape, 7.0, device=DEV, dtype=dtype)
    got = stage_partial(a, b, arena[1])
    want = a + b
    assert torch.equal(got, want)
    assert torch.equal(arena[1], want)
    assert (arena[0] == 7.0).all() and (arena[2] == 7.0).all()  # neighbours untouched


def test_stage_partial_unaligned_slot_uses_the_element_path():
    a, b = _pair((5, 64), torch.bfloat16, 2)
    flat = torch.zeros(5 * 64 + 1, device=DEV, dtype=torch.bfloat16)
    slot = flat[1:].view(5, 64)  # 2-byte offset: not 16-byte aligned
    got = stage_partial(a, b, slot)
    assert torch.equal(got, a + b) and torch.equal(slot, a + b) and flat[0].item() == 0.0


def test_stage_partial_autograd_and_errors():
    a, b = _pair((2, 16, 256), torch.bfloat16, 3)
    a.requires_grad_(True)
    b.requires_grad_(True)
    slot = torch.empty(2, 16, 256, device=DEV, dtype=torch.bfloat16)
    g = torch.randn(2, 16, 256, device=DEV).to(torch.bfloat16)
    stage_partial(a, b, slot).backward(g)
    assert torch.equal(a.grad, g) and torch.equal(b.grad, g)
    with pytest.raises(ValueError, match="one shape"):
        stage_partial(a.detach(), b.detach()[:1], slot)
    with pytest.raises(ValueError, match="same dtype"):
        stage_partial(a.detach(), b.detach().float(), slot)
    with pytest.raises(ValueError, match="contiguous"):
        stage_partial(a.detach(), b.detach(), torch.empty(256, 16, 2, device=DEV,
                                                           dtype=torch.bfloat16).permute(2, 1, 0))
    empty = torch.empty(0, 8, device=DEV, dtype=torch.bfloat16)
    assert stage_partial(empty, empty, torch.empty_like(empty)).shape == (0, 8)


def test_decoder_loop_with_fused_staging_matches_reference_staging():
    """A decoder-shaped loop (model.py:517-540): sublayer outputs accumulate
    into the partial, staged into the arena, and each site reads the arena's
    filled prefix with block_attn_res_triton. Outputs and gradients with the
    fused staging equal those with add-then-copy, bit for bit."""
    n_sub, block, b, t, d = 6, 3, 1, 64, 512
    gen = torch.Generator().manual_seed(4)
    x0 = torch.randn(b, t, d, generator=gen).to(torch.bfloat16).to(DEV)
    ws = [(torch.randn(d, generator=gen) / d**0.5).to(torch.bfloat16).to(DEV) for _ in range(n_sub)]
    mats = [(torch.randn(d, d, generator=gen) / d**0.5).to(torch.bfloat16).to(DEV) for _ in range(n_sub)]

    def run(fused: bool):
        w_req = [w.clone().requires_grad_(True) for w in ws]
        arena = torch.zeros(n_sub // block + 2, b, t, d, device=DEV, dtype=torch.bfloat16)
        arena[0].copy_(x0)
        blocks, partial = 1, None
        for i in range(n_sub):
            if i and i % block == 0:
                blocks, partial = blocks + 1, None
            n_src = blocks + (partial is not None)
            h = block_attn_res_triton(arena[:n_src].clone(), w_req[i])
            out = torch.tanh(h @ mats[i])
            if partial is None:
                partial = out
                with torch.no_grad():
                    arena[blocks].copy_(partial)
            elif fused:
                partial = stage_partial(partial, out, arena[blocks])
            else:
                partial = partial + out
                with torch.no_grad():
                    arena[blocks].copy_(partial)
        loss = partial.float().square().mean()
        loss.backward()
        return partial.detach(), arena.clone(), [w.grad for w in w_req]

    p1, a1, g1 = run(True)
    p0, a0, g0 = run(False)
    assert torch.equal(p1, p0) and torch.equal(a1, a0)
    # sites of earlier blocks reach the loss only through the arena, which
    # (as in the reference) is written outside autograd: their grads are None
    assert [x is None for x in g1] == [y is None for y in g0]
    assert sum(x is not None for x in g1) >= block
    assert all(x is None or torch.equal(x, y) for x, y in zip(g1, g0))
