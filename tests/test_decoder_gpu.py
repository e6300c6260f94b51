"""The decoder on the GPU with this package's kernels: the reference's own model
checks (``tests/test_model.py`` of the reference) run against
``switchyard.decoder``, plus the reference decoder's golden fixture.

* fused mode (``"switchyard"``) against the reference decoder's fixture
  (``decoder_golden.npz``, written by the reference's ``model.py``) within the
  reference's framework-vs-fused bar: loss to 1e-5 relative, gradients to 1e-5
  relative L2 (``tests/test_model.py:147-162``);
* arena and stack agree: forward bitwise, gradients to 1e-6 relative L2
  (``:106-144``);
* framework and fused modes agree on the reference test's own configuration
  (``:147-162``);
* it trains: 60 AdamW steps on one batch halve the loss (``:190-208``);
* zero-initialised queries give uniform attention at every site, and a bf16
  model's step runs the fused kernels end to end.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent))
from test_decoder import flat_grads, load_golden_decoder  # noqa: E402

DEV = "cuda"


def _cfg(**kw):
    """The reference test's configuration (tests/test_model.py:29-35)."""
    from switchyard.decoder import DecoderConfig

    base = dict(vocab_size=512, d_model=128, n_heads=4, d_ff=256, n_layers=6, n_blocks=3,
                max_seq_len=64)
    base.update(kw)
    return DecoderConfig(**base)


def _build(residual, sources, seed=0, dtype=torch.float32):
    from switchyard.decoder import Decoder

    torch.manual_seed(seed)
    return Decoder(_cfg(residual=residual, sources=sources)).to(DEV, dtype)


def _batch(b=2, t=32, vocab=512):
    torch.manual_seed(99)
    return (torch.randint(0, vocab, (b, t), device=DEV),
            torch.randint(0, vocab, (b, t), device=DEV))


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("residual", ["switchyard", "attnres"])
@pytest.mark.parametrize("sources", ["arena", "stack"])
def test_matches_the_reference_decoder_fixture(residual, sources):
    model, idx, tgt, z = load_golden_decoder(residual, sources, DEV)
    logits, loss = model(idx, tgt)
    loss.backward()
    np.testing.assert_allclose(loss.item(), float(z["loss"]), rtol=1e-5, atol=1e-5)
    want = torch.cat([torch.from_numpy(z[f"grad:{n}"]).flatten()
                      for n, _ in sorted(model.named_parameters())]).to(DEV)
    assert _rel(flat_grads(model), want) < 1e-5
    np.testing.assert_allclose(logits.detach().cpu().numpy(), z["logits"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("residual", ["switchyard", "attnres"])
def test_arena_and_stack_agree(residual):
    idx, tgt = _batch()
    outs = {}
    for sources in ("stack", "arena"):
        m = _build(residual, sources)
        logits, loss = m(idx, tgt)
        loss.backward()
        outs[sources] = (loss.detach(), logits.detach(), flat_grads(m))
    assert torch.equal(outs["arena"][0], outs["stack"][0])
    assert torch.equal(outs["arena"][1], outs["stack"][1])
    assert _rel(outs["arena"][2], outs["stack"][2]) < 1e-6


def test_framework_and_fused_modes_agree():
    idx, tgt = _batch()
    ref = _build("attnres", "arena")
    ours = _build("switchyard", "arena")
    _, l1 = ref(idx, tgt)
    _, l2 = ours(idx, tgt)
    l1.backward()
    l2.backward()
    torch.testing.assert_close(l2, l1, rtol=1e-5, atol=1e-5)
    assert _rel(flat_grads(ours), flat_grads(ref)) < 1e-5


@pytest.mark.parametrize("residual", ["standard", "switchyard"])
def test_overfits_a_fixed_batch(residual):
    m = _build(residual, "arena")
    opt = torch.optim.AdamW(m.parameters(), lr=3e-3)
    idx, tgt = _batch()
    first = None
    for _ in range(60):
        opt.zero_grad(set_to_none=True)
        _, loss = m(idx, tgt)
        loss.backward()
        opt.step()
        if first is None:
            first = loss.item()
    assert torch.isfinite(loss)
    assert loss.item() < first * 0.5, f"{residual}: {first:.3f} -> {loss.item():.3f}"


def test_initial_attention_is_uniform():
    """Zero queries: every site's output is the plain mean of its sources, so
    the fused model equals the framework model with any gains."""
    from oracle import attnres_oracle as O

    m = _build("switchyard", "arena")
    v = torch.randn(5, 2, 8, 128, device=DEV)
    site = m.attn_res[0]
    from switchyard.decoder import _ArenaSite

    arena = v.clone()
    out = _ArenaSite.apply(site.w, site.g, arena, 5, False, 1e-6, True, *v.unbind(0))
    np.testing.assert_allclose(out.detach().cpu().numpy(), O.forward(v.double().cpu().numpy(),
                               np.zeros(128)), rtol=1e-5, atol=1e-6)


def test_bf16_step_runs_the_fused_kernels():
    """A bf16 training step of the fused model agrees with the framework model
    within bf16 noise, and its AttnRes gradients are finite."""
    idx, tgt = _batch()
    losses = {}
    for residual in ("attnres", "switchyard"):
        m = _build(residual, "arena", dtype=torch.bfloat16)
        with torch.no_grad():
            for site in m.attn_res:
                site.w.normal_(0.0, 0.05)
        _, loss = m(idx, tgt)
        loss.backward()
        losses[residual] = loss.item()
        assert all(torch.isfinite(p.grad).all() for p in m.parameters() if p.grad is not None)
    assert abs(losses["switchyard"] - losses["attnres"]) < 2e-2 * abs(losses["attnres"])
