"""The decoder restatement (``switchyard.decoder``) against the reference's own
decoder, on the CPU.

``tests/golden/decoder_golden.npz`` was written by running the reference's
``src/switchyard/model.py`` (``tests/golden/make_decoder_golden.py``): a tiny
configuration in float32 with the framework residual (``"attnres"``), its
weights, a token batch, the loss, the logits and every parameter's gradient.
Here the same weights are loaded into ``switchyard.decoder.Decoder`` and the
framework mode (autograd ops only, so it runs on the CPU) must reproduce the
reference bitwise -- loss, logits and every gradient -- since it performs the
same torch operations in the same order (one CPU thread, as the fixture was
made). The fused mode is checked against the same fixture on the GPU
(``tests/test_decoder_gpu.py``).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden" / "decoder_golden.npz"


def _fixture():
    return dict(np.load(GOLDEN))


def _config(z, **kw):
    from switchyard.decoder import DecoderConfig

    keys = ("vocab_size", "d_model", "n_layers", "n_heads", "d_ff", "n_blocks", "max_seq_len")
    return DecoderConfig(**{k: int(z[f"meta_{k}"]) for k in keys}, **kw)


def load_golden_decoder(residual: str, sources: str, device="cpu"):
    """The fixture's model (weights loaded by name) and batch."""
    from switchyard.decoder import Decoder

    z = _fixture()
    model = Decoder(_config(z, residual=residual, sources=sources))
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name, p in params.items():
            p.copy_(torch.from_numpy(z[f"param:{name}"]))
    names = sorted(k[len("param:"):] for k in z if k.startswith("param:"))
    assert names == sorted(params), "parameter names differ from the reference's"
    model = model.to(device)
    idx = torch.from_numpy(z["idx"]).to(device)
    tgt = torch.from_numpy(z["tgt"]).to(device)
    return model, idx, tgt, z


def flat_grads(model) -> torch.Tensor:
    return torch.cat([p.grad.flatten() for _, p in sorted(model.named_parameters())])


@pytest.mark.parametrize("sources", ["arena", "stack"])
def test_framework_mode_reproduces_the_reference_decoder(sources):
    torch.set_num_threads(1)
    model, idx, tgt, z = load_golden_decoder("attnres", sources)
    logits, loss = model(idx, tgt)
    loss.backward()
    assert model.last_source_counts == z["counts"].tolist()
    assert loss.item() == float(z["loss"])
    np.testing.assert_array_equal(logits.detach().numpy(), z["logits"])
    for name, p in sorted(model.named_parameters()):
        np.testing.assert_array_equal(p.grad.numpy(), z[f"grad:{name}"], err_msg=name)
    if sources == "stack":
        assert loss.item() == float(z["loss_stack"])


def test_source_schedule_and_slab_counts():
    """The paper's Eq. 6 schedule and the arena's slab arithmetic, as the
    reference states them (model.py:205-235, tests/test_model.py:55-67)."""
    from switchyard.decoder import slab_copies, source_count_schedule

    assert source_count_schedule(12, 3) == [1, 2, 2, 2, 2, 3, 3, 3, 3, 4, 4, 4, 4]
    sched = source_count_schedule(48, 8)
    assert sched[:7] == [1, 2, 2, 2, 2, 2, 2] and sched[-1] == 9 and len(sched) == 49
    assert slab_copies(48, 8, "arena") == 49
    assert slab_copies(48, 8, "stack") == sum(sched) == 265


def test_parameter_counts_match_the_paper():
    """One pseudo-query and one gain of D per site (2 * n_layers + 1 sites),
    nothing else; the fused and framework modes have the same parameters."""
    from switchyard.decoder import Decoder

    z = _fixture()
    counts = {r: sum(p.numel() for p in Decoder(_config(z, residual=r)).parameters())
              for r in ("standard", "attnres", "switchyard")}
    d, nl = int(z["meta_d_model"]), int(z["meta_n_layers"])
    assert counts["attnres"] == counts["switchyard"]
    assert counts["attnres"] - counts["standard"] == 2 * d * (2 * nl + 1)


def test_the_1_3b_configuration():
    """The 1.3 B benchmark model: 24 layers, hidden 2048, 16 heads, SwiGLU 5632, 8
    blocks, vocabulary 32000 -- about 1.3 B parameters with tied embeddings."""
    from switchyard.decoder import Decoder, DecoderConfig

    cfg = DecoderConfig()
    assert (cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.d_ff, cfg.n_blocks, cfg.vocab_size) == (
        24, 2048, 16, 5632, 8, 32000)
    with torch.device("meta"):
        model = Decoder(cfg)
    n = sum(p.numel() for p in model.parameters())
    assert 1.2e9 < n < 1.4e9, n


def test_configuration_is_validated():
    from switchyard.decoder import DecoderConfig

    with pytest.raises(ValueError, match="residual"):
        DecoderConfig(residual="bogus")
    with pytest.raises(ValueError, match="sources"):
        DecoderConfig(sources="bogus")
    with pytest.raises(ValueError, match="n_blocks"):
        DecoderConfig(n_layers=3, n_blocks=4)
