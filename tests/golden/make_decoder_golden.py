"""Generate the decoder golden fixture by running the REFERENCE decoder.

Run where a checkout of the reference (sabdulmajid/blackwell-switchyard) is
available, naming its root by argument or by ``SWITCHYARD_REFERENCE``::

    python tests/golden/make_decoder_golden.py <reference checkout>

It imports the reference's own ``src/switchyard/model.py`` (read-only), builds
its ``Transformer`` at a tiny configuration in float32 on the CPU with the
framework residual (``residual="attnres"``, the eager ``folded_form``: the
reference's fused mode needs a GPU and Triton), runs one forward + backward on
a fixed token batch, and writes ``decoder_golden.npz`` next to this file:

* ``meta_*``: the configuration and batch shape;
* ``param:<name>``: every parameter after the reference's seeded
  initialisation (``torch.manual_seed(0)`` before construction), so the test
  loads exactly these weights;
* ``idx``, ``tgt``: the token batch; ``loss``; ``logits``;
* ``grad:<name>``: every parameter's gradient of the loss;
* ``counts``: the source count of every Block AttnRes site
  (``last_source_counts``);
* ``loss_stack``: the same model with ``sources="stack"`` (the reference's
  arena and stack agree bitwise in this mode).

``tests/test_decoder.py`` checks ``switchyard.decoder`` against it on the CPU
(framework mode) and ``tests/test_decoder_gpu.py`` on the GPU (both modes).
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CONFIG = dict(vocab_size=64, d_model=32, n_layers=2, n_heads=2, d_ff=64, n_blocks=2,
              max_seq_len=16)
BATCH = (2, 12)


def reference_root() -> Path:
    where = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SWITCHYARD_REFERENCE")
    if not where:
        raise SystemExit("name the reference checkout: make_decoder_golden.py <path> "
                         "(or set SWITCHYARD_REFERENCE)")
    return Path(where)


def main() -> int:
    root = reference_root() / "src"
    sys.path.insert(0, str(root))
    spec = importlib.util.find_spec("switchyard.model")
    if spec is None or not str(spec.origin).startswith(str(root)):
        raise SystemExit(f"reference not importable from {root}")
    import torch  # noqa: PLC0415
    from switchyard.model import ModelConfig, Transformer  # noqa: PLC0415

    torch.set_num_threads(1)  # a fixed reduction order for the fixture
    out = {}
    for sources in ("arena", "stack"):
        torch.manual_seed(0)
        model = Transformer(ModelConfig(**CONFIG, residual="attnres", sources=sources)).float()
        torch.manual_seed(99)
        b, t = BATCH
        idx = torch.randint(0, CONFIG["vocab_size"], (b, t))
        tgt = torch.randint(0, CONFIG["vocab_size"], (b, t))
        logits, loss = model(idx, tgt)
        loss.backward()
        if sources == "stack":
            out["loss_stack"] = np.array(loss.item())
            continue
        for k, v in CONFIG.items():
            out[f"meta_{k}"] = np.array(v)
        out["idx"], out["tgt"] = idx.numpy(), tgt.numpy()
        out["loss"] = np.array(loss.item(), dtype=np.float64)
        out["logits"] = logits.detach().numpy()
        out["counts"] = np.array(model.last_source_counts)
        for name, p in sorted(model.named_parameters()):
            out[f"param:{name}"] = p.detach().numpy()
            out[f"grad:{name}"] = p.grad.numpy()
    path = HERE / "decoder_golden.npz"
    np.savez_compressed(path, **out)
    print(f"{path.name}: {path.stat().st_size / 1024:.1f} KiB, "
          f"{sum(1 for k in out if k.startswith('param:'))} parameters")
    return 0


if __name__ == "__main__":
    sys.exit(main())
