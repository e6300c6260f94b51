"""The reference's PyTorch eager path, restated -- TEST/BENCH INFRASTRUCTURE ONLY.

Used as the timed CPU baseline (``bench.py``'s ``cpu_baseline`` leg and
``bench.py --impl reference``) and nowhere on the product path. The reference
itself cannot travel to the GPU box, so this restates its eager operator with
the same sequence of torch operations, so that its CPU cost is the reference's:

* ``block_attn_res_eager``: ``src/switchyard/reference.py:107-133``
  (materialise ``k = v * rsqrt(mean(v^2) + eps)``, einsum for the logits,
  softmax over the source axis, einsum for the weighted sum of raw ``v``);
  autograd provides the backward, as it does for the reference.
* ``folded_eager``: ``src/switchyard/baselines.py:64-73`` (never materialises
  ``k``), timed beside it.

``tests/test_oracle.py`` checks both against the golden fixtures.
"""

from __future__ import annotations

import torch

DEFAULT_EPS = 1e-6


def block_attn_res_eager(v: torch.Tensor, w: torch.Tensor, eps: float = DEFAULT_EPS):
    k = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps)
    scores = torch.einsum("d,nbtd->nbt", w, k)
    return torch.einsum("nbt,nbtd->btd", scores.softmax(0), v)


def folded_eager(v: torch.Tensor, w: torch.Tensor, eps: float = DEFAULT_EPS):
    scores = torch.einsum("d,nbtd->nbt", w, v) * torch.rsqrt(v.pow(2).mean(-1) + eps)
    return torch.einsum("nbt,nbtd->btd", scores.softmax(0), v)


def fwd_bwd(v: torch.Tensor, w: torch.Tensor, g: torch.Tensor, eps: float = DEFAULT_EPS,
            fn=block_attn_res_eager):
    """One forward + backward through autograd; returns ``(out, dv, dw)``."""
    vv = v.detach().requires_grad_(True)
    ww = w.detach().requires_grad_(True)
    out = fn(vv, ww, eps)
    out.backward(g)
    return out.detach(), vv.grad, ww.grad
