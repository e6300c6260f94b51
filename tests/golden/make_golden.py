"""Generate the golden fixtures by running the REFERENCE implementation.

Run where a checkout of the reference (sabdulmajid/blackwell-switchyard) is
available, naming its root by argument or by ``SWITCHYARD_REFERENCE``::

    python tests/golden/make_golden.py <reference checkout>

It imports the reference's own ``src/switchyard/reference.py`` and
``baselines.py`` (read-only), evaluates them in float64 on the deterministic
inputs of ``inputs.py`` and writes ``golden_<case>.npz`` next to this file.
Inputs are not stored: tests regenerate them from the seed and check the
stored checksums. The fixtures pin ``oracle/attnres_oracle.py``
(``tests/test_oracle.py``) and are compared with the GPU kernels directly
(``tests/test_parity_gpu.py``).

Each fixture holds: ``out`` (reference forward), ``dv``/``dw`` (autograd of
the reference forward against upstream gradient ``g``), the statistics
``logits``/``r``/``m``/``lse``, an ``attn_with_stats`` split and its
``merge_online_softmax``, ``batched`` (``batched_folded_form``) when the case
has queries, and the reference byte/flop models. Large arrays are stored with
a stride on the last axis (``sub``) to keep the fixtures small.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from inputs import case_inputs  # noqa: E402

# name: (N, B, T, D, seed, input dtype, n_queries, w scale, last-axis subsample)
CASES = {
    "s_5_2_7_16": (5, 2, 7, 16, 10, "float64", 4, 1.0, 1),
    "s_1_1_1_1": (1, 1, 1, 1, 11, "float64", 1, 1.0, 1),
    "s_2_1_1_3": (2, 1, 1, 3, 12, "float64", 2, 1.0, 1),
    "s_17_1_2_63": (17, 1, 2, 63, 13, "float64", 3, 1.0, 1),
    "s_3_4_5_129": (3, 4, 5, 129, 14, "float64", 2, 1.0, 1),
    "s_6_1_3_24_x200": (6, 1, 3, 24, 15, "float64", 0, 200.0, 1),
    "b_9_1_4_2048": (9, 1, 4, 2048, 20, "bfloat16", 8, 1.0, 8),
    "b_4_2_8_512": (4, 2, 8, 512, 21, "bfloat16", 4, 1.0, 4),
    "b_3_1_5_777": (3, 1, 5, 777, 22, "bfloat16", 3, 1.0, 1),
    "b_33_1_3_512": (33, 1, 3, 512, 23, "bfloat16", 0, 1.0, 4),
    "b_17_1_2_4096": (17, 1, 2, 4096, 24, "bfloat16", 8, 1.0, 16),
    "h_5_1_9_320": (5, 1, 9, 320, 25, "float16", 2, 1.0, 2),
    "c1_4_1_256_512": (4, 1, 256, 512, 0, "float32", 0, 1.0, 1),
}


def reference_root() -> Path:
    """The reference checkout: the first command-line argument, else
    ``SWITCHYARD_REFERENCE``; there is no default location."""
    where = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SWITCHYARD_REFERENCE")
    if not where:
        raise SystemExit("name the reference checkout: make_golden.py <path> "
                         "(or set SWITCHYARD_REFERENCE)")
    return Path(where)


def _load_reference():
    root = reference_root() / "src"
    sys.path.insert(0, str(root))
    spec = importlib.util.find_spec("switchyard.reference")
    if spec is None or not str(spec.origin).startswith(str(root)):
        raise SystemExit(f"reference not importable from {root}")
    import switchyard.baselines as baselines  # noqa: PLC0415
    import switchyard.reference as reference  # noqa: PLC0415

    return reference, baselines


def rounded(x: np.ndarray, dtype: str):
    import torch  # noqa: PLC0415

    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype != "float64":
        t = t.to(getattr(torch, dtype)).to(torch.float64)
    return t


def make_case(reference, baselines, spec) -> dict:
    import torch  # noqa: PLC0415

    n, b, t, d, seed, dtype, nq, scale, sub = spec
    v_np, w_np, g_np, q_np = case_inputs(n, b, t, d, seed, nq)
    w_np = w_np * scale
    v, w, g, q = (rounded(x, dtype) for x in (v_np, w_np, g_np, q_np))
    eps = reference.DEFAULT_EPS

    out = reference.block_attn_res_oracle(v, w, eps)
    vv = v.clone().requires_grad_(True)
    ww = w.clone().requires_grad_(True)
    reference.block_attn_res_reference(vv, ww, eps).backward(g)
    logits = torch.einsum("d,nbtd->nbt", w, reference.rms_norm(v, eps))
    r = torch.rsqrt(v.pow(2).mean(-1) + eps)
    _, m, ell = reference.attn_with_stats(v, w, eps)
    split = max(1, n // 2) if n > 1 else 1
    o1, m1, l1 = reference.attn_with_stats(v[:split], w, eps)
    res = {
        "meta_shape": np.array([n, b, t, d]),
        "meta_seed": np.array(seed),
        "meta_dtype": np.array(dtype),
        "meta_scale": np.array(scale),
        "meta_nq": np.array(nq),
        "meta_sub": np.array(sub),
        "meta_eps": np.array(eps),
        "check_v": np.array([float(v.sum()), float(v.abs().sum())]),
        "check_w": np.array([float(w.sum()), float(w.abs().sum())]),
        "check_g": np.array([float(g.sum()), float(g.abs().sum())]),
        "out": out.numpy()[..., ::sub],
        "dv": vv.grad.numpy()[..., ::sub],
        "dw": ww.grad.numpy(),
        "logits": logits.numpy(),
        "r": r.numpy(),
        "m": m.numpy(),
        "lse": (m + ell.log()).numpy(),
        "split": np.array(split),
        "aws1_o": o1.numpy()[..., ::sub],
        "aws1_m": m1.numpy(),
        "aws1_l": l1.numpy(),
        "min_bytes_bf16": np.array(reference.attn_res_min_bytes(n, b, t, d, 2)),
        "flops": np.array(reference.attn_res_flops(n, b, t, d)),
    }
    if split < n:
        o2, m2, l2 = reference.attn_with_stats(v[split:], w, eps)
        om, mm, lm = reference.merge_online_softmax(o1, m1, l1, o2, m2, l2)
        res["merged"] = (om / lm.unsqueeze(-1)).numpy()[..., ::sub]
    if nq > 0:
        res["batched"] = baselines.batched_folded_form(v, q, eps).numpy()[..., ::sub]
        res["check_q"] = np.array([float(q.sum()), float(q.abs().sum())])
    if n * b * t * d <= 65536:
        res["folded"] = baselines.folded_form(v, w, eps).numpy()
    if name_is_config1(spec):
        # keep the full forward output; the larger arrays only for 16 tokens
        res["dv"] = vv.grad.numpy()[:, :, :16]
        res["aws1_o"] = res["aws1_o"][:, :16]
        res["merged"] = res["merged"][:, :16]
    return res


def name_is_config1(spec) -> bool:
    return tuple(spec[:4]) == (4, 1, 256, 512)


def main() -> int:
    reference, baselines = _load_reference()
    import torch  # noqa: PLC0415

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, spec in CASES.items():
        res = make_case(reference, baselines, spec)
        path = HERE / f"golden_{name}.npz"
        np.savez_compressed(path, **res)
        print(f"{path.name}: {path.stat().st_size / 1024:.1f} KiB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
