"""Shared test setup.

* registers the ``gpu`` marker (tests that need a CUDA device; the CPU suite
  runs with ``-m "not gpu"``);
* puts the package directory (``blackwell-switchyard_b200/``, not importable by
  name because of the hyphen) and the repository root on ``sys.path``;
* builds the native library and the PyTorch C++ extension in-tree if they are
  missing or stale (nvcc cross-compiles for sm_100a without a GPU), so both
  suites load the real ``libswitchyard_b200.so`` and ``_sy_torch.so``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "blackwell-switchyard_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")
    sys.path.insert(0, str(PKG / "csrc"))
    import build as _build  # noqa: PLC0415

    if not _build.up_to_date():
        # On a GPU box the library arrives prebuilt; rebuilding there would
        # only happen if a source is newer than it, which nvcc handles too.
        _build.build()
    if not _build.ext_up_to_date():
        _build.build_ext()  # the PyTorch C++ extension, linked to the library


def golden_cases() -> list[str]:
    return sorted(p.stem[len("golden_"):] for p in GOLDEN.glob("golden_*.npz"))


def load_golden(name: str):
    """Fixture arrays plus the regenerated (and checksum-verified) inputs."""
    from inputs import case_inputs  # noqa: PLC0415

    from oracle.attnres_oracle import round_to  # noqa: PLC0415

    z = dict(np.load(GOLDEN / f"golden_{name}.npz"))
    n, b, t, d = (int(x) for x in z["meta_shape"])
    dtype = str(z["meta_dtype"])
    v, w, g, q = case_inputs(n, b, t, d, int(z["meta_seed"]), int(z["meta_nq"]))
    w = w * float(z["meta_scale"])
    if dtype != "float64":
        v, w, g, q = (round_to(x, dtype) for x in (v, w, g, q))
    for key, arr in (("check_v", v), ("check_w", w), ("check_g", g), ("check_q", q)):
        if key in z:
            got = np.array([arr.sum(), np.abs(arr).sum()])
            np.testing.assert_allclose(got, z[key], rtol=1e-9, atol=1e-9, err_msg=f"{name} {key}")
    return z, (v, w, g, q)
