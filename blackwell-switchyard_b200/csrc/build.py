"""Build libswitchyard_b200.so (the C-ABI library) in-tree with nvcc.

Every ``.cu`` file in this directory is compiled for sm_100a only, as
relocatable device code (the device error word is shared across files), in
parallel, then device-linked into one shared library that lands next to the
Python package that loads it. The library links the *shared* CUDA runtime, so
in a process that already imported torch it uses torch's runtime and sees the
same current device.

Then the thin PyTorch C++ extension over that C ABI (``torch_ext/``) is
compiled with g++ against torch's headers into ``switchyard/_sy_torch.so``.

Usage: ``python build.py [--force] [--jobs N]``. Rebuilds only when the
content of a source, header or of this script changed since the last build (a
hash stamp beside each library; file times are unreliable after copies).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent / "switchyard"
LIB = PKG / "libswitchyard_b200.so"
STAMP = PKG / "libswitchyard_b200.stamp"
INCLUDE = HERE.parent.parent / "include"
BUILD = HERE.parent / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the switchyard CUDA library cannot be built")


def _sources() -> list[Path]:
    return sorted(HERE.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(HERE.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__)]


def _digest() -> str:
    h = hashlib.sha256()
    for p in _deps():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def up_to_date() -> bool:
    return LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == _digest()


def _run(cmd: list[str]) -> tuple[list[str], int, str]:
    r = subprocess.run(cmd, capture_output=True, text=True)
    return cmd, r.returncode, r.stdout + r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          defines: tuple[str, ...] = (), out: Path | None = None) -> Path:
    """Build the library. ``defines`` (``NAME=VALUE``) and ``out`` build a
    variant elsewhere (tuning experiments) without touching the in-tree one."""
    lib = Path(out) if out is not None else LIB
    if not force and not defines and out is None and up_to_date():
        return LIB
    nvcc = _nvcc()
    bdir = BUILD if out is None else lib.parent / (lib.stem + "_obj")
    bdir.mkdir(parents=True, exist_ok=True)
    dflags = [f"-D{d}" for d in defines]
    objs = []
    cmds = []
    for src in _sources():
        obj = bdir / (src.stem + ".o")
        objs.append(obj)
        cmds.append([nvcc, *ARCH, *FLAGS, *dflags, "-Xptxas", "-v", "-dc", str(src), "-o", str(obj)])
    jobs = jobs or min(len(cmds), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for cmd, rc, log in ex.map(_run, cmds):
            if verbose:
                print(log)
            if rc != 0:
                raise RuntimeError(f"nvcc failed ({rc}): {' '.join(cmd)}\n{log}")
            (bdir / (Path(cmd[-3]).stem + ".ptxas.txt")).write_text(log)
    tmp = lib.with_suffix(".so.tmp")
    link = [nvcc, *ARCH, "-rdc=true", "-shared", "-cudart", "shared", *map(str, objs), "-o", str(tmp)]
    cmd, rc, log = _run(link)
    if rc != 0:
        raise RuntimeError(f"link failed ({rc}): {' '.join(cmd)}\n{log}")
    os.replace(tmp, lib)
    if out is None and not defines:
        STAMP.write_text(_digest() + "\n")
    return lib


# ---------------------------------------------------------------------------
# the PyTorch C++ extension over the C ABI (switchyard/_sy_torch*.so)
# ---------------------------------------------------------------------------

EXT_SRC = HERE / "torch_ext" / "sy_torch.cpp"
EXT = PKG / "_sy_torch.so"
EXT_STAMP = PKG / "_sy_torch.stamp"


def _ext_cmd() -> list[str]:
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    inc += [f"-I{sysconfig.get_paths()['include']}", f"-I{INCLUDE}"]
    cuda_home = cpp_extension.CUDA_HOME or "/usr/local/cuda"
    inc.append(f"-I{Path(cuda_home) / 'include'}")
    libs = [f"-L{p}" for p in cpp_extension.library_paths()]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            "-DTORCH_EXTENSION_NAME=_sy_torch", *inc, str(EXT_SRC), *libs,
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            f"-L{PKG}", "-l:libswitchyard_b200.so", "-Wl,-rpath,$ORIGIN"]


def _ext_digest() -> str:
    import torch

    h = hashlib.sha256()
    for p in [EXT_SRC, *sorted(INCLUDE.glob("*.h")), Path(__file__)]:
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(torch.__version__.encode())
    return h.hexdigest()


def ext_up_to_date() -> bool:
    return EXT.exists() and EXT_STAMP.exists() and EXT_STAMP.read_text().strip() == _ext_digest()


def build_ext(force: bool = False) -> Path:
    """Compile the extension (g++ against torch's headers, linked to the C-ABI
    library beside it). Rebuilds only when its source, the header or torch
    changed."""
    if not force and ext_up_to_date():
        return EXT
    tmp = EXT.with_suffix(".so.tmp")
    cmd = _ext_cmd()
    cmd[cmd.index(str(EXT_SRC)) + 1:cmd.index(str(EXT_SRC)) + 1] = ["-o", str(tmp)]
    _, rc, log = _run(cmd)
    if rc != 0:
        raise RuntimeError(f"extension build failed ({rc}): {' '.join(cmd)}\n{log}")
    os.replace(tmp, EXT)
    EXT_STAMP.write_text(_ext_digest() + "\n")
    return EXT


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose))
    print(build_ext(force=a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
