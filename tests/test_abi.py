"""The C-ABI library on the CPU: it loads, exports every entry point the header
declares, and validates arguments on the host before any CUDA call. No test
here launches a kernel."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def _declared() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        names |= set(re.findall(r"^SY_API\s+[\w\s\*]+?\b(sy_\w+)\s*\(", text, flags=re.M))
    return names


@pytest.fixture(scope="module")
def native():
    from switchyard import _native

    return _native


def test_header_declares_the_entry_points():
    names = _declared()
    for required in ("sy_fwd", "sy_bwd", "sy_bwd_partials", "sy_dw_reduce", "sy_dw_reduce_gain",
                     "sy_fwd_batched", "sy_fwd_batched_stats", "sy_bwd_batched",
                     "sy_bwd_batched_partials", "sy_merge_stats", "sy_stage_partial",
                     "sy_speed_of_light", "sy_stats_stride", "sy_status_string"):
        assert required in names


def test_library_exports_every_declared_symbol(native):
    lib = ctypes.CDLL(str(native.LIB_PATH))
    for name in sorted(_declared()):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in native.SIGNATURES, f"{name} has no ctypes signature in _native"


def test_library_is_built_for_sm100a_only():
    """The build compiles for sm_100a and nothing else (no PTX for JIT)."""
    import build

    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_status_strings(native):
    for code in range(7):
        assert native.lib.sy_status_string(code)
    assert native.lib.sy_version().startswith(b"switchyard-b200")


@pytest.mark.parametrize("n", [1, 2, 3, 9, 16, 33, 64])
def test_stats_stride(native, n):
    assert native.stats_stride(n) == (2 * n + 2 + 3) // 4 * 4
    assert native.stats_stride(n) % 4 == 0  # 16-byte rows for the bulk copy


def test_host_validation_rejects_bad_arguments(native):
    L = native.lib
    bf16, bad = native.SY_BF16, 7
    # unknown dtype codes
    assert L.sy_fwd(1, 1, 1, None, 2, 4, 8, bad, bf16, 1e-6, None) == native.SY_ERR_DTYPE
    assert L.sy_fwd(1, 1, 1, None, 2, 4, 8, bf16, bad, 1e-6, None) == native.SY_ERR_DTYPE
    assert L.sy_fwd_batched(1, 1, 1, 2, 4, 8, 2, bad, 1e-6, None) == native.SY_ERR_DTYPE
    # bad sizes and null pointers
    assert L.sy_fwd(1, 1, 1, None, 0, 4, 8, bf16, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd(None, 1, 1, None, 2, 4, 8, bf16, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd(1, 1, 1, None, 2, -1, 8, bf16, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd_batched(1, 1, 1, 2, 4, 8, 0, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_dw_reduce(None, 0, 8, None, bf16, None) == native.SY_ERR_ARG
    assert L.sy_speed_of_light(None, 1, 2, 4, 8, bf16, None) == native.SY_ERR_ARG
    # empty problems are a successful no-op (no launch, no CUDA call)
    assert L.sy_fwd(None, None, None, None, 2, 0, 8, bf16, bf16, 1e-6, None) == native.SY_OK
    assert L.sy_fwd(None, None, None, None, 2, 4, 0, bf16, bf16, 1e-6, None) == native.SY_OK
    assert L.sy_dw_reduce(None, 1, 0, None, bf16, None) == native.SY_OK
    assert L.sy_bwd_partials(3, 0, 16, bf16) == 1
    assert L.sy_bwd_partials(0, 4, 16, bf16) < 0
    # dw exchange (part, P, L, bases, world, rank, buf_off, tag, dw, dtype, limit, timing,
    # fail, stream): rank outside the world, misaligned offset, bad world size, no
    # partial rows, tag 0, dtype, misaligned timing counters
    def ex(part=1, p=4, length=8, bases=1, world=2, rank=0, off=0, tag=1, dw=1, dtype=bf16,
           timing=None):
        return L.sy_dw_exchange(part, p, length, bases, world, rank, off, tag, dw, dtype, 0,
                                timing, None, None)

    assert ex(rank=2) == native.SY_ERR_ARG
    assert ex(off=4) == native.SY_ERR_ARG
    assert ex(off=-8) == native.SY_ERR_ARG
    assert ex(world=0) == native.SY_ERR_ARG
    assert ex(world=65, rank=0) == native.SY_ERR_ARG
    assert ex(p=0) == native.SY_ERR_ARG
    assert ex(tag=0) == native.SY_ERR_ARG
    assert ex(dtype=bad) == native.SY_ERR_DTYPE
    assert ex(timing=12) == native.SY_ERR_ARG
    assert ex(bases=None) == native.SY_ERR_ARG
    assert ex(part=None, bases=None, dw=None, length=0) == native.SY_OK
    # bytes per rank buffer: two slots of world x L 8-byte words
    assert L.sy_dw_exchange_bytes(2048, 8) == 2 * 8 * 2048 * 8
    assert L.sy_dw_exchange_bytes(33, 2) == 2 * 2 * 33 * 8
    assert L.sy_dw_exchange_bytes(0, 3) == 0
    assert L.sy_dw_exchange_bytes(8, 0) < 0
    # gain-split dw reduction: dtype, null inputs, nothing to write, empty D
    assert L.sy_dw_reduce_gain(1, 4, 8, 1, 1, 1, 1, bad, None) == native.SY_ERR_DTYPE
    assert L.sy_dw_reduce_gain(1, 4, 8, None, 1, 1, 1, bf16, None) == native.SY_ERR_ARG
    assert L.sy_dw_reduce_gain(1, 0, 8, 1, 1, 1, 1, bf16, None) == native.SY_ERR_ARG
    assert L.sy_dw_reduce_gain(1, 4, 8, 1, 1, None, None, bf16, None) == native.SY_OK
    assert L.sy_dw_reduce_gain(None, 4, 0, None, None, 1, 1, bf16, None) == native.SY_OK
    # batched forward with merge statistics: dtype, S, raw flag, null statistics, empty
    assert L.sy_fwd_batched_stats(1, 1, 1, 8, 0, 2, 4, 8, 2, bad, 1e-6, None) == native.SY_ERR_DTYPE
    assert L.sy_fwd_batched_stats(1, 1, 1, 8, 0, 2, 4, 8, 0, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd_batched_stats(1, 1, 1, 8, 2, 2, 4, 8, 2, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd_batched_stats(1, 1, 1, None, 1, 2, 4, 8, 2, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_fwd_batched_stats(None, None, None, None, 0, 2, 0, 8, 2, bf16, 1e-6, None) == native.SY_OK
    # batched backward: partial-row count, dtype, S, empty problems
    assert L.sy_bwd_batched_partials(0, 4, 8, 2, bf16) < 0
    assert L.sy_bwd_batched_partials(3, 0, 8, 2, bf16) == 1
    assert L.sy_bwd_batched(1, 1, 1, 1, 1, 1, 3, 4, 8, 2, bad, 1e-6, None) == native.SY_ERR_DTYPE
    assert L.sy_bwd_batched(1, 1, 1, 1, 1, 1, 3, 4, 8, 0, bf16, 1e-6, None) == native.SY_ERR_ARG
    assert L.sy_bwd_batched(None, None, None, None, None, 1, 3, 0, 0, 2, bf16, 1e-6, None) == native.SY_OK
    # merge: dtype, normalize flag, null inputs, misaligned statistics, no rows
    assert L.sy_merge_stats(8, 8, 8, 8, 8, 8, 0, 4, 8, bad, None) == native.SY_ERR_DTYPE
    assert L.sy_merge_stats(8, 8, 8, 8, 8, 8, 2, 4, 8, bf16, None) == native.SY_ERR_ARG
    assert L.sy_merge_stats(8, None, 8, 8, 8, 8, 0, 4, 8, bf16, None) == native.SY_ERR_ARG
    assert L.sy_merge_stats(8, 4, 8, 8, 8, 8, 0, 4, 8, bf16, None) == native.SY_ERR_ARG
    assert L.sy_merge_stats(None, None, None, None, None, None, 1, 0, 8, bf16, None) == native.SY_OK
    # arena staging: dtype, negative length, null buffers, empty
    assert L.sy_stage_partial(1, 1, 1, 1, 8, bad, None) == native.SY_ERR_DTYPE
    assert L.sy_stage_partial(1, 1, 1, 1, -1, bf16, None) == native.SY_ERR_ARG
    assert L.sy_stage_partial(1, None, 1, 1, 8, bf16, None) == native.SY_ERR_ARG
    assert L.sy_stage_partial(None, None, None, None, 0, bf16, None) == native.SY_OK


B200 = dict(sms=148, max_smem=232448)  # multiprocessors, opt-in shared memory per block


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16", "float32"])
def test_planner_invariants_for_b200(native, dtype_name):
    """Every tile plan fits the device and keeps the pipeline's invariants:
    at least two stages, groups within the 256 consumer threads, the
    shared-memory tile's stage count a multiple of its group count (its
    parity protocol needs it), and the representative shape on the
    register-tile kernels. Pure host logic: no GPU needed."""
    import torch

    dt = getattr(torch, dtype_name)
    for n in (1, 2, 3, 5, 8, 9, 10, 16, 17, 33, 64):
        for d in (64, 320, 512, 1024, 1536, 2048, 4096, 8192):
            for op in (0, 1):
                p = native.plan_info(op, n, 4096, d, 1, dt, **B200)
                if p["kind"] == 0:
                    continue
                assert p["smem_bytes"] <= B200["max_smem"]
                assert p["stages"] >= 2 and p["groups"] >= 1
                assert p["grid"] == 148
                if p["kind"] == 3:
                    continue_checks = False
                else:
                    continue_checks = True
                if continue_checks:
                    # register-tile CTAs have up to 512 threads, shared-memory tile ones 256
                    assert p["groups"] * p["threads_per_group"] <= (512 if p["kind"] == 1 else 256)
                    assert p["threads_per_group"] % 32 == 0
                    assert p["chunks_per_thread"] * p["threads_per_group"] * 16 >= d * dt.itemsize
                if p["kind"] == 2:
                    assert p["stages"] % p["groups"] == 0
                    assert n <= 64
                if p["kind"] == 1:
                    assert n <= 16
                if p["kind"] == 3 and op == 0:  # row-stream forward: a token per 1, 2, 4 or 8 warps
                    assert p["threads_per_group"] in (32, 64, 128, 256)
                    assert p["chunks_per_thread"] * p["threads_per_group"] * 16 >= d * dt.itemsize
                    assert p["groups"] * p["threads_per_group"] <= 512 and p["stages"] >= 2
                if p["kind"] == 3 and op == 1:  # row-stream backward: 4 chunks per lane, exact
                    kw = p["threads_per_group"] // 32
                    assert 1 <= kw <= 16 and n <= 64
                    assert p["chunks_per_thread"] * p["threads_per_group"] * 16 == d * dt.itemsize
                    assert p["groups"] * p["threads_per_group"] <= 512 and p["stages"] >= 2
                    if kw > 1:
                        assert p["groups"] <= 15  # named barrier ids 1..15
    # representative forward: re-read row stream, 14 warps x 2 whole tokens each
    # (28 tokens per SM), at least 3 row buffers per warp
    rep = native.plan_info(0, 9, 4096, 2048, 1, torch.bfloat16, **B200)
    assert rep["kind"] == 3 and rep["groups"] == 14 and rep["stages"] >= 3
    assert rep["grid"] * rep["groups"] * 2 >= 4096
    assert native.plan_info(0, 17, 4096, 2048, 1, torch.bfloat16, **B200)["kind"] == 3
    assert native.plan_info(0, 9, 4096, 512, 1, torch.bfloat16, **B200)["kind"] == 1
    # 2 KiB rows: the re-read row stream with 4 chunks per lane
    p = native.plan_info(0, 9, 4096, 1024, 1, torch.bfloat16, **B200)
    assert p["kind"] == 3 and p["chunks_per_thread"] == 4 and p["threads_per_group"] == 32
    # 8, 16 and 32 KiB rows: the split row stream, 2, 4 and 8 warps per token
    for d, kw in ((4096, 2), (8192, 4), (16384, 8)):
        p = native.plan_info(0, 9, 4096, d, 1, torch.bfloat16, **B200)
        assert p["kind"] == 3 and p["threads_per_group"] == 32 * kw and p["stages"] >= 3
    assert native.plan_info(1, 9, 4096, 2048, 1, torch.bfloat16, **B200)["kind"] == 1
    # backward rows the register tile cannot hold: the row stream, K = rows / 2 KiB
    # (chunks per lane, warps per token): the most chunks per lane (4, 2, 1)
    # that divide the row, then K = row chunks / (32 x chunks per lane)
    for n, d, cpl, kw in ((9, 8192, 4, 8), (17, 4096, 4, 4), (17, 2048, 4, 2), (33, 2048, 4, 2),
                          (64, 4096, 4, 4), (33, 8192, 4, 8), (17, 1024, 4, 1), (33, 1024, 4, 1),
                          (64, 1024, 4, 1), (17, 1536, 2, 3), (20, 1280, 1, 5)):
        p = native.plan_info(1, n, 4096, d, 1, torch.bfloat16, **B200)
        assert p["kind"] == 3 and p["stages"] >= 2, (n, d, p)
        assert (p["chunks_per_thread"], p["threads_per_group"] // 32) == (cpl, kw), (n, d, p)
    # the register tile keeps N <= 16 at 2 KiB rows; N = 65 leaves the row stream
    assert native.plan_info(1, 9, 4096, 1024, 1, torch.bfloat16, **B200)["kind"] == 1
    assert native.plan_info(1, 65, 4096, 2048, 1, torch.bfloat16, **B200)["kind"] != 3
    # batched queries beyond the register tile: the row-stream batched kernel,
    # K warps per token, as many chunks per lane as the queries' registers allow
    for n, d, s, kw, cpl in ((17, 4096, 8, 8, 2), (20, 2048, 16, 8, 1), (32, 1024, 2, 2, 2),
                             (17, 4096, 3, 8, 2)):
        p = native.plan_info(2, n, 4096, d, s, torch.bfloat16, **B200)
        assert p["kind"] == 3 and p["threads_per_group"] == 32 * kw
        assert p["chunks_per_thread"] == cpl
        assert p["groups"] * p["threads_per_group"] <= 512 and p["stages"] >= 2
        assert p["smem_bytes"] <= B200["max_smem"]
    # rows that are not a multiple of 16 bytes go to the generic kernels
    assert native.plan_info(0, 3, 64, 777, 1, torch.bfloat16, **B200)["kind"] == 0


def test_torch_extension_loads_over_the_same_library():
    """The PyTorch C++ extension (_sy_torch) that the autograd functions call
    imports on the CPU, exposes its entry points, and uses the same in-tree
    C-ABI library as the ctypes binding (one copy mapped, not two)."""
    import torch  # noqa: F401  (the extension links against torch)
    from switchyard import _native, _sy_torch

    for name in ("forward", "backward_partials", "backward", "backward_gain", "version"):
        assert hasattr(_sy_torch, name), name
    assert _sy_torch.version() == _native.version()
    maps = open("/proc/self/maps").read()
    mapped = {line.split()[-1] for line in maps.splitlines() if "libswitchyard_b200.so" in line}
    assert mapped == {str(_native.LIB_PATH.resolve())}, mapped


def test_batched_planner_sizes_query_slots(native):
    """The register-tile batched forward is compiled for 4, 8 or 16 query slots
    (S rounded up, the extra slots zero rows): its plan depends only on the
    slot count, every plan fits the opt-in shared memory with at least a stage
    per group, and the slot rows take shared memory from the ring."""
    import torch

    plans = {s: native.plan_info(2, 9, 4096, 2048, s, torch.bfloat16, **B200)
             for s in (2, 3, 4, 5, 8, 9, 12, 16)}
    for a, b in ((2, 4), (3, 4), (5, 8), (9, 16), (12, 16)):
        assert plans[a] == plans[b], (a, b)
    for p in plans.values():
        assert p["kind"] == 1 and p["stages"] >= p["groups"]
        assert p["smem_bytes"] <= B200["max_smem"]
    assert plans[4]["smem_bytes"] < plans[8]["smem_bytes"]
    assert plans[16]["stages"] < plans[8]["stages"]
