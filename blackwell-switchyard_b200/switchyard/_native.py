"""ctypes binding of ``libswitchyard_b200.so`` (the C ABI in ``include/switchyard_b200.h``).

This module is the only place Python touches the native library. It maps
torch tensors to raw device pointers, the current CUDA stream and the ABI's
dtype codes, and turns nonzero status codes into Python exceptions.

There is no fallback: if the library is missing or cannot be loaded, importing
this module raises ``ImportError`` with the command that builds it.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libswitchyard_b200.so"
LIB_PATH = Path(os.environ.get("SWITCHYARD_B200_LIB", Path(__file__).resolve().parent / LIB_NAME))

SY_BF16, SY_F16, SY_F32 = 0, 1, 2
SY_OK, SY_ERR_ARG, SY_ERR_DTYPE, SY_ERR_UNSUPPORTED, SY_ERR_CUDA, SY_ERR_DEVICE = range(6)
SY_ERR_SCRATCH = 6

DTYPE_CODES = {torch.bfloat16: SY_BF16, torch.float16: SY_F16, torch.float32: SY_F32}

# Every symbol the header declares, with its ctypes signature.
_c = ctypes
_P, _I64, _I, _F = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_float
SIGNATURES: dict[str, tuple[list, object]] = {
    "sy_status_string": ([_I], _c.c_char_p),
    "sy_version": ([], _c.c_char_p),
    "sy_stats_stride": ([_I64], _I64),
    "sy_fwd": ([_P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _F, _P], _I),
    "sy_bwd_partials": ([_I64, _I64, _I64, _I], _I64),
    "sy_bwd": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _F, _P], _I),
    "sy_dw_reduce": ([_P, _I64, _I64, _P, _I, _P], _I),
    "sy_dw_reduce_gain": ([_P, _I64, _I64, _P, _P, _P, _P, _I, _P], _I),
    "sy_fwd_batched": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I, _F, _P], _I),
    "sy_fwd_batched_stats": ([_P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I, _F, _P], _I),
    "sy_bwd_batched_partials": ([_I64, _I64, _I64, _I64, _I], _I64),
    "sy_bwd_batched": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I, _F, _P], _I),
    "sy_merge_stats": ([_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I, _P], _I),
    "sy_stage_partial": ([_P, _P, _P, _P, _I64, _I, _P], _I),
    "sy_speed_of_light": ([_P, _P, _I64, _I64, _I64, _I, _P], _I),
    "sy_plan_kind": ([_I, _I64, _I64, _I64, _I64, _I], _I),
    "sy_plan_info": ([_I, _I64, _I64, _I64, _I64, _I, _I, _I, _c.POINTER(_I64)], _I),
    "sy_device_error": ([_c.POINTER(_c.c_int)], _I),
    "sy_bwd_noalloc": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _F, _P], _I),
    "sy_bwd_noalloc_max_floats": ([], _I64),
    "sy_dw_exchange": ([_P, _I64, _I64, _P, _I, _I, _I64, _c.c_uint32, _P, _I,
                        _c.c_uint64, _P, _P, _P], _I),
    "sy_dw_exchange_bytes": ([_I64, _I], _I64),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"switchyard: native library {LIB_PATH} is missing; build it with "
            "`python blackwell-switchyard_b200/csrc/build.py` (or __graft_entry__.build())"
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:  # pragma: no cover - exercised only on a broken install
        raise ImportError(f"switchyard: cannot load {LIB_PATH}: {exc}") from exc
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    return lib


lib = _load()


class NativeError(RuntimeError):
    """A nonzero status from the native library."""

    def __init__(self, what: str, status: int):
        msg = lib.sy_status_string(status).decode()
        super().__init__(f"switchyard: {what} failed (status {status}): {msg}")
        self.status = status


def check(status: int, what: str) -> None:
    if status != SY_OK:
        raise NativeError(what, status)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(
            f"switchyard kernels take bfloat16, float16 or float32 tensors, got {dtype}"
        ) from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def stats_stride(n: int) -> int:
    return int(lib.sy_stats_stride(n))


def version() -> str:
    return lib.sy_version().decode()


def fwd(v, w, out, stats, n, bt, d, eps) -> None:
    check(
        lib.sy_fwd(
            v.data_ptr(), w.data_ptr(), out.data_ptr(),
            stats.data_ptr() if stats is not None else None,
            n, bt, d, dtype_code(v.dtype), dtype_code(w.dtype), float(eps), stream_of(v),
        ),
        "sy_fwd",
    )


def bwd_partials(n, bt, d, dtype) -> int:
    p = int(lib.sy_bwd_partials(n, bt, d, dtype_code(dtype)))
    if p < 1:
        raise NativeError("sy_bwd_partials", -p)
    return p


def bwd(v, w, g, stats, dv, dw_partial, n, bt, d, eps) -> None:
    check(
        lib.sy_bwd(
            v.data_ptr(), w.data_ptr(), g.data_ptr(), stats.data_ptr(), dv.data_ptr(),
            dw_partial.data_ptr(), dw_partial.shape[0], n, bt, d,
            dtype_code(v.dtype), dtype_code(w.dtype), float(eps), stream_of(v),
        ),
        "sy_bwd",
    )


def dw_reduce(dw_partial, dw) -> None:
    p, d = dw_partial.shape
    check(
        lib.sy_dw_reduce(dw_partial.data_ptr(), p, d, dw.data_ptr(), dtype_code(dw.dtype),
                         stream_of(dw)),
        "sy_dw_reduce",
    )


def dw_reduce_gain(dw_partial, w, g, dw, dg) -> None:
    """dq = sum of the partial rows, then dw = dq * g and dg = dq * w (either
    output may be None)."""
    p, d = dw_partial.shape
    check(
        lib.sy_dw_reduce_gain(dw_partial.data_ptr(), p, d, w.data_ptr(), g.data_ptr(),
                              dw.data_ptr() if dw is not None else None,
                              dg.data_ptr() if dg is not None else None,
                              dtype_code(w.dtype), stream_of(w)),
        "sy_dw_reduce_gain",
    )


def fwd_batched(v, q, out, n, bt, d, s, eps) -> None:
    check(
        lib.sy_fwd_batched(v.data_ptr(), q.data_ptr(), out.data_ptr(), n, bt, d, s,
                           dtype_code(v.dtype), float(eps), stream_of(v)),
        "sy_fwd_batched",
    )


def fwd_batched_stats(v, q, out, mstats, raw: bool, n, bt, d, s, eps) -> None:
    """Batched forward writing (m, l) per (query, token) into ``mstats``
    ([S, BT, 2] fp32); ``raw`` leaves the output unnormalised."""
    check(
        lib.sy_fwd_batched_stats(v.data_ptr(), q.data_ptr(), out.data_ptr(), mstats.data_ptr(),
                                 1 if raw else 0, n, bt, d, s, dtype_code(v.dtype), float(eps),
                                 stream_of(v)),
        "sy_fwd_batched_stats",
    )


def bwd_batched_partials(n, bt, d, s, dtype) -> int:
    p = int(lib.sy_bwd_batched_partials(n, bt, d, s, dtype_code(dtype)))
    if p < 1:
        raise NativeError("sy_bwd_batched_partials", -p)
    return p


def bwd_batched(v, q, g, dv, dq_partial, n, bt, d, s, eps) -> None:
    check(
        lib.sy_bwd_batched(v.data_ptr(), q.data_ptr(), g.data_ptr(), dv.data_ptr(),
                           dq_partial.data_ptr(), dq_partial.shape[0], n, bt, d, s,
                           dtype_code(v.dtype), float(eps), stream_of(v)),
        "sy_bwd_batched",
    )


def merge_stats(o1, ms1, o2, ms2, o, ms, normalize: bool, rows: int, d: int) -> None:
    check(
        lib.sy_merge_stats(o1.data_ptr(), ms1.data_ptr(), o2.data_ptr(), ms2.data_ptr(),
                           o.data_ptr(), ms.data_ptr() if ms is not None else None,
                           1 if normalize else 0, rows, d, dtype_code(o1.dtype), stream_of(o1)),
        "sy_merge_stats",
    )


def stage_partial(partial, out, new_partial, arena_slot) -> None:
    check(
        lib.sy_stage_partial(partial.data_ptr(), out.data_ptr(),
                             new_partial.data_ptr() if new_partial is not None else None,
                             arena_slot.data_ptr(), partial.numel(), dtype_code(partial.dtype),
                             stream_of(partial)),
        "sy_stage_partial",
    )


def speed_of_light(v, out, n, bt, d) -> None:
    check(
        lib.sy_speed_of_light(v.data_ptr(), out.data_ptr(), n, bt, d, dtype_code(v.dtype),
                              stream_of(v)),
        "sy_speed_of_light",
    )


def plan_kind(op: int, n: int, bt: int, d: int, s: int, dtype: torch.dtype) -> int:
    return int(lib.sy_plan_kind(op, n, bt, d, s, dtype_code(dtype)))


PLAN_FIELDS = ("kind", "grid", "stages", "groups", "threads_per_group", "chunks_per_thread",
               "stage_bytes", "smem_bytes")


def plan_info(op: int, n: int, bt: int, d: int, s: int, dtype: torch.dtype, sms: int = 0,
              max_smem: int = 0) -> dict:
    """The launch plan for a shape (on the current device unless sms/max_smem given)."""
    out = (_I64 * 8)()
    check(lib.sy_plan_info(op, n, bt, d, s, dtype_code(dtype), sms, max_smem, out), "sy_plan_info")
    return dict(zip(PLAN_FIELDS, (int(x) for x in out)))


def device_error() -> int:
    code = ctypes.c_int(0)
    check(lib.sy_device_error(ctypes.byref(code)), "sy_device_error")
    return code.value


def dw_exchange_bytes(length: int, world: int) -> int:
    n = int(lib.sy_dw_exchange_bytes(length, world))
    if n < 0:
        raise NativeError("sy_dw_exchange_bytes", -n)
    return n


def dw_exchange(part, peer_bases, world: int, rank: int, buf_off: int, tag: int, dw,
                wait_limit_ns: int = 0, timing=None, fail_word=None) -> None:
    """Sum this rank's fp32 partial rows ``part`` [P, L] and every rank's rows
    in rank order into ``dw`` [L] (sy_dw_exchange); ``peer_bases`` is a CUDA
    int64 tensor of the ranks' buffer addresses, ``timing`` an optional CUDA
    int64 tensor of 8 counters, ``fail_word`` an optional device-visible int32
    tensor (pinned host memory) that receives the tag of a call whose wait ran
    out."""
    p, length = part.shape
    check(
        lib.sy_dw_exchange(part.data_ptr(), p, length, peer_bases.data_ptr(), world, rank,
                           buf_off, tag & 0xFFFFFFFF, dw.data_ptr(), dtype_code(dw.dtype),
                           int(wait_limit_ns),
                           timing.data_ptr() if timing is not None else None,
                           fail_word.data_ptr() if fail_word is not None else None,
                           stream_of(dw)),
        "sy_dw_exchange",
    )
