"""Benchmark of the Block AttnRes operator on B200 at its representative shape.

Workload (one "step"): forward + backward of ``block_attn_res_triton`` at
N=9, B=1, T=4096, D=2048 bf16 with v ~ N(0,1), w ~ N(0,1/D), dout ~ N(0,1)
(synthetic; the reference uses no dataset). Before every timed step, outside
that step's CUDA events, L2 (126 MB) is flushed: a 384 MiB buffer is written
(as the reference harness does, bench/harness.py:73-77) and then a separate
256 MiB buffer is read, so the L2 holds only clean, unrelated lines and the
flush's own dirty write-back is not charged to the step. A short spin kernel
then lets the host queue the whole step before it starts, so the events see
device time only.

Printed: ONE JSON line (rank 0). ``value`` = achieved HBM TB/s of the step's
algorithmic bytes, (3N+2)*B*T*D*2 per rank, summed over ranks, divided by the
max-over-ranks mean step time. Extra keys carry the forward-alone latency and
TB/s, the speed-of-light kernel, per-kernel rooflines, batched queries, the
CPU baseline, the end-to-end number through the public API with host buffers,
and the SM clocks sampled (NVML) during the timed region.

``--gpus N`` (under torchrun): each rank runs the same shape on its own token
shard (weak scaling); the step's only exchange is the fp32 dw sum of
``switchyard.sharding``: one kernel (``sy_dw_exchange``) reduces the rank's
partial rows and adds all ranks' rows over NVLink peer loads in rank order, no
NCCL on the step. Each timed step starts after a device-side barrier across the
ranks' streams, so no rank's events hold another rank's flush or host jitter;
the line also carries each rank's mean, the exchange kernel timed alone, and
the exchange's own flag-wait time read from device counters.

``--sweep``: forward, backward and step times for bf16, fp16 and fp32 at a few
shapes (one JSON line each; no bench line).

``--impl reference``: the reference's PyTorch eager CPU path (restated in
``oracle/eager_port.py``; the reference itself cannot run on the GPU box),
fwd+bwd of the whole workload on all host threads; rank 0 only.
"""

from __future__ import annotations

import argparse
import faulthandler
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "blackwell-switchyard_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "fwd & fwd+bwd µs and achieved HBM TB/s (% of roofline) at N=9 T=4096 D=2048 bf16"
REP = (9, 1, 4096, 2048)
ITEM = 2  # bf16
FLUSH_BYTES = 384 * 2**20
FALLBACK_HBM_GBS = 6650.0


# ----------------------------------------------------------------------------- setup


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline budget")
    ap.add_argument("--no-extras", action="store_true", help="skip batched/SoL/e2e extras")
    ap.add_argument("--profile", choices=["fwd", "bwd", "step", "sol", "batched8", "batched16",
                                          "batched_bwd8", "merge"],
                    default=None,
                    help="no timing: run 5 launches of one kernel (or step) at the representative "
                         "shape, for an ncu capture; prints nothing")
    ap.add_argument("--shape", default=None,
                    help="N,B,T,D for --profile (default: the representative shape)")
    ap.add_argument("--decoder", action="store_true",
                    help="no bench line: the 1.3B Block AttnRes decoder, a bf16 "
                         "AdamW training step of the standard and the switchyard residual at B=4 "
                         "T=2048 per GPU, DDP over NCCL under torchrun; one JSON line")
    ap.add_argument("--decoder-batch", type=int, default=4)
    ap.add_argument("--decoder-seq", type=int, default=2048)
    ap.add_argument("--grid", action="store_true",
                    help="no bench line: the benchmark shape grid N x B x T x D in bf16 with "
                         "the token axis sharded over the torchrun world; fwd and fwd+bwd per shape, "
                         "checked against a float64 evaluation; one JSON line per shape")
    ap.add_argument("--grid-max-shapes", type=int, default=0,
                    help="with --grid: stop after this many shapes (0: all)")
    ap.add_argument("--sweep", action="store_true",
                    help="no bench line: time forward, backward and the fwd+bwd step through the "
                         "C ABI for bf16, fp16 and fp32 at a few shapes, one JSON line each")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def load_peak_field(name: str):
    """A field of MEASURED_PEAKS.json, or None."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        v = json.loads(p.read_text()).get(name)
        return float(v) if v is not None else None
    return None


def alg_bytes(n, b, t, d, itemsize=ITEM):
    fwd = (n + 1) * b * t * d * itemsize
    bwd = (2 * n + 1) * b * t * d * itemsize
    return fwd, bwd, fwd + bwd


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML every few ms."""

    REASONS = {
        "sw_power_cap": 0x4,
        "hw_slowdown": 0x8,
        "sync_boost": 0x10,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.ok = False
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            # NVML wants the "DDDDDDDD:BB:DD.F" string; torch reports integers.
            bus = "{:08X}:{:02X}:{:02X}.0".format(
                int(getattr(props, "pci_domain_id", 0)), int(props.pci_bus_id),
                int(props.pci_device_id)).encode()
            try:
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # noqa: BLE001
            self.err = str(exc)

    def _sample(self):
        nv = self.nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
                nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
            mask = get(self.h)
            for name, bit in self.REASONS.items():
                if mask & bit:
                    self.reasons.add(name)
        except Exception:  # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._sample()  # one at the start, whatever the thread's start-up delay
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": f"nvml unavailable: {self.err}"}
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


# ----------------------------------------------------------------------------- timing


class L2Flush:
    """Write 384 MiB (evicting every line of the 126 MB L2), then read 256 MiB
    of another buffer so the written lines are flushed back to HBM before the
    timed region and L2 holds only clean lines unrelated to the step."""

    def __init__(self, dev):
        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(64 * 2**20, dtype=torch.float32, device=dev)
        self.o = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.o)


def timed_steps(fn, steps, flush, lead_cycles=2_000_000, align=None, on_queued=None):
    """Per-step device times (ms): flush L2, let a spin kernel cover the host's
    queueing of the step, then bracket only the step with CUDA events on the
    current stream. ``align`` (multi-GPU) queues a device-side barrier across
    the ranks' streams after the spin kernel, so every rank's step starts at
    the same moment and no rank's events include another rank's flush or
    host jitter. ``on_queued`` runs once every step is queued, while the GPU
    works through them (the clock sampler takes a sample there)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush()
        torch.cuda._sleep(lead_cycles)
        if align is not None:
            align()
        starts[i].record()
        fn()
        ends[i].record()
    if on_queued is not None:
        on_queued()  # the steps are queued and running: a sample inside the timed region
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def streamed_ms(fn, launches, groups, lead_cycles=4_000_000):
    """Per-launch device time (ms) of back-to-back calls: ``launches`` calls of
    ``fn`` between one pair of CUDA events, after a spin kernel long enough to
    cover the host's queueing of them; the median over ``groups`` such groups.
    No L2 flush between the calls: the inputs (v, 151 MB at the representative
    shape, read evict-first) exceed the 126 MB L2, so every call streams them
    from HBM again, while the GPU's launch handling of one call overlaps the
    previous one -- the kernels' throughput in a stream of calls, as in a
    decoder step, without the per-call event-to-kernel latency that the
    per-step timing carries."""
    per = []
    for _ in range(groups):
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(lead_cycles)
        start.record()
        for _ in range(launches):
            fn()
        end.record()
        torch.cuda.synchronize()
        per.append(start.elapsed_time(end) / launches)
    return sorted(per)[len(per) // 2]


def summarize(ms):
    order = sorted(ms)
    n = len(order)
    med = order[n // 2]
    slow = [i for i, x in enumerate(ms) if x > 1.2 * med]
    return {
        "mean_ms": statistics.fmean(order),
        "median_ms": med,
        "p10_ms": order[max(0, int(0.1 * n))],
        "p90_ms": order[min(n - 1, int(0.9 * n))],
        "min_ms": order[0],
        "max_ms": order[-1],
        # steps more than 20 % above the median, by position in the timed sequence
        "slow_steps": {"count": len(slow), "first_indices": slow[:8]},
    }


# ----------------------------------------------------------------------------- our arm


def make_inputs(dev, rank, n, b, t, d, dtype=torch.bfloat16):
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    v = torch.randn(n, b, t, d, device=dev, generator=g, dtype=torch.float32).to(dtype)
    gw = torch.Generator(device=dev).manual_seed(1)  # the query is shared by all ranks
    w = (torch.randn(d, device=dev, generator=gw) / math.sqrt(d)).to(dtype)
    dout = torch.randn(b, t, d, device=dev, generator=g, dtype=torch.float32).to(dtype)
    return v, w, dout


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_time(n, b, t, d, dtype, seconds, min_reps=3, fwd_only=False):
    """Median seconds of one reference eager CPU call (oracle/eager_port.py,
    the reference's operator sequence): forward + backward through autograd,
    or the forward alone. Synthetic inputs as the bench's."""
    from oracle.eager_port import block_attn_res_eager, fwd_bwd

    gen = torch.Generator().manual_seed(0)
    v = torch.randn(n, b, t, d, generator=gen).to(dtype)
    w = (torch.randn(d, generator=gen) / math.sqrt(d)).to(dtype)
    g = torch.randn(b, t, d, generator=gen).to(dtype)

    def call():
        if fwd_only:
            with torch.no_grad():
                block_attn_res_eager(v, w)
        else:
            fwd_bwd(v, w, g)

    call()
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def cpu_baseline(seconds: float):
    """The reference's eager CPU path (restated in oracle/eager_port.py) on the
    bench's own workload, N=9 B=1 T=4096 D=2048 bf16, forward + backward, on
    all host threads; beside it the same in fp32, the forward alone, and
    the small fp32 case N=4 B=1 T=256 D=512."""
    torch.set_num_threads(os.cpu_count() or 1)
    n, b, t, d = REP
    per, reps = cpu_time(n, b, t, d, torch.bfloat16, seconds)
    fwd_s, _ = cpu_time(n, b, t, d, torch.bfloat16, seconds / 4, fwd_only=True)
    f32, _ = cpu_time(n, b, t, d, torch.float32, seconds / 2)
    c1, _ = cpu_time(4, 1, 256, 512, torch.float32, 2.0)
    _, _, tot = alg_bytes(n, b, t, d)
    return {
        "value": tot / per / 1e12,
        "unit": "TB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"the whole workload: fwd+bwd of the reference eager path (oracle/eager_port.py) at "
                  f"N={n} B={b} T={t} D={d} bf16, median of {reps} runs, {per * 1e3:.1f} ms each",
        "same_config": True,
        "ms_per_step": per * 1e3,
        "fwd_ms": fwd_s * 1e3,
        "fp32_ms_per_step": f32 * 1e3,
        "config1_fp32_ms_per_step": c1 * 1e3,
        "cpu_count": os.cpu_count(),
        "cpu_model": cpu_model(),
    }


def kernel_times(native, v, w, dout, steps, flush, stream):
    """Device time of each of our kernels launched alone through the C ABI."""
    n, b, t, d = v.shape
    bt = b * t
    out = torch.empty(b, t, d, device=v.device, dtype=v.dtype)
    stats = torch.empty(bt, native.stats_stride(n), device=v.device, dtype=torch.float32)
    dv = torch.empty_like(v)
    p = native.bwd_partials(n, bt, d, v.dtype)
    part = torch.empty(p, d, device=v.device, dtype=torch.float32)
    dw = torch.empty(d, device=v.device, dtype=w.dtype)
    sol = torch.empty_like(out)
    res = {}
    calls = {
        "fwd": lambda: native.fwd(v, w, out, stats, n, bt, d, 1e-6),
        "bwd": lambda: native.bwd(v, w, dout, stats, dv, part, n, bt, d, 1e-6),
        "dw_reduce": lambda: native.dw_reduce(part, dw),
        "speed_of_light": lambda: native.speed_of_light(v, sol, n, bt, d),
    }
    calls["fwd"]()
    for name, fn in calls.items():
        for _ in range(3):
            fn()
        res[name] = summarize(timed_steps(fn, steps, flush))
        if name in ("fwd", "bwd"):
            # the same launch 20 times back to back (no flush; see streamed_ms)
            res[name]["back_to_back_ms"] = streamed_ms(fn, 20, 5)
    return res, p


def launch_floor(dev, steps, flush):
    """Device time, by the bench's own method (L2 flush, spin kernel, CUDA
    events around one launch), of this library's smallest kernel: sy_dw_reduce
    over one partial row of 32 columns (one CTA, 32 loads). What any single
    kernel measures at least with this method: the two events plus launching
    and retiring a grid."""
    from switchyard import _native

    part = torch.zeros(1, 32, device=dev, dtype=torch.float32)
    out = torch.empty(32, device=dev, dtype=torch.float32)
    fn = lambda: _native.dw_reduce(part, out)  # noqa: E731
    for _ in range(3):
        fn()
    return summarize(timed_steps(fn, steps, flush))["mean_ms"] * 1e3


def batched_times(v, steps, flush, hbm_gbs, qs=(1, 4, 8, 16)):
    """block_attn_res_batched at Q queries. Roofline: the larger of the HBM time
    (algorithmic bytes at the measured copy bandwidth) and the FP32 time
    ((2+4Q)*N*BT*D FLOP at the device's nominal FP32 FMA rate, SMs x 128 lanes x
    2 FLOP x the maximum SM clock), naming which one binds."""
    from switchyard import block_attn_res_batched

    n, b, t, d = v.shape
    props = torch.cuda.get_device_properties(v.device)
    clock_mhz = load_peak_field("sm_max_mhz") or 1965.0
    fp32_tflops = props.multi_processor_count * 128 * 2 * clock_mhz * 1e6 / 1e12
    out = {}
    gen = torch.Generator(device=v.device).manual_seed(7)
    for q in qs:
        queries = (torch.randn(q, d, device=v.device, generator=gen) / math.sqrt(d)).to(v.dtype)
        with torch.no_grad():
            fn = lambda: block_attn_res_batched(v, queries)  # noqa: E731
            for _ in range(3):
                fn()
            s = summarize(timed_steps(fn, steps, flush))
        byts = ((n + q) * b * t * d + q * d) * ITEM
        flops = (2 + 4 * q) * n * b * t * d
        s["tbps"] = byts / (s["mean_ms"] * 1e-3) / 1e12
        s["bytes"] = byts
        s["flops"] = flops
        t_hbm = byts / (hbm_gbs * 1e9) * 1e3
        t_fp32 = flops / (fp32_tflops * 1e12) * 1e3
        s["roofline"] = {
            "bound": "hbm" if t_hbm >= t_fp32 else "fp32",
            "roofline_ms": max(t_hbm, t_fp32),
            "hbm_ms": t_hbm,
            "fp32_ms": t_fp32,
            "fp32_tflops_nominal": fp32_tflops,
            "frac": max(t_hbm, t_fp32) / s["mean_ms"],
        }
        out[f"Q{q}"] = s
    return out


def batched_train_times(v, steps, flush, hbm_gbs, qs=(1, 4, 8, 16)):
    """The batched training contract at Q queries: the backward alone
    (sy_bwd_batched + the dq reduction, reads v and g, writes dv) and the whole
    autograd step (block_attn_res_batched_train forward + backward), and the
    two-phase schedule (attn_with_stats over the first N // 2 sources and the
    rest, then merge_online_softmax with the division fused). Roofline as in
    batched_times: the larger of the HBM time and the FP32 time, the backward
    doing (5Q + 2) N multiply-adds per token element."""
    from switchyard import _native, attn_with_stats, block_attn_res_batched_train
    from switchyard import merge_online_softmax

    n, b, t, d = v.shape
    bt = b * t
    props = torch.cuda.get_device_properties(v.device)
    clock_mhz = load_peak_field("sm_max_mhz") or 1965.0
    fp32_tflops = props.multi_processor_count * 128 * 2 * clock_mhz * 1e6 / 1e12
    slab = bt * d * ITEM
    out = {}
    gen = torch.Generator(device=v.device).manual_seed(11)
    for q in qs:
        queries = (torch.randn(q, d, device=v.device, generator=gen) / math.sqrt(d)).to(v.dtype)
        g = torch.randn(q, b, t, d, device=v.device, generator=gen).to(v.dtype)
        p_rows = _native.bwd_batched_partials(n, bt, d, q, v.dtype)
        part = torch.empty(p_rows, q * d, device=v.device, dtype=torch.float32)
        dv = torch.empty_like(v)
        dq = torch.empty_like(queries)

        def bwd():
            _native.bwd_batched(v, queries, g, dv, part, n, bt, d, q, 1e-6)
            _native.dw_reduce(part, dq.view(q * d))

        vt = v.detach().requires_grad_(True)
        qt = queries.detach().requires_grad_(True)

        def step():
            vt.grad = None
            qt.grad = None
            block_attn_res_batched_train(vt, qt).backward(g)

        res = {}
        for name, fn, byts in (("bwd", bwd, (2 * n + q) * slab),
                               ("step", step, (3 * n + 2 * q) * slab)):
            for _ in range(3):
                fn()
            st = summarize(timed_steps(fn, steps, flush))
            flops = 2 * (5 * q + 2) * n * bt * d + (2 + 4 * q) * n * bt * d * (name == "step")
            t_hbm = byts / (hbm_gbs * 1e9) * 1e3
            t_fp32 = flops / (fp32_tflops * 1e12) * 1e3
            res[name] = {
                "us": st["mean_ms"] * 1e3,
                "tbps": byts / (st["mean_ms"] * 1e-3) / 1e12,
                "bytes": byts,
                "flops": flops,
                "bound": "hbm" if t_hbm >= t_fp32 else "fp32",
                "frac": max(t_hbm, t_fp32) / st["mean_ms"],
            }
        out[f"Q{q}"] = res
    w = (torch.randn(d, device=v.device, generator=gen) / math.sqrt(d)).to(v.dtype)
    k = n // 2

    def two_phase():
        o1, m1, l1 = attn_with_stats(v[:k], w)
        o2, m2, l2 = attn_with_stats(v[k:], w)
        return merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize=True)

    o1, m1, l1 = attn_with_stats(v[:k], w)
    o2, m2, l2 = attn_with_stats(v[k:], w)
    with torch.no_grad():
        for name, fn, byts in (
                ("two_phase", two_phase, (n + 5) * slab),
                ("merge", lambda: merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize=True),
                 3 * slab)):
            for _ in range(3):
                fn()
            st = summarize(timed_steps(fn, steps, flush))
            out[name] = {"us": st["mean_ms"] * 1e3, "bytes": byts,
                         "tbps": byts / (st["mean_ms"] * 1e-3) / 1e12,
                         "frac": byts / (hbm_gbs * 1e9) / (st["mean_ms"] * 1e-3)}
    return out


def stage_times(v, steps, flush, hbm_gbs):
    """The decoder's arena staging at one slab [B, T, D]: stage_partial (one
    kernel: partial + out written to the new partial and the arena slot, 4 slab
    passes) against the reference's partial + out then arena.copy_ (two
    kernels, 5 slab passes)."""
    from switchyard import stage_partial

    n, b, t, d = v.shape
    slab = b * t * d * ITEM
    partial, out = v[0], v[1]
    arena = torch.empty(2, b, t, d, device=v.device, dtype=v.dtype)
    res = {}
    with torch.no_grad():
        for name, fn, byts in (
                ("fused", lambda: stage_partial(partial, out, arena[1]), 4 * slab),
                ("add_then_copy", lambda: arena[1].copy_(partial + out), 5 * slab)):
            for _ in range(3):
                fn()
            st = summarize(timed_steps(fn, steps, flush))
            res[name] = {"us": st["mean_ms"] * 1e3, "bytes": byts,
                         "tbps": byts / (st["mean_ms"] * 1e-3) / 1e12,
                         "frac": byts / (hbm_gbs * 1e9) / (st["mean_ms"] * 1e-3)}
    return res


def host_cost(dev, calls=400):
    """Host time per call of the public API on a tiny shape (N=9, 8 tokens,
    D=2048 bf16; the kernels take a few microseconds, so the host is the
    slower side and nothing waits on the GPU): the forward under no_grad, the
    forward + backward through autograd, and one raw C-ABI call (sy_plan_kind)
    for the ctypes cost alone. Microseconds per call."""
    from switchyard import _native, block_attn_res_triton

    gen = torch.Generator(device=dev).manual_seed(5)
    v = torch.randn(9, 1, 8, 2048, device=dev, generator=gen).to(torch.bfloat16)
    w = (torch.randn(2048, device=dev, generator=gen) / 45.0).to(torch.bfloat16)
    g = torch.randn(1, 8, 2048, device=dev, generator=gen).to(torch.bfloat16)

    def fwd():
        with torch.no_grad():
            block_attn_res_triton(v, w)

    def fwd_bwd():
        vv = v.detach().requires_grad_(True)
        ww = w.detach().requires_grad_(True)
        block_attn_res_triton(vv, ww).backward(g)

    def raw():
        _native.lib.sy_plan_kind(0, 9, 8, 2048, 1, 0)

    res = {}
    for name, fn in (("forward", fwd), ("forward_backward", fwd_bwd), ("ctypes_call", raw)):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(calls):
            fn()
        res[name + "_us"] = (time.perf_counter() - t0) / calls * 1e6
        torch.cuda.synchronize()
    return res


def e2e_times(dev, steps, n, b, t, d, op, pipe_steps=30):
    """The step through the public API from pinned host buffers, every step:
    H2D of v, w and dout, forward + backward (block_attn_res_triton), and D2H
    of the results out, dv and dw -- all inside the events.

    ``serial``: each step alone (copy in, compute, copy out, one after the
    other). ``pipelined``: the same K steps with the next step's H2D on a copy
    stream and the previous step's D2H on another, overlapping the compute (two
    device buffer sets; PCIe carries the two directions at once); the time is
    from before the first H2D to after the last D2H, divided by K = pipe_steps
    (the first step's H2D and the last step's D2H, which nothing overlaps, are
    spread over K steps: ~1/K of a step's copy time)."""
    gen = torch.Generator().manual_seed(3)
    v_h = torch.randn(n, b, t, d, generator=gen).to(torch.bfloat16).pin_memory()
    w_h = (torch.randn(d, generator=gen) / math.sqrt(d)).to(torch.bfloat16).pin_memory()
    g_h = torch.randn(b, t, d, generator=gen).to(torch.bfloat16).pin_memory()
    outs_h = [(torch.empty(b, t, d, dtype=torch.bfloat16).pin_memory(),
               torch.empty(n, b, t, d, dtype=torch.bfloat16).pin_memory(),
               torch.empty(d, dtype=torch.bfloat16).pin_memory()) for _ in range(2)]
    ins_d = [(torch.empty(n, b, t, d, dtype=torch.bfloat16, device=dev),
              torch.empty(d, dtype=torch.bfloat16, device=dev),
              torch.empty(b, t, d, dtype=torch.bfloat16, device=dev)) for _ in range(2)]
    h2d = v_h.numel() * 2 + w_h.numel() * 2 + g_h.numel() * 2
    d2h = sum(x.numel() * 2 for x in outs_h[0])

    def compute(k):
        vd, wd, gd = ins_d[k]
        vv = vd.detach().requires_grad_(True)
        ww = wd.detach().requires_grad_(True)
        out = op(vv, ww)
        out.backward(gd)
        return out.detach(), vv.grad, ww.grad

    def serial_step():
        vd, wd, gd = ins_d[0]
        vd.copy_(v_h, non_blocking=True)
        wd.copy_(w_h, non_blocking=True)
        gd.copy_(g_h, non_blocking=True)
        for dst, src in zip(outs_h[0], compute(0)):
            dst.copy_(src, non_blocking=True)

    for _ in range(3):
        serial_step()
    torch.cuda.synchronize()
    ms = []
    for _ in range(steps):
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        serial_step()
        e_.record()
        torch.cuda.synchronize()
        ms.append(s_.elapsed_time(e_))

    main = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def pipelined(k_steps):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        loaded = [torch.cuda.Event() for _ in range(k_steps)]
        consumed = [torch.cuda.Event() for _ in range(k_steps)]
        start.record(main)
        up.wait_event(start)
        down.wait_event(start)
        for i in range(k_steps):
            k = i & 1
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(consumed[i - 2])  # compute of step i-2 is done with set k
                for dst, src in zip(ins_d[k], (v_h, w_h, g_h)):
                    dst.copy_(src, non_blocking=True)
                loaded[i].record(up)
            main.wait_event(loaded[i])
            res = compute(k)
            consumed[i].record(main)
            down.wait_event(consumed[i])
            with torch.cuda.stream(down):
                for dst, src in zip(outs_h[k], res):
                    src.record_stream(down)
                    dst.copy_(src, non_blocking=True)
        main.wait_stream(down)
        end.record(main)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / k_steps

    pipelined(3)
    pipe_ms = pipelined(pipe_steps)
    return summarize(ms), pipe_ms, h2d, d2h


def exchange_alone(peer, part, dw, steps, align):
    """Device time of the fused partial-row reduction + peer exchange alone
    (sy_dw_exchange), each call after a device barrier across the ranks, with
    the backward's real partial rows. Returns this rank's mean in ms."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        torch.cuda._sleep(200_000)
        align()
        starts[i].record()
        peer.reduce_exchange(part, dw)
        ends[i].record()
    torch.cuda.synchronize()
    return statistics.fmean(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))


def run_ours(args):
    import torch.distributed as dist

    from switchyard import _native, block_attn_res_triton, speed_of_light  # noqa: F401
    from switchyard import sharding
    from switchyard.sharding import block_attn_res_sharded

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    n, b, t, d = REP
    v, w, dout = make_inputs(dev, rank, n, b, t, d)
    flush = L2Flush(dev)
    op = block_attn_res_triton if world == 1 else block_attn_res_sharded
    align = (lambda: sharding.device_barrier(None, dev)) if world > 1 else None

    def step():
        vv = v.detach().requires_grad_(True)
        ww = w.detach().requires_grad_(True)
        op(vv, ww).backward(dout)

    def fwd_only():
        with torch.no_grad():
            block_attn_res_triton(v, w)

    for _ in range(max(args.warmup, 3)):
        step()
        fwd_only()
        if align is not None:
            align()
    torch.cuda.synchronize()
    peer = sharding.peer_exchange(None, d, dev) if world > 1 else None

    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
        peer.start_timing()
    torch.cuda.synchronize()
    with sampler:
        step_ms = timed_steps(step, args.steps, flush, align=align, on_queued=sampler._sample
                              if sampler.ok else None)
    torch.cuda.synchronize()
    exch = None
    if world > 1:
        exch = peer.read_timing()
        dist.barrier()
    fwd_ms = timed_steps(fwd_only, args.steps, flush, align=align)
    streamed = None
    if world == 1:
        k_launch, n_groups = 20, 5
        streamed = {"fwd_ms": streamed_ms(fwd_only, k_launch, n_groups),
                    "step_ms": streamed_ms(step, k_launch, n_groups),
                    "launches_per_group": k_launch, "groups": n_groups}

    st_step, st_fwd = summarize(step_ms), summarize(fwd_ms)
    mean_step, mean_fwd = st_step["mean_ms"], st_fwd["mean_ms"]
    per_rank = None
    if world > 1:
        # the same step timed without the per-step device barrier, started
        # right after a host barrier as an unaligned loop would be: each
        # rank's events then also hold the other ranks' skew (host jitter at
        # the start, flush differences); reported beside the aligned number
        torch.cuda.synchronize()
        dist.barrier()
        unaligned = summarize(timed_steps(step, args.steps, flush))
        # the exchange kernel alone, with the backward's own partial rows
        from switchyard.triton_op import _backward_partials, _forward

        stats = _forward(v, w, 1e-6)[3]
        _, part = _backward_partials(v, w, stats, dout, 1e-6)
        dw_ = torch.empty_like(w)
        ex_ms = exchange_alone(peer, part, dw_, max(20, args.steps), align)
        mine = torch.tensor([mean_step, mean_fwd, unaligned["mean_ms"], ex_ms,
                             exch["wait_mean_us"], exch["wait_max_us"], exch["kernel_mean_us"],
                             exch["reduce_mean_us"], exch["announce_mean_us"],
                             exch["peer_sum_mean_us"]],
                            device=dev, dtype=torch.float64)
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        allr = torch.stack(allr).tolist()
        mean_step = max(r[0] for r in allr)
        mean_fwd = max(r[1] for r in allr)
        per_rank = {
            "step_ms": [r[0] for r in allr],
            "fwd_ms": [r[1] for r in allr],
            "step_unaligned_ms": [r[2] for r in allr],
            "exchange_kernel_alone_us": [r[3] * 1e3 for r in allr],
            "exchange_flag_wait_mean_us": [r[4] for r in allr],
            "exchange_flag_wait_max_us": [r[5] for r in allr],
            "exchange_kernel_in_step_mean_us": [r[6] for r in allr],
            "exchange_phase_partial_sum_us": [r[7] for r in allr],
            "exchange_phase_announce_us": [r[8] for r in allr],
            "exchange_phase_peer_sum_us": [r[9] for r in allr],
        }

    fwd_b, bwd_b, tot_b = alg_bytes(n, b, t, d)
    peak, peak_kind = load_peaks()
    e2e = None
    if not args.no_extras:
        # every rank (the sharded op's backward exchanges dw with all of them)
        if world > 1:
            dist.barrier()
        e2e_serial, pipe_ms, h2d, d2h = e2e_times(dev, 10, n, b, t, d, op)
        pipe_max, serial_max = pipe_ms, e2e_serial["mean_ms"]
        if world > 1:
            tt = torch.tensor([pipe_ms, serial_max], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            pipe_max, serial_max = tt.tolist()
        e2e = {
            "value": world * tot_b / (pipe_max * 1e-3) / 1e12,
            "unit": "TB/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": pipe_max,
            "serial_ms_per_step": serial_max,
            "serial_value": world * tot_b / (serial_max * 1e-3) / 1e12,
            "api": ("switchyard.block_attn_res_triton" if world == 1 else
                    "switchyard.sharding.block_attn_res_sharded") +
                   " (autograd) from pinned host buffers on every rank: H2D of v, w, dout and D2H "
                   "of out, dv, dw every step (bytes per rank); value: the next step's H2D and the "
                   "previous step's D2H overlap the compute on two copy streams, 30 steps "
                   "from the first H2D to the last D2H (serial_*: one step at a time, 10 "
                   "steps); max over ranks",
        }
    result = None
    if rank == 0:
        kt, p_rows = kernel_times(_native, v, w, dout, args.steps, flush, None)
        floor_us = launch_floor(dev, args.steps, flush)
        value = world * tot_b / (mean_step * 1e-3) / 1e12
        bwd_ach = bwd_b / (kt["bwd"]["mean_ms"] * 1e-3) / 1e9
        fwd_ach = fwd_b / (kt["fwd"]["mean_ms"] * 1e-3) / 1e9
        sol_ach = fwd_b / (kt["speed_of_light"]["mean_ms"] * 1e-3) / 1e9
        traffic = read_traffic()
        result = {
            "metric": METRIC,
            "value": value,
            "unit": "TB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": mean_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: v~N(0,1), w~N(0,1/D), dout~N(0,1), seeds 1000+rank / 1 / 1000+rank",
            "config": {
                "workload": "Block AttnRes forward+backward (block_attn_res_triton, autograd) per step",
                "N": n, "B": b, "T": t, "D": d, "tokens_per_rank": b * t,
                "l2": "flushed before every timed step, outside its events: 384 MiB written, "
                      "then 256 MiB of another buffer read (no dirty flush lines left in L2)",
                "parallelism": f"token-axis shards x{world}" if world > 1 else "single GPU",
                "timing": ("per step: L2 flush, spin kernel, device-side barrier across the ranks' "
                           "streams (sy_dw_exchange on one value), then CUDA events around the "
                           "step on every rank; value uses the max over ranks of the mean"
                           if world > 1 else
                           "per step: L2 flush, spin kernel, then CUDA events around the step"),
            },
            "fwd_us": mean_fwd * 1e3,
            "fwd_bwd_us": mean_step * 1e3,
            "fwd_tbps": world * fwd_b / (mean_fwd * 1e-3) / 1e12,
            "fwd_frac_of_peak": (fwd_b / (mean_fwd * 1e-3) / 1e9) / peak,
            "fwd_bwd_frac_of_peak": (tot_b / (mean_step * 1e-3) / 1e9) / peak,
            "step_stats": st_step,
            "fwd_stats": st_fwd,
            "roofline": {
                "kernel": kernel_label(_native, "bwd", n, b * t, d),
                "bound": "hbm",
                "achieved": bwd_ach,
                "peak": peak,
                "unit": "GB/s",
                "frac": bwd_ach / peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "algorithmic_bytes": bwd_b,
                "traffic": traffic.get("bwd"),
            },
            "roofline_fwd": {
                "kernel": kernel_label(_native, "fwd", n, b * t, d),
                "bound": "hbm",
                "achieved": fwd_ach,
                "peak": peak,
                "unit": "GB/s",
                "frac": fwd_ach / peak,
                "algorithmic_bytes": fwd_b,
                "traffic": traffic.get("fwd"),
                "speed_of_light_kernel_gbs": sol_ach,
                "frac_of_speed_of_light": fwd_ach / sol_ach,
            },
            "kernels_ms": {k: v_["mean_ms"] for k, v_ in kt.items()},
            # one-CTA kernel of ours timed the same way: the fixed cost of the
            # method (two events, one grid launched and retired)
            "launch_floor_us": floor_us,
            "dw_partial_rows": p_rows,
            # per step: forward, backward, and the dw reduction -- fused with the
            # peer exchange on N > 1 (sy_dw_exchange); on N > 1 also the per-step
            # device barrier (outside each step's events)
            "gpu_launches": (3 if world == 1 else 4) * args.steps,
            "clocks": sampler.summary(),
        }
        if per_rank is not None:
            result["per_rank"] = per_rank
        # each kernel alone, 20 launches back to back: what it sustains without the
        # per-launch event-to-kernel latency (launch_floor_us) of the figures above
        for key, kname, nbytes in (("roofline", "bwd", bwd_b), ("roofline_fwd", "fwd", fwd_b)):
            b2b = kt[kname].get("back_to_back_ms")
            if b2b:
                result[key]["back_to_back_us"] = b2b * 1e3
                result[key]["achieved_back_to_back"] = nbytes / (b2b * 1e-3) / 1e9
                result[key]["frac_back_to_back"] = nbytes / (b2b * 1e-3) / 1e9 / peak
        if streamed is not None:
            sf, ss = streamed["fwd_ms"], streamed["step_ms"]
            result["streamed"] = {
                "method": "20 back-to-back calls (forward: block_attn_res_triton under no_grad; "
                          "step: forward + backward through autograd) between one pair of CUDA "
                          "events after a spin kernel covering their queueing, no L2 flush "
                          "(v is 151 MB, L2 126 MB, v read evict-first), median of 5 groups; "
                          "the per-step numbers above include each call's event-to-kernel "
                          "latency (launch_floor_us), these do not",
                "launches_per_group": streamed["launches_per_group"],
                "groups": streamed["groups"],
                "fwd_us": sf * 1e3,
                "fwd_tbps": fwd_b / (sf * 1e-3) / 1e12,
                "fwd_frac_of_peak": (fwd_b / (sf * 1e-3) / 1e9) / peak,
                "fwd_bwd_us": ss * 1e3,
                "fwd_bwd_tbps": tot_b / (ss * 1e-3) / 1e12,
                "fwd_bwd_frac_of_peak": (tot_b / (ss * 1e-3) / 1e9) / peak,
            }

    if not args.no_extras and rank == 0:
        result["batched"] = batched_times(v, max(20, args.steps // 4), flush, peak)
        result["batched_train"] = batched_train_times(v, max(10, args.steps // 10), flush, peak)
        result["arena_stage"] = stage_times(v, max(20, args.steps // 4), flush, peak)
        result["host_us_per_call"] = host_cost(dev)
        result["e2e"] = e2e
    if rank == 0 and world == 1:
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if world > 1:
        dist.barrier()
        sharding._PEER.clear()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def kernel_label(native, op: str, n: int, bt: int, d: int, dtype=torch.bfloat16) -> str:
    """Name of the kernel the C ABI plans for this shape (sy_plan_info)."""
    code = {"fwd": 0, "bwd": 1}[op]
    info = native.plan_info(code, n, bt, d, 1, dtype)
    kind = info["kind"]
    if kind == 3:
        streams = info["grid"] * info["groups"]
        per = -(-bt // streams)  # whole tokens per token stream (at most)
        kw = info["threads_per_group"] // 32
        if op == "bwd":
            name = "stream_bwd_kernel"
        elif info["chunks_per_thread"] == 8:
            name = "stream_fwd_reread_kernel" if kw == 1 else "stream_fwd_split_kernel"
        else:
            name = "stream_fwd_kernel"
        who = "warps" if kw == 1 else f"streams of {kw} warps"
        shape = (f"row stream, {info['groups']} {who} x {per} tokens, "
                 f"{info['stages']} row buffers per stream")
    elif kind == 1:
        name = f"reg_{op}_kernel"
        shape = (f"register tile, {info['groups']} groups x {info['threads_per_group'] // 32} warps, "
                 f"{info['chunks_per_thread']} chunk/thread, {info['stages']} stages")
    elif kind == 2:
        name, shape = f"tile_{op}_kernel", "shared-memory tile"
    else:
        name, shape = f"gen_{op}_kernel", "generic"
    return f"{name} (sy_{op}; {shape})"


def read_traffic():
    """DRAM bytes per launch from the committed ncu summary, if one exists:
    lines ``traffic_bytes_per_launch <fwd|bwd> <bytes>`` in profiles/*.txt."""
    out = {}
    for p in sorted((ROOT / "profiles").glob("*.txt")):
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) == 3 and parts[0] == "traffic_bytes_per_launch":
                try:
                    out[parts[1]] = float(parts[2])
                except ValueError:
                    pass
    return out


# ----------------------------------------------------------------------------- reference arm


def run_reference(args):
    """The reference's PyTorch eager CPU path (restated in oracle/eager_port.py:
    the reference's own package cannot travel to the GPU box) on the bench's
    own workload -- N=9 B=1 T=4096 D=2048 bf16, forward + backward through
    autograd -- on all host threads; rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle.eager_port import fwd_bwd

    torch.set_num_threads(os.cpu_count() or 1)
    n, b, t, d = REP
    gen = torch.Generator().manual_seed(0)
    v = torch.randn(n, b, t, d, generator=gen).to(torch.bfloat16)
    w = (torch.randn(d, generator=gen) / math.sqrt(d)).to(torch.bfloat16)
    g = torch.randn(b, t, d, generator=gen).to(torch.bfloat16)
    for _ in range(max(args.warmup, 1)):
        fwd_bwd(v, w, g)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fwd_bwd(v, w, g)
        times.append(time.perf_counter() - t0)
    mean = statistics.fmean(times)
    _, _, tot = alg_bytes(n, b, t, d)
    value = tot / mean / 1e12
    sample = (f"the whole workload each step: reference eager fwd+bwd (oracle/eager_port.py) at "
              f"N={n} B={b} T={t} D={d} bf16, {torch.get_num_threads()} threads of {cpu_model()}")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "TB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": mean * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: v~N(0,1), w~N(0,1/D), dout~N(0,1)",
        "config": {"workload": "Block AttnRes forward+backward, reference PyTorch eager on CPU",
                   "N": n, "B": b, "T": t, "D": d},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample, "same_config": True,
                         "cpu_count": os.cpu_count(), "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


SWEEP_SHAPES = [(9, 1, 4096, 2048), (9, 1, 32768, 2048), (4, 2, 4096, 2048), (9, 1, 4096, 1024),
                (9, 1, 4096, 4096), (17, 1, 4096, 2048), (9, 1, 4096, 8192)]


def run_sweep(args):
    """Forward, backward and fwd+bwd step (forward, backward, dw reduction as
    one step, timed like the bench's kernels: clean L2, CUDA events) for each
    dtype at each of SWEEP_SHAPES; TB/s of the algorithmic bytes and the
    fraction of the measured copy peak. Synthetic inputs as the bench's."""
    from switchyard import _native

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = L2Flush(dev)
    peak = load_peak_field("hbm_gbs")
    steps = min(args.steps, 30)
    for shape in SWEEP_SHAPES:
        n, b, t, d = shape
        bt = b * t
        for dt in (torch.bfloat16, torch.float16, torch.float32):
            v, w, dout = make_inputs(dev, 0, n, b, t, d, dtype=dt)
            res, p = kernel_times(_native, v, w, dout, steps, flush, None)
            out = torch.empty(b, t, d, device=dev, dtype=dt)
            stats = torch.empty(bt, _native.stats_stride(n), device=dev, dtype=torch.float32)
            dv = torch.empty_like(v)
            part = torch.empty(p, d, device=dev, dtype=torch.float32)
            dw = torch.empty(d, device=dev, dtype=dt)

            def step():
                _native.fwd(v, w, out, stats, n, bt, d, 1e-6)
                _native.bwd(v, w, dout, stats, dv, part, n, bt, d, 1e-6)
                _native.dw_reduce(part, dw)

            for _ in range(3):
                step()
            st = summarize(timed_steps(step, steps, flush))
            fb, bb, tot = alg_bytes(n, b, t, d, dt.itemsize)
            line = {"shape": {"N": n, "B": b, "T": t, "D": d}, "dtype": str(dt).replace("torch.", ""),
                    "fwd_kernel": kernel_label(_native, "fwd", n, bt, d, dt),
                    "bwd_kernel": kernel_label(_native, "bwd", n, bt, d, dt)}
            for name, byts, ms in (("fwd", fb, res["fwd"]["median_ms"]), ("bwd", bb, res["bwd"]["median_ms"]),
                                   ("step", tot, st["median_ms"])):
                line[name] = {"us": round(ms * 1e3, 1), "tbps": round(byts / ms / 1e9, 3),
                              "frac_of_peak": round(byts / ms / 1e6 / peak, 3) if peak else None}
            print(json.dumps(line), flush=True)
            del v, dout, dv, out, part
            torch.cuda.empty_cache()


GRID_N = (2, 3, 5, 9, 17, 33)
GRID_B = (1, 4)
GRID_T = (4096, 16384, 65536)
GRID_D = (1024, 2048, 4096, 8192)


def f64_tokens(v, w, g, eps=1e-6):
    """Float64 evaluation of the operator on a few tokens, on the GPU (the
    sweep's checker; the math of reference.py:42-59 and its gradient):
    v [N, K, D], w [D], g [K, D] -> out [K, D], dv [N, K, D], and the tokens'
    contribution to dw [D]."""
    v, w, g = v.double(), w.double(), g.double()
    d = v.shape[-1]
    r = torch.rsqrt(v.pow(2).mean(-1) + eps)              # [N, K]
    a = torch.einsum("d,nkd->nk", w, v)
    alpha = torch.softmax(a * r, dim=0)
    out = torch.einsum("nk,nkd->kd", alpha, v)
    G = torch.einsum("kd,nkd->nk", g, v)
    dlogit = alpha * (G - (alpha * G).sum(0, keepdim=True))
    da = dlogit * r
    dssq = -dlogit * a * r.pow(3) / (2.0 * d)
    dv = alpha[..., None] * g[None] + da[..., None] * w + 2.0 * dssq[..., None] * v
    dw = torch.einsum("nk,nkd->d", da, v)
    return out, dv, dw


def f64_dw(v, w, g, eps=1e-6):
    """The tokens' float64 contribution to dw (as f64_tokens, without dv)."""
    v, w, g = v.double(), w.double(), g.double()
    r = torch.rsqrt(v.pow(2).mean(-1) + eps)
    a = torch.einsum("d,nkd->nk", w, v)
    alpha = torch.softmax(a * r, dim=0)
    G = torch.einsum("kd,nkd->nk", g, v)
    da = alpha * (G - (alpha * G).sum(0, keepdim=True)) * r
    return torch.einsum("nk,nkd->d", da, v)


def rel_l2_t(got, want) -> float:
    return ((got.double() - want).norm() / want.norm().clamp_min(1e-300)).item()


def bf16_floor(want) -> float:
    """Relative L2 error of rounding the float64 values to bf16 (the dtype
    floor the parity bar is a multiple of)."""
    return rel_l2_t(want.to(torch.bfloat16), want)


def run_grid(args):
    """The shape grid: N in GRID_N, B in GRID_B, T in GRID_T, D in GRID_D,
    bf16, v ~ N(0,1), w ~ N(0, 1/D), dout ~ N(0,1), each rank generating its
    own contiguous token shard (seed 1000 + rank; w shared). Shapes whose
    per-GPU footprint (v, dv, dout, out, statistics, partial rows) does not fit
    in 85 % of the free memory are skipped, as the reference skips its > 24
    GiB cases (bench/bench_operator.py:321-324).

    Per shape: the forward and the fwd+bwd step (forward, backward, dw
    reduction fused with the peer exchange on N > 1), each timed with CUDA
    events after a device barrier across the ranks (max over ranks of the
    mean), L2 flushed before each; TB/s of the global algorithmic bytes and the
    per-GPU fraction of the measured copy peak. Checked in float64 on the GPU:
    out and dv on 8 sampled tokens per rank, dw over every token (chunked) --
    relative L2 against the float64 values as a multiple of the bf16 floor."""
    import torch.distributed as dist

    from switchyard import block_attn_res_triton, sharding
    from switchyard.sharding import block_attn_res_sharded, token_range

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    align = (lambda: sharding.device_barrier(None, dev)) if world > 1 else None
    op = block_attn_res_sharded if world > 1 else block_attn_res_triton
    peak = load_peak_field("hbm_gbs") or FALLBACK_HBM_GBS
    flush = L2Flush(dev)
    shapes = sorted(((n, b, t, d) for n in GRID_N for b in GRID_B for t in GRID_T for d in GRID_D),
                    key=lambda s: (s[0] * s[1] * s[2] * s[3], s))
    done = 0
    for n, b, t, d in shapes:
        if args.grid_max_shapes and done >= args.grid_max_shapes:
            break
        bt = b * t
        lo, hi = token_range(bt, world, rank)
        btl = hi - lo
        free, _ = torch.cuda.mem_get_info(dev)
        need = ((2 * n + 2) * btl * d * 2 + btl * 128 * 4 + 1024 * d * 4) * 1.05
        fits = torch.tensor([1.0 if need < 0.85 * free else 0.0], device=dev)
        if world > 1:
            dist.all_reduce(fits, op=dist.ReduceOp.MIN)
        line = {"shape": {"N": n, "B": b, "T": t, "D": d}, "world": world, "dtype": "bf16",
                "tokens_per_rank": btl}
        if fits.item() < 1.0:
            if rank == 0:
                line["skipped"] = f"per-GPU footprint {need / 2**30:.1f} GiB > 85% of free memory"
                print(json.dumps(line), flush=True)
            continue
        gen = torch.Generator(device=dev).manual_seed(1000 + rank)
        v = torch.empty(n, 1, btl, d, device=dev, dtype=torch.bfloat16).normal_(generator=gen)
        dout = torch.empty(1, btl, d, device=dev, dtype=torch.bfloat16).normal_(generator=gen)
        gw = torch.Generator(device=dev).manual_seed(1)
        w = (torch.randn(d, device=dev, generator=gw) / math.sqrt(d)).to(torch.bfloat16)
        fwd_b, _, tot_b = alg_bytes(n, 1, btl, d)
        est_ms = tot_b / 5e9
        steps = int(min(20, max(3, 300 / max(est_ms, 1e-3))))
        res = {}

        def fwd():
            with torch.no_grad():
                op(v, w)

        def step():
            vv = v.detach().requires_grad_(True)
            ww = w.detach().requires_grad_(True)
            op(vv, ww).backward(dout)

        for name, fn, byts in (("fwd", fwd, fwd_b), ("fwd_bwd", step, tot_b)):
            for _ in range(2):
                fn()
                if align is not None:
                    align()
            ms = statistics.fmean(timed_steps(fn, steps, flush, align=align))
            if world > 1:
                tt = torch.tensor([ms], device=dev, dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                ms = tt.item()
            res[name] = {"us": ms * 1e3, "tbps": world * byts / (ms * 1e-3) / 1e12,
                         "frac_of_peak": byts / (ms * 1e-3) / 1e9 / peak}
        # parity: out and dv on 8 sampled tokens of this rank, dw over all tokens
        vv = v.detach().requires_grad_(True)
        ww = w.detach().requires_grad_(True)
        out = op(vv, ww)
        out.backward(dout)
        pick = torch.linspace(0, btl - 1, 8, device=dev).long()
        o64, dv64, _ = f64_tokens(v[:, 0, pick], w, dout[0, pick])
        err = torch.tensor([rel_l2_t(out[0, pick], o64) / bf16_floor(o64),
                            rel_l2_t(vv.grad[:, 0, pick], dv64) / bf16_floor(dv64)],
                           device=dev, dtype=torch.float64)
        dw64 = torch.zeros(d, device=dev, dtype=torch.float64)
        chunk = max(1, int(2**26 // (n * d)))  # 512 MiB per float64 temporary
        for c0 in range(0, btl, chunk):
            dw64 += f64_dw(v[:, 0, c0:c0 + chunk], w, dout[0, c0:c0 + chunk])
        if world > 1:
            dist.all_reduce(err, op=dist.ReduceOp.MAX)
            dist.all_reduce(dw64)
        dw_err = rel_l2_t(ww.grad, dw64) / bf16_floor(dw64)
        res["parity_x_bf16_floor"] = {"out_sampled": err[0].item(), "dv_sampled": err[1].item(),
                                      "dw": dw_err}
        line.update(res)
        line["timed_steps"] = steps
        if rank == 0:
            print(json.dumps(line), flush=True)
        del v, dout, vv, ww, out, dw64
        torch.cuda.empty_cache()
        done += 1
    if world > 1:
        dist.barrier()
        sharding._PEER.clear()
        dist.destroy_process_group()


def run_decoder(args):
    """The 1.3B decoder (switchyard.decoder, 24 layers, hidden
    2048, 16 heads, SwiGLU 5632, 8 blocks, vocabulary 32000, N(0, 0.02) init)
    trained in bf16 with AdamW on synthetic tokens uniform over the vocabulary,
    B x T tokens per GPU, for the standard residual and for Block AttnRes on
    this package's kernels (arena sources). Under torchrun the model is wrapped
    in DistributedDataParallel: NCCL all-reduces the gradient buckets during
    the backward, the only collective (the operator itself needs none). The
    pattern of the reference's bench/bench_ddp.py:40-126, for any world size.

    Per mode: the step's device time (CUDA events around each step, mean, max
    over ranks) and global tokens/s; at N > 1 also the same step without the
    gradient all-reduce (DDP no_sync) -- the difference is the all-reduce's
    exposed share of the step -- an all-reduce of one flat buffer of the
    model's gradient size on its own, and the rank-gradient check: every
    rank's gradients after a synchronised backward against rank 0's
    (broadcast), max abs deviation."""
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel

    from switchyard.decoder import Decoder, DecoderConfig

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    b, t = args.decoder_batch, args.decoder_seq
    steps, warmup = max(args.steps, 1), max(args.warmup, 3)
    results = {}
    for residual in ("standard", "switchyard"):
        cfg = DecoderConfig(residual=residual, sources="arena")
        torch.manual_seed(0)
        with torch.device(dev):
            model = Decoder(cfg)
        model = model.to(torch.bfloat16)
        n_params = sum(p.numel() for p in model.parameters())
        net = DistributedDataParallel(model, device_ids=[local]) if world > 1 else model
        opt = torch.optim.AdamW(net.parameters(), lr=1e-6)
        gen = torch.Generator(device=dev).manual_seed(1234 + rank)
        idx = torch.randint(0, cfg.vocab_size, (b, t), device=dev, generator=gen)
        tgt = torch.randint(0, cfg.vocab_size, (b, t), device=dev, generator=gen)

        def step(sync=True):
            opt.zero_grad(set_to_none=True)
            if sync or world == 1:
                net(idx, tgt)[1].backward()
            else:
                with net.no_sync():
                    net(idx, tgt)[1].backward()
            opt.step()

        def timed(sync=True):
            for _ in range(warmup):
                step(sync)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(steps)]
            for s_, e_ in ev:
                s_.record()
                step(sync)
                e_.record()
            torch.cuda.synchronize()
            ms = statistics.fmean(s_.elapsed_time(e_) for s_, e_ in ev)
            if world > 1:
                tt = torch.tensor([ms], device=dev, dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                ms = tt.item()
            return ms

        torch.cuda.reset_peak_memory_stats(dev)
        ms = timed(True)
        res = {"step_ms": ms, "tokens_per_s": world * b * t / (ms * 1e-3), "params": n_params,
               "peak_memory_gib": torch.cuda.max_memory_allocated(dev) / 2**30}
        if world > 1:
            ms_local = timed(False)
            res["step_no_allreduce_ms"] = ms_local
            res["allreduce_exposed_ms"] = ms - ms_local
            res["allreduce_exposed_share"] = (ms - ms_local) / ms
            opt.zero_grad(set_to_none=True)
            net(idx, tgt)[1].backward()
            flat = torch.cat([p.grad.flatten().float() for _, p in sorted(model.named_parameters())
                              if p.grad is not None])
            other = flat.clone()
            dist.broadcast(other, src=0)
            res["max_abs_grad_deviation_from_rank0"] = (flat - other).abs().max().item()
            dev_all = torch.tensor([res["max_abs_grad_deviation_from_rank0"]], device=dev)
            dist.all_reduce(dev_all, op=dist.ReduceOp.MAX)
            res["max_abs_grad_deviation_from_rank0"] = dev_all.item()
            res["grad_norm"] = flat.norm().item()
            del flat, other
            opt.zero_grad(set_to_none=True)
        results[residual] = res
        del net, model, opt
        torch.cuda.empty_cache()
    if world > 1:
        # the gradient all-reduce alone: one flat bf16 buffer of the model's size
        buf = torch.ones(results["switchyard"]["params"], dtype=torch.bfloat16, device=dev)
        for _ in range(2):
            dist.all_reduce(buf)
        torch.cuda.synchronize()
        dist.barrier()
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        for _ in range(5):
            dist.all_reduce(buf)
        e_.record()
        torch.cuda.synchronize()
        ar_ms = s_.elapsed_time(e_) / 5
        nbytes = buf.numel() * 2
        results["allreduce_alone"] = {"bytes": nbytes, "ms": ar_ms,
                                      "bus_gbs": 2 * (world - 1) / world * nbytes / (ar_ms * 1e-3) / 1e9}
        del buf
    if rank == 0:
        print(json.dumps({
            "metric": "1.3B Block AttnRes decoder bf16 training step (ms, tokens/s)",
            "n_gpus": world, "steps": steps, "warmup": warmup,
            "config": {"workload": "switchyard.decoder.Decoder 1.3B (24 layers, hidden 2048, 16 heads, "
                                   "SwiGLU 5632, 8 blocks, vocab 32000), AdamW lr 1e-6, bf16",
                       "batch_per_gpu": b, "seq_len": t,
                       "parallelism": f"DDP x{world} (NCCL gradient all-reduce)" if world > 1
                       else "single GPU"},
            "data": "synthetic tokens uniform over the vocabulary, seed 1234 + rank",
            "results": results,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile(kind: str, shape: str | None = None):
    """A handful of launches at the representative shape (or `shape`,
    "N,B,T,D") and nothing else, so that an ncu capture ends by itself in
    seconds."""
    from switchyard import _native, attn_with_stats, block_attn_res_batched, block_attn_res_triton
    from switchyard import merge_online_softmax

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, b, t, d = tuple(int(x) for x in shape.split(",")) if shape else REP
    v, w, dout = make_inputs(dev, 0, n, b, t, d)
    bt = b * t
    out = torch.empty(b, t, d, device=dev, dtype=v.dtype)
    stats = torch.empty(bt, _native.stats_stride(n), device=dev, dtype=torch.float32)
    dv = torch.empty_like(v)
    part = torch.empty(_native.bwd_partials(n, bt, d, v.dtype), d, device=dev, dtype=torch.float32)
    if kind == "bwd":
        _native.fwd(v, w, out, stats, n, bt, d, 1e-6)
    q = (torch.randn(16, d, device=dev) / math.sqrt(d)).to(v.dtype)
    for _ in range(5):
        if kind == "fwd":
            _native.fwd(v, w, out, stats, n, bt, d, 1e-6)
        elif kind == "bwd":
            _native.bwd(v, w, dout, stats, dv, part, n, bt, d, 1e-6)
        elif kind == "sol":
            _native.speed_of_light(v, out, n, bt, d)
        elif kind == "step":
            vv = v.detach().requires_grad_(True)
            ww = w.detach().requires_grad_(True)
            block_attn_res_triton(vv, ww).backward(dout)
        elif kind == "batched_bwd8":
            g8 = dout.unsqueeze(0).expand(8, b, t, d).contiguous() if _ == 0 else g8
            p8 = _native.bwd_batched_partials(n, bt, d, 8, v.dtype)
            part8 = torch.empty(p8, 8 * d, device=dev, dtype=torch.float32)
            _native.bwd_batched(v, q[:8], g8, dv, part8, n, bt, d, 8, 1e-6)
        elif kind == "merge":
            with torch.no_grad():
                if _ == 0:
                    o1, m1, l1 = attn_with_stats(v[: n // 2], w)
                    o2, m2, l2 = attn_with_stats(v[n // 2:], w)
                merge_online_softmax(o1, m1, l1, o2, m2, l2, normalize=True)
        elif kind.startswith("batched"):
            with torch.no_grad():
                block_attn_res_batched(v, q[: int(kind[len("batched"):])])
    torch.cuda.synchronize()


def main():
    faulthandler.enable()
    args = parse_args()
    if args.profile:
        run_profile(args.profile, args.shape)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.decoder:
        run_decoder(args)
        return
    if args.grid:
        run_grid(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
