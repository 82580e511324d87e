#!/usr/bin/env python3
"""Benchmark of the B200 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl amp_b200|reference]

Default workload ``fp8_quant``: per-tensor amax-scaled FP8 E4M3 quantise +
dequantise of 2^26 bf16 values (N(0,1) with 0.1% N(0,50) outliers).  One step
is one quantise (amax pass + encode pass) and one dequantise of the whole
tensor; the metric is algorithmic bytes moved (8 B/element: 5 quantise +
3 dequantise) per second.  For N > 1 (torchrun, one process per GPU) every
rank quantises its own 2^26-element shard (weak scaling) against the global
amax, obtained by a 1-float NCCL all-reduce(MAX) inside the step.

Timing: W untimed warm-up steps; then K steps, each bracketed by CUDA events
on the launching stream, with a 256 MiB L2 flush before every step (outside
the events); barrier + synchronize on both sides; max over ranks.
``e2e`` repeats the metric through the host-pointer C entry point
(pinned host input, H2D + kernels + D2H inside the timed region).

``--impl reference`` times AMP's own CPU codec (include/fp8.hpp, compiled from
the reference sources into oracle/_ref) on this host's cores, on a bounded
sample of the same workload; without that build it times the oracle port.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def load_traffic():
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
class Dist:
    def __init__(self, n_gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            import torch
            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = dist
        if n_gpus != self.world and self.world > 1:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# --------------------------------------------------------------------------
# clocks during the timed region (NVML, the library nvidia-smi reads)
# --------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML absent: report no samples rather than fail the bench
            self.nv = None
        self.period = period_s

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = sorted(v for k, v in self.REASONS.items() if bits & k and k != 0x1)
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# --------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------
class QuantWorkload:
    name = "fp8_quant"
    metric = "fp8_e4m3_quant_dequant_GBps"
    unit = "GB/s"
    dtype = "bf16->e4m3->bf16"
    bytes_per_elem = 8  # quantise 5 (amax read 2 + read 2 + write 1) + dequantise 3

    def __init__(self, dist: Dist, n: int):
        import torch
        from amp_b200 import fp8, workloads
        self.torch, self.fp8, self.dist = torch, fp8, dist
        self.n = n
        dev = torch.device("cuda", torch.cuda.current_device())
        self.x = workloads.quant_input_torch(n, seed=1234 + dist.rank, device=dev)
        self.q = torch.empty(n, dtype=torch.uint8, device=dev)
        self.y = torch.empty(n, dtype=torch.bfloat16, device=dev)
        self.scale = torch.empty(1, dtype=torch.float32, device=dev)
        self.amax = torch.empty(1, dtype=torch.float32, device=dev)
        self.ws = torch.empty(fp8.workspace_bytes(n), dtype=torch.uint8, device=dev)
        self.stream = torch.cuda.current_stream()
        self.kernel_events = None

    def launches_per_step(self) -> int:
        return 3 if self.dist.world == 1 else 4

    def config(self):
        return {"workload": "fp8_e4m3_per_tensor_quant_dequant", "elements_per_gpu": self.n,
                "input": "bf16 N(0,1) + 0.1% N(0,50) outliers (seeded, synthetic)",
                "scale": "amax/448, RNE satfinite", "global_elements": self.n * self.dist.world,
                "l2": "256 MiB flush before every timed step",
                "parallelism": f"shard{self.dist.world}+allreduce_max(1 float)"
                if self.dist.world > 1 else "single"}

    def step(self, ev=None):
        fp8, torch = self.fp8, self.torch
        if self.dist.world == 1:
            if ev: ev[0].record()
            fp8.quantize_e4m3(self.x, workspace=self.ws, out=self.q, scale=self.scale)
            if ev: ev[1].record()
            fp8.dequantize_e4m3(self.q, self.scale, out=self.y)
            if ev: ev[2].record()
        else:
            fp8.amax_bf16(self.x, workspace=self.ws, out=self.amax)
            self.dist.pg.all_reduce(self.amax, op=self.dist.pg.ReduceOp.MAX)
            if ev: ev[0].record()
            fp8.quantize_e4m3_from_amax(self.x, self.amax, out=self.q, scale=self.scale)
            if ev: ev[1].record()
            fp8.dequantize_e4m3(self.q, self.scale, out=self.y)
            if ev: ev[2].record()

    def kernel_table(self):
        """(name, algorithmic bytes per launch) for the per-kernel event spans."""
        if self.dist.world == 1:
            return [("quantise (amax + encode)", 5 * self.n), ("dequantise", 3 * self.n)]
        return [("encode_from_amax", 3 * self.n), ("dequantise", 3 * self.n)]

    # ---- end to end through the host-pointer C entry point -------------
    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        from amp_b200._lib import call
        n = self.n
        xh = self.x.cpu().pin_memory()
        qh = torch.empty(n, dtype=torch.uint8).pin_memory()
        yh = torch.empty(n, dtype=torch.bfloat16).pin_memory()
        sc = C.c_float()
        args = (xh.data_ptr(), n, qh.data_ptr(), C.byref(sc), yh.data_ptr())
        for _ in range(warmup):
            call("amp_user_fp8_quant_e4m3", *args)
        legacy = torch.cuda.default_stream()  # the entry point enqueues on stream 0
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        times = []
        for _ in range(steps):
            s.record(legacy)
            call("amp_user_fp8_quant_e4m3", *args)
            e.record(legacy)
            e.synchronize()
            times.append(s.elapsed_time(e))
        ms = sum(times) / len(times)
        return {"value": self.bytes_per_elem * n / (ms * 1e-3) / 1e9, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": 2 * n,
                "d2h_bytes_per_step": n + 2 * n + 4, "api": "amp_user_fp8_quant_e4m3"}

    # ---- CPU baseline: AMP's own codec on the host cores ----------------
    @staticmethod
    def cpu_baseline(n_full: int, budget_s: float = 10.0):
        import oracle
        from amp_b200 import workloads
        threads = len(os.sched_getaffinity(0))
        r = oracle.ref_lib()
        sample = min(n_full, 1 << 22)
        xb = workloads.quant_input_numpy(sample, seed=3)
        q = np.empty(sample, np.uint8)
        y = np.empty(sample, np.uint16)
        if r is not None:
            kind, cores = "reference", threads

            def run():
                r.ref_quant_dequant_bf16(xb.ctypes.data, sample, q.ctypes.data, y.ctypes.data,
                                         threads)
        else:
            kind, cores = "port", 1

            def run():
                qq, s, _ = oracle.quant_e4m3(xb)
                oracle.dequant_e4m3(qq, s)
        run()
        t0 = time.perf_counter()
        reps = 0
        while True:
            run()
            reps += 1
            if time.perf_counter() - t0 >= budget_s:
                break
        dt = time.perf_counter() - t0
        v = QuantWorkload.bytes_per_elem * sample * reps / dt / 1e9
        what = ("AMP fp8::f32_to_e4m3/e4m3_to_f32 (include/fp8.hpp) + amax loop, "
                f"{threads} host threads" if kind == "reference"
                else "oracle restatement (oracle/oracle.c), 1 thread")
        return {"value": v, "unit": "GB/s", "cores": cores, "kind": kind,
                "sample": f"{reps} x {sample} bf16 elements of the same distribution "
                          f"({dt:.1f} s); {what}"}


WORKLOADS = {"fp8_quant": QuantWorkload}


def l2_flusher(torch):
    buf = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def flush():
        buf.zero_()
    return flush


def run_amp(args, dist: Dist):
    import torch
    from amp_b200 import build as ampbuild
    import amp_b200
    if not amp_b200.LIB_PATH.exists():
        ampbuild.build()
    torch.cuda.set_device(dist.local_rank)
    W = WORKLOADS[args.workload](dist, args.elements)
    flush = l2_flusher(torch)
    for _ in range(args.warmup):
        flush()
        W.step()
    nk = len(W.kernel_table())
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)]
              for _ in range(args.steps)]
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    dev_index = torch.cuda.current_device()
    phys = os.environ.get("CUDA_VISIBLE_DEVICES")
    nvml_index = int(phys.split(",")[dev_index]) if phys else dev_index
    with ClockSampler(nvml_index) as clocks:
        for i in range(args.steps):
            flush()
            step_ev[i][0].record()
            W.step(events[i])
            step_ev[i][1].record()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in step_ev]
    total_ms = dist.max(sum(step_ms))
    ms_per_step = total_ms / args.steps
    units = W.bytes_per_elem * W.n * dist.world
    value = units / (ms_per_step * 1e-3) / 1e9

    # per-kernel spans -> dominant kernel roofline
    spans = []
    for k, (name, algo_bytes) in enumerate(W.kernel_table()):
        ms = statistics.mean(events[i][k].elapsed_time(events[i][k + 1])
                             for i in range(args.steps))
        spans.append((ms, name, algo_bytes))
    spans.sort(reverse=True)
    dom_ms, dom_name, dom_bytes = spans[0]
    peaks, peak_src = load_peaks()
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = load_traffic().get(W.name, {}).get(dom_name)
    roofline = {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_src == "measured" else "fallback 6650 GB/s",
                "traffic": traffic, "algorithmic_bytes": dom_bytes,
                "kernel_ms": round(dom_ms, 5),
                "all_kernels": [{"kernel": n, "ms": round(m, 5),
                                 "GBps": round(b / (m * 1e-3) / 1e9, 1)} for m, n, b in spans]}

    e2e = W.e2e(max(3, min(args.steps, 20)), 2)
    out = {
        "metric": W.metric, "value": round(value, 2), "unit": W.unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": W.dtype, "data": "synthetic (seeded, reference distribution)",
        "config": W.config(), "impl": "amp_b200",
        "gpu_launches": W.launches_per_step() * args.steps,
        "clocks": clocks.summary(), "roofline": roofline,
        "e2e": {k: (round(v, 3) if isinstance(v, float) else v) for k, v in e2e.items()},
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = WORKLOADS[args.workload].cpu_baseline(W.n)
    return out


def run_reference(args, dist: Dist):
    W = WORKLOADS[args.workload]
    if dist.rank != 0:
        return None
    n = args.elements
    import oracle
    from amp_b200 import workloads
    threads = len(os.sched_getaffinity(0))
    r = oracle.ref_lib()
    sample = min(n, 1 << 22)
    xb = workloads.quant_input_numpy(sample, seed=3)
    q = np.empty(sample, np.uint8)
    y = np.empty(sample, np.uint16)
    if r is not None:
        kind = "reference"

        def run():
            r.ref_quant_dequant_bf16(xb.ctypes.data, sample, q.ctypes.data, y.ctypes.data,
                                     threads)
    else:
        kind, threads = "port", 1

        def run():
            qq, s, _ = oracle.quant_e4m3(xb)
            oracle.dequant_e4m3(qq, s)
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    v = W.bytes_per_elem * sample / (ms * 1e-3) / 1e9
    sample_desc = (f"each step {sample} of the {n} bf16 elements (same distribution); "
                   + ("AMP fp8::f32_to_e4m3/e4m3_to_f32 (include/fp8.hpp) + amax loop"
                      if kind == "reference" else "oracle restatement (oracle/oracle.c)"))
    return {
        "metric": W.metric, "value": round(v, 3), "unit": W.unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": W.dtype, "data": "synthetic (seeded, reference distribution)",
        "config": {"workload": "fp8_e4m3_per_tensor_quant_dequant", "elements_per_gpu": n,
                   "sample_elements_per_step": sample},
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 3), "unit": W.unit, "cores": threads, "kind": kind,
                         "sample": sample_desc},
        "e2e": {"value": round(v, 3), "unit": W.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="fp8_quant")
    ap.add_argument("--impl", choices=["amp_b200", "reference"], default="amp_b200")
    ap.add_argument("--elements", type=int, default=1 << 26)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        # Only rank 0 works; the other ranks exit without touching a GPU.
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        out = run_reference(args, _RefDist())
        print(json.dumps(out), flush=True)
        return
    dist = Dist(args.gpus)
    try:
        out = run_amp(args, dist)
        if dist.rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        dist.close()


class _RefDist:
    """Rank bookkeeping for the reference arm (no process group, no GPU)."""
    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))


if __name__ == "__main__":
    main()
