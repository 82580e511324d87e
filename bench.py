#!/usr/bin/env python3
"""Benchmark of the B200 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl amp_b200|reference] [--size S]

The default (``--workload suite``) prints the headline workload's line with
every other workload's full record (value, ms_per_step, roofline with traffic,
clocks, e2e, cpu_baseline) in its ``workloads`` array, all measured in the
same process; the non-headline workloads time min(K, --suite-steps) steps.

Workloads (``--workload``):
  fp8_quant (headline) per-tensor amax-scaled FP8 E4M3 quantise + dequantise of
                       2^26 bf16 values (N(0,1), 0.1% N(0,50) outliers); metric =
                       algorithmic bytes (8 B/element) per second.  N > 1: each
                       rank its own 2^26 shard against the global amax (a 1-float
                       max all-reduce through peer mailboxes), weak scaling.
  gemm_bf16            C = A @ B, M=N=K=S (default 8192), bf16 in, fp32 accumulate,
                       bf16 out; metric = 2*S^3 FLOP per second.  N > 1: B and C
                       split along N; the all-gather of C is fused into the GEMM
                       epilogue (``--gather nccl``: NCCL after it), strong scaling.
                       ``library_bar``: cuBLAS at the same shape, same run.
  gemm_fp8             same with E4M3 operands, per-row A / per-column B scales;
                       the roofline's peak is cuBLASLt's FP8 GEMM timed in the run.
  fa2_fwd              FlashAttention-2 forward, B=4 H=32 S=4096 D=128 causal;
                       N > 1: (batch*head) split, O and lse all-gathered in the epilogue.
  fa2_bwd              the backward of the same configuration (dQ, dK, dV).
  paged_decode         GQA decode over the paged KV cache (B=8, Hq=32, Hkv=8,
                       context U[512, 16384], 16-token pages); replicas at N > 1.
  paged_prefill        the last 512 tokens of each context as a paged prefill.
  gemm_fp32            AMP's fp32 plugin GEMM, M=N=K=1024, U[-1,1] seed 0, exact
                       accumulation; e2e through amp_user_gemm_fp32 (pinned and
                       pageable host buffers); replicas at N > 1.

Timing: W untimed warm-up steps; then K steps, each bracketed by CUDA events on
the launching stream with an L2 flush before every step (256 MiB written, then
1 GiB read, outside the events); barrier + synchronize on both sides; the max over ranks.  NVML samples
SM clocks and throttle reasons during the timed region.  ``e2e`` repeats the
metric through the host-pointer C entry point (pinned host buffers, H2D +
kernels + D2H inside the timed region).  ``roofline`` reports the dominant
kernel: algorithmic bytes (or FLOPs) per launch over its event-timed duration.

``--impl reference`` times the reference's own CPU code for the workload on this
host's cores (built from the AMP sources into oracle/_ref), on a bounded sample;
without that build it times the oracle's restatement.
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
# rank 0's stdout carries exactly one JSON line: keep NCCL's banner off it
os.environ["NCCL_DEBUG"] = os.environ.get("AMP_B200_NCCL_DEBUG", "WARN")

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def load_traffic():
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


def traffic_for(W, world: int, kernel: str):
    """DRAM bytes per launch of `kernel` from the 1-GPU ncu captures
    (profiles/traffic.json).  Under weak scaling a rank's launch is the captured
    one at any N; under strong scaling at N > 1 it is a smaller one, and no figure
    is reported."""
    if world > 1 and W.scaling != "weak":
        return None
    return load_traffic().get(W.name, {}).get(kernel)


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


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
            import torch
            import torch.distributed as dist
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
        0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML absent: report no samples rather than fail the bench
            self.nv = None

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
        bits = 0
        for _, r in self.samples:
            bits |= r
        return {"sm_mhz": float(statistics.median(m for m, _ in self.samples)),
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(v for k, v in self.REASONS.items() if bits & k),
                "samples": len(self.samples)}


def timed_reps(fn, budget_s: float):
    """Run fn repeatedly for ~budget_s seconds; returns (reps, seconds)."""
    fn()
    t0 = time.perf_counter()
    reps = 0
    while True:
        fn()
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            return reps, dt


# --------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------
class QuantWorkload:
    name = "fp8_quant"
    metric = "fp8_e4m3_quant_dequant_GBps"
    unit = "GB/s"
    scale = 1e9
    dtype = "bf16->e4m3->bf16"
    bound = "hbm"
    scaling = "weak"
    bytes_per_elem = 8  # quantise 5 (amax read 2 + read 2 + write 1) + dequantise 3

    def __init__(self, dist: Dist, args):
        import torch
        from amp_b200 import fp8, workloads
        self.torch, self.fp8, self.dist, self.args = torch, fp8, dist, args
        self.n = n = args.elements
        dev = torch.device("cuda", torch.cuda.current_device())
        self.x = workloads.quant_input_torch(n, seed=1234 + dist.rank, device=dev)
        self.q = torch.empty(n, dtype=torch.uint8, device=dev)
        self.y = torch.empty(n, dtype=torch.bfloat16, device=dev)
        self.scale_t = torch.empty(1, dtype=torch.float32, device=dev)
        self.amax = torch.empty(1, dtype=torch.float32, device=dev)
        self.ws = torch.empty(fp8.workspace_bytes(n), dtype=torch.uint8, device=dev)
        self.mbox = None
        if dist.world > 1:
            # the global amax travels through peer mailboxes (one NVLink store per peer)
            from amp_b200.collective import CommGroup, PeerMailboxes
            self.mbox = PeerMailboxes(CommGroup.current())

    def close(self):
        if self.mbox is not None:
            self.mbox.close()
            self.mbox = None

    def units_per_step(self) -> float:
        return self.bytes_per_elem * self.n

    def launches_per_step(self) -> int:
        return 3 if self.dist.world == 1 else 4

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        n = args.elements
        return {"workload": "fp8_e4m3_per_tensor_quant_dequant", "elements_per_gpu": n,
                "global_elements": n * world,
                "input": "bf16 N(0,1) + 0.1% N(0,50) outliers (seeded, synthetic)",
                "scale": "amax/448, RNE satfinite", "l2": "L2 flushed before every step (256 MiB written, then 1 GiB read)",
                "parallelism": f"shard{world}+all-reduce(max) of 1 float through peer "
                               "mailboxes (NVLink stores, no NCCL)"
                if world > 1 else "single"}

    def config(self):
        return self.describe(self.args, self.dist.world, self.dist.rank)

    def kernel_table(self):
        if self.dist.world == 1:
            return [("quantise (k_amax_partials + k_quant_encode)", 5 * self.n),
                    ("dequantise (k_dequant)", 3 * self.n)]
        return [("encode_from_amax (k_quant_encode)", 3 * self.n),
                ("dequantise (k_dequant)", 3 * self.n)]

    def step(self, ev=None):
        fp8 = self.fp8
        if self.dist.world > 1:
            fp8.amax_allreduce_peer(self.x, self.mbox, workspace=self.ws, out=self.amax)
        if ev: ev[0].record()
        if self.dist.world == 1:
            fp8.quantize_e4m3(self.x, workspace=self.ws, out=self.q, scale=self.scale_t)
        else:
            fp8.quantize_e4m3_from_amax(self.x, self.amax, out=self.q, scale=self.scale_t)
        if ev: ev[1].record()
        fp8.dequantize_e4m3(self.q, self.scale_t, out=self.y)
        if ev: ev[2].record()

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        from amp_b200._lib import call
        n = self.n
        xh = self.x.cpu().pin_memory()
        qh = torch.empty(n, dtype=torch.uint8).pin_memory()
        yh = torch.empty(n, dtype=torch.bfloat16).pin_memory()
        sc = C.c_float()
        args = (xh.data_ptr(), n, qh.data_ptr(), C.byref(sc), yh.data_ptr())
        ms = _e2e_time(torch, lambda: call("amp_user_fp8_quant_e4m3", *args), steps, warmup)
        # the same call on pageable host arrays (what a plain C++ caller hands over)
        xp = xh.view(torch.int16).numpy().copy()
        qp = np.empty(n, np.uint8)
        yp = np.empty(n, np.uint16)
        argsp = (xp.ctypes.data, n, qp.ctypes.data, C.byref(sc), yp.ctypes.data)
        ms_p = _e2e_time(torch, lambda: call("amp_user_fp8_quant_e4m3", *argsp), steps, warmup)
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": 2 * n,
                "d2h_bytes_per_step": n + 2 * n + 4,
                "api": "amp_user_fp8_quant_e4m3 (pinned host buffers)",
                "pageable": {"value": self.units_per_step() / (ms_p * 1e-3) / self.scale,
                             "ms_per_step": ms_p,
                             "api": "amp_user_fp8_quant_e4m3 (pageable host arrays)"}}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        import oracle
        from amp_b200 import workloads
        r = oracle.ref_lib()
        sample = min(args.elements, 1 << 22)
        xb = workloads.quant_input_numpy(sample, seed=3)
        q = np.empty(sample, np.uint8)
        y = np.empty(sample, np.uint16)
        if r is not None:
            kind, cores = "reference", threads

            def run():
                r.ref_quant_dequant_bf16(xb.ctypes.data, sample, q.ctypes.data, y.ctypes.data,
                                         threads)
            what = "AMP fp8::f32_to_e4m3/e4m3_to_f32 (include/fp8.hpp) + amax loop"
        else:
            kind, cores = "port", 1

            def run():
                qq, s, _ = oracle.quant_e4m3(xb)
                oracle.dequant_e4m3(qq, s)
            what = "oracle restatement (oracle/oracle.c)"
        reps, dt = timed_reps(run, budget_s)
        return {"value": cls.bytes_per_elem * sample * reps / dt / cls.scale, "unit": cls.unit,
                "cores": cores, "kind": kind,
                "sample": f"{reps} x {sample} bf16 elements of the same distribution in "
                          f"{dt:.1f} s; {what}, {cores} host thread(s)"}


class GemmWorkload:
    name = "gemm_bf16"
    metric = "bf16_gemm_TFLOPS"
    unit = "TFLOP/s"
    scale = 1e12
    dtype = "bf16"
    bound = "tensor"
    scaling = "strong"
    fp8 = False

    def __init__(self, dist: Dist, args):
        import torch
        from amp_b200 import gemm
        self.torch, self.gemm, self.dist, self.args = torch, gemm, dist, args
        S = self.S = args.size
        p = dist.world
        if S % (256 * p):
            raise SystemExit(f"--size must be a multiple of {256 * p} for {p} GPUs")
        self.Np = S // p
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(77)
        a = torch.randn(S, S, generator=g, device=dev)
        b = torch.randn(S, S, generator=g, device=dev)[:, dist.rank * self.Np:(dist.rank + 1) * self.Np]
        if self.fp8:
            amax_a = a.abs().amax(dim=1).clamp_min(1e-30)
            amax_b = b.abs().amax(dim=0).clamp_min(1e-30)
            self.sa = (amax_a / 448.0).float().contiguous()
            self.sb = (amax_b / 448.0).float().contiguous()
            self.A = (a / self.sa[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
            self.B = (b / self.sb[None, :]).to(torch.float8_e4m3fn).view(torch.uint8).contiguous()
        else:
            self.A = a.to(torch.bfloat16).contiguous()
            self.B = b.to(torch.bfloat16).contiguous()
        del a, b
        self.C = torch.empty(S, self.Np, dtype=torch.bfloat16, device=dev)
        # N > 1: the all-gather is fused into the GEMM epilogue (stores into every
        # rank's C over NVLink) unless --gather nccl asks for launch + NCCL all-gather
        self.peer = None
        self.Cfull = None
        if p > 1 and args.gather == "peer":
            from amp_b200.collective import CommGroup, PeerBuffer
            self.peer = PeerBuffer(CommGroup.current(), S, S, torch.bfloat16)
        elif p > 1:
            self.Cfull = torch.empty(p, S, self.Np, dtype=torch.bfloat16, device=dev)

    def units_per_step(self) -> float:
        return 2.0 * self.S * self.S * self.Np

    def launches_per_step(self) -> int:
        return 1

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        S, p = args.size, world
        return {"workload": f"{'fp8_e4m3' if cls.fp8 else 'bf16'}_gemm", "M": S,
                "N": S, "K": S, "out": "bf16",
                "inputs": "N(0,1)" + (" quantised per row (A) / per column (B), amax/448"
                                      if cls.fp8 else ""),
                "l2": "operands (2 x %d MiB) exceed L2; L2 flushed before every step"
                      % (S * S * (1 if cls.fp8 else 2) >> 20),
                "parallelism": (f"N-split over {p} GPUs, all-gather of C fused into the GEMM "
                                "epilogue (stores into every rank's C over NVLink)"
                                if args.gather == "peer" else
                                f"N-split over {p} GPUs + NCCL all-gather of C") if p > 1
                else "single"}

    def config(self):
        return self.describe(self.args, self.dist.world, self.dist.rank)

    def kernel_table(self):
        # 256 x 256 tiles on SM pairs (k_gemm_tc2), with the all-gather epilogue at N > 1
        return [(f"k_gemm_tc2<{'e4m3' if self.fp8 else 'bf16'}>", self.units_per_step())]

    def _launch(self):
        if self.peer is not None:
            from amp_b200 import sharded
            sharded.matmul_allgather(self.A, self.B, self.peer, self.sa if self.fp8 else None,
                                     self.sb if self.fp8 else None)
        elif self.fp8:
            self.gemm.launch_matmul_fp8e4m3(self.A, self.B, self.C, self.S, self.Np, self.S,
                                            self.sa, self.sb)
        else:
            self.gemm.launch_matmul_bf16(self.A, self.B, self.C, self.S, self.Np, self.S)

    def step(self, ev=None):
        if ev: ev[0].record()
        self._launch()
        if ev: ev[1].record()
        if self.Cfull is not None:
            self.dist.pg.all_gather_into_tensor(self.Cfull, self.C)

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        from amp_b200._lib import call
        S, Np = self.S, self.Np
        Ah = self.A.cpu().pin_memory()
        Bh = self.B.cpu().pin_memory()
        Ch = torch.empty(S, Np, dtype=torch.bfloat16).pin_memory()
        if self.fp8:
            sah, sbh = self.sa.cpu().pin_memory(), self.sb.cpu().pin_memory()
            fn = lambda: call("amp_user_gemm_fp8e4m3", Ah.data_ptr(), Bh.data_ptr(),
                              sah.data_ptr(), sbh.data_ptr(), 2, Ch.data_ptr(), 1, S, Np, S)
            h2d = Ah.numel() + Bh.numel() + 4 * (S + Np)
        else:
            fn = lambda: call("amp_user_gemm_bf16", Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr(), 1,
                              S, Np, S)
            h2d = 2 * (Ah.numel() + Bh.numel())
        ms = _e2e_time(torch, fn, steps, warmup)
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 2 * S * Np,
                "api": "amp_user_gemm_fp8e4m3" if self.fp8 else "amp_user_gemm_bf16"}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        """AMP's cpu_reference_gemm on a block of C rows (fp32 operands)."""
        import oracle
        S = args.size
        g = oracle.ref_gemm_lib()
        rng = np.random.default_rng(0)
        B = rng.standard_normal((S, S), dtype=np.float32)
        rows = max(threads, 1)
        A = rng.standard_normal((rows, S), dtype=np.float32)
        Cm = np.empty((rows, S), np.float32)
        if g is not None:
            kind, cores = "reference", threads
            run = lambda: g.ref_cpu_reference_gemm_mt(A.ctypes.data, B.ctypes.data,
                                                      Cm.ctypes.data, rows, S, S, threads)
            what = "AMP cpu_reference_gemm (tests/amp_validate_kernel.cpp), rows split over threads"
        else:
            kind, cores = "port", 1
            run = lambda: oracle.lib().orc_gemm_fp32_amp(A.ctypes.data, B.ctypes.data,
                                                         Cm.ctypes.data, rows, S, S)
            what = "oracle restatement of AMP's cpu_reference_gemm"
        reps, dt = timed_reps(run, budget_s)
        flops = 2.0 * rows * S * S * reps
        return {"value": flops / dt / cls.scale, "unit": cls.unit, "cores": cores, "kind": kind,
                "sample": f"{reps} x ({rows} rows of C, N=K={S}) in {dt:.1f} s; {what}, fp32"}


class GemmFp8Workload(GemmWorkload):
    name = "gemm_fp8"
    metric = "fp8_e4m3_gemm_TFLOPS"
    dtype = "e4m3"
    fp8 = True


class GemmFp32Workload:
    """AMP's fp32 GEMM, the plugin contract's path: C = A B with M = N = K = S
    (default 1024), A and B ~ U[-1, 1] from seed 0, through the exact form
    (AMP's CPU accumulation order and rounding; bit-identical to its CPU
    reference GEMM).  The reference's tile names only label dump entries."""
    name = "gemm_fp32"
    metric = "fp32_gemm_TFLOPS"
    unit = "TFLOP/s"
    scale = 1e12
    dtype = "fp32"
    bound = "fp32"
    scaling = "weak"

    def __init__(self, dist: Dist, args):
        import torch
        from amp_b200 import gemm, workloads as wl
        self.torch, self.gemm, self.dist, self.args = torch, gemm, dist, args
        S = self.S = args.fp32_size
        dev = torch.device("cuda", torch.cuda.current_device())
        A, B = wl.gemm_fp32_inputs(S, S, S, seed=0)
        self.A_h, self.B_h = A, B
        self.A = torch.from_numpy(A).to(dev)
        self.B = torch.from_numpy(B).to(dev)
        self.C = torch.empty(S, S, dtype=torch.float32, device=dev)
        self.cfg = gemm.TileCfg(32, 32, 32)

    def units_per_step(self) -> float:
        return 2.0 * self.S ** 3

    def launches_per_step(self) -> int:
        return 1

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        S = args.fp32_size
        return {"workload": "fp32_gemm", "M": S, "N": S, "K": S,
                "inputs": "A, B ~ U[-1, 1], seed 0 (row-major fp32)",
                "accumulation": "exact: fp32 product then fp32 sum, k ascending (AMP's "
                                "cpu_reference_gemm order; bit-identical to it)",
                "tiles": "AMP tile configs (16,16,16),(32,16,16),(32,32,16),(32,32,32) name "
                         "dump entries; one blocking chosen by size",
                "l2": "L2 flushed before every step",
                "parallelism": "replicas (too small to shard)" if world > 1 else "single"}

    def config(self):
        return self.describe(self.args, self.dist.world, self.dist.rank)

    def kernel_table(self):
        return [("k_gemm_fp32<exact>", self.units_per_step())]

    def step(self, ev=None):
        if ev: ev[0].record()
        S = self.S
        self.gemm.launch_matmul(self.cfg, self.A, self.B, self.C, S, S, S)
        if ev: ev[1].record()

    def e2e(self, steps: int, warmup: int):
        """AMP's plugin symbol amp_user_gemm_fp32 on host buffers: pinned, and
        (e2e_pageable) the plain pageable arrays AMP's validator passes."""
        torch = self.torch
        from amp_b200._lib import call
        S = self.S
        Ah = torch.from_numpy(self.A_h).pin_memory()
        Bh = torch.from_numpy(self.B_h).pin_memory()
        Ch = torch.empty(S, S, dtype=torch.float32).pin_memory()
        fn = lambda: call("amp_user_gemm_fp32", Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr(), S,
                          S, S)
        ms = _e2e_time(torch, fn, steps, warmup)
        Cp = np.empty((S, S), np.float32)
        fnp = lambda: call("amp_user_gemm_fp32", self.A_h.ctypes.data, self.B_h.ctypes.data,
                           Cp.ctypes.data, S, S, S)
        ms_p = _e2e_time(torch, fnp, steps, warmup)
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": 2 * 4 * S * S,
                "d2h_bytes_per_step": 4 * S * S, "api": "amp_user_gemm_fp32 (pinned host buffers)",
                "pageable": {"value": self.units_per_step() / (ms_p * 1e-3) / self.scale,
                             "ms_per_step": ms_p,
                             "api": "amp_user_gemm_fp32 (pageable host arrays, as AMP's "
                                    "validator passes them)"}}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        """AMP's cpu_reference_gemm at the full size (fp32, rows split over threads)."""
        import oracle
        from amp_b200 import workloads as wl
        S = args.fp32_size
        A, B = wl.gemm_fp32_inputs(S, S, S, seed=0)
        Cm = np.empty((S, S), np.float32)
        g = oracle.ref_gemm_lib()
        if g is not None:
            kind, cores = "reference", threads
            run = lambda: g.ref_cpu_reference_gemm_mt(A.ctypes.data, B.ctypes.data,
                                                      Cm.ctypes.data, S, S, S, threads)
            what = "AMP cpu_reference_gemm (tests/amp_validate_kernel.cpp), rows split over threads"
        else:
            kind, cores = "port", 1
            run = lambda: oracle.lib().orc_gemm_fp32_amp(A.ctypes.data, B.ctypes.data,
                                                         Cm.ctypes.data, S, S, S)
            what = "oracle restatement of AMP's cpu_reference_gemm"
        reps, dt = timed_reps(run, budget_s)
        return {"value": 2.0 * S ** 3 * reps / dt / cls.scale, "unit": cls.unit, "cores": cores,
                "kind": kind, "sample": f"{reps} x the full {S}^3 GEMM in {dt:.1f} s; {what}"}


class AttentionWorkload:
    name = "fa2_fwd"
    fused_gather = True
    metric = "fa2_fwd_causal_TFLOPS"
    unit = "TFLOP/s"
    scale = 1e12
    dtype = "bf16"
    bound = "tensor"
    scaling = "strong"

    def __init__(self, dist: Dist, args):
        import torch
        from amp_b200 import attention
        self.torch, self.att, self.dist, self.args = torch, attention, dist, args
        self.B, self.H, self.S, self.D = args.batch, args.heads, args.seq, 128
        p = dist.world
        if (self.B * self.H) % p:
            raise SystemExit("batch*heads must divide over the GPUs")
        self.bh = self.B * self.H // p      # (batch*head) shard of this rank
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(99 + dist.rank)
        shape = (1, self.bh, self.S, self.D)
        self.q = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        self.k = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        self.v = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        self.o = torch.empty_like(self.q)
        self.lse = torch.empty(1, self.bh, self.S, dtype=torch.float32, device=dev)
        self.cfg = attention.AttnCfg(self.bh, self.bh, self.D, True, 0.0)
        # N > 1: the all-gather of O and lse is fused into the attention epilogue
        # (stores into every rank's O over NVLink) unless --gather nccl
        self.peer_o = self.peer_l = self.o_all = None
        if p > 1 and self.fused_gather and args.gather == "peer":
            from amp_b200.collective import CommGroup, PeerBuffer
            cg = CommGroup.current()
            self.peer_o = PeerBuffer(cg, self.B * self.H * self.S, self.D, torch.bfloat16)
            self.peer_l = PeerBuffer(cg, self.B * self.H, self.S, torch.float32,
                                     mailboxes=self.peer_o.mailboxes)
        elif p > 1:
            self.o_all = torch.empty(p, self.bh, self.S, self.D, dtype=torch.bfloat16, device=dev)

    def units_per_step(self) -> float:
        # causal: 2 matmuls x 2 flop x D per (query, visible key) pair
        return 4.0 * self.bh * self.D * self.S * (self.S + 1) / 2

    def launches_per_step(self) -> int:
        return 1

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        B, H, S, D, p = args.batch, args.heads, args.seq, 128, world
        return {"workload": "flash_attn2_fwd_causal", "batch": B, "heads": H,
                "seq_len": S, "head_dim": D, "dtype": "bf16, fp32 softmax/accumulate",
                "flop_convention": "4*B*H*D*S*(S+1)/2 (visible pairs)",
                "l2": "Q/K/V %d MiB each exceed L2; L2 flushed before every step"
                      % (B * H * S * D * 2 >> 20),
                "parallelism": (f"(batch*head) split over {p} GPUs, all-gather of O and lse fused "
                                "into the attention epilogue (stores into every rank's O over "
                                "NVLink)" if cls.fused_gather and args.gather == "peer" else
                                f"(batch*head) split over {p} GPUs + NCCL all-gather of O")
                if p > 1 else "single"}

    def config(self):
        return self.describe(self.args, self.dist.world, self.dist.rank)

    def kernel_table(self):
        return [("k_flash_fwd<128>", self.units_per_step())]

    def step(self, ev=None):
        if ev: ev[0].record()
        if self.peer_o is not None:
            from amp_b200._lib import call
            call("amp_flash_attn_fwd_allgather_dev", self.q.data_ptr(), self.k.data_ptr(),
                 self.v.data_ptr(), self.peer_o.table.data_ptr(), self.peer_l.table.data_ptr(),
                 self.dist.rank, self.dist.world, self.dist.rank * self.bh,
                 self.peer_o.mailboxes.table.data_ptr(), self.peer_o.mailboxes.next_seq(), 1,
                 self.bh, self.bh, self.S, self.S, self.D, 1, 0.0,
                 self.torch.cuda.current_stream(self.q.device).cuda_stream)
        else:
            self.att.launch_flash_attn_bf16(self.q, self.k, self.v, self.o, self.lse, 1, self.S,
                                            self.S, self.cfg)
        if ev: ev[1].record()
        if self.o_all is not None:
            self.dist.pg.all_gather_into_tensor(self.o_all, self.o[0])

    def close(self):
        for b in (self.peer_l, self.peer_o):
            if b is not None:
                b.close()
        self.peer_l = self.peer_o = None

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        from amp_b200._lib import call
        qh, kh, vh = (t.cpu().pin_memory() for t in (self.q, self.k, self.v))
        oh = torch.empty_like(qh).pin_memory()
        lh = torch.empty(1, self.bh, self.S, dtype=torch.float32).pin_memory()
        fn = lambda: call("amp_user_flash_attn_fwd_bf16", qh.data_ptr(), kh.data_ptr(),
                          vh.data_ptr(), oh.data_ptr(), lh.data_ptr(), 1, self.bh, self.bh,
                          self.S, self.S, self.D, 1, 0.0)
        ms = _e2e_time(torch, fn, steps, warmup)
        n = qh.numel() * 2
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": 3 * n,
                "d2h_bytes_per_step": n + lh.numel() * 4, "api": "amp_user_flash_attn_fwd_bf16"}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        """AMP has no CPU attention path: the fp64 oracle (oracle/attention.py) on
        whole heads of the same configuration, labelled as a port."""
        from oracle import attention as ref
        S, D = args.seq, 128
        rng = np.random.default_rng(0)
        q, k, v = (rng.standard_normal((1, 1, S, D)).astype(np.float32) for _ in range(3))
        run = lambda: ref.flash_attn_fwd(q, k, v, True)
        reps, dt = timed_reps(run, budget_s)
        flops = 4.0 * D * S * (S + 1) / 2 * reps
        return {"value": flops / dt / cls.scale, "unit": cls.unit, "cores": threads,
                "kind": "port",
                "sample": f"{reps} head(s) of S={S}, D={D} in {dt:.1f} s; fp64 numpy oracle "
                          "(the reference has no CPU attention path)"}


class PagedDecodeWorkload:
    """GQA decode over the paged KV cache (B=8, Hq=32, Hkv=8, D=128, ctx ~ U[512,16384],
    16-token pages, seeded random-permutation block table); HBM-bound."""
    name = "paged_decode"
    metric = "paged_gqa_decode_GBps"
    unit = "GB/s"
    scale = 1e9
    dtype = "bf16"
    bound = "hbm"
    scaling = "weak"
    prefill = False

    def __init__(self, dist: Dist, args):
        import torch
        from amp_b200 import paged, workloads as wl
        self.torch, self.paged, self.dist, self.args = torch, paged, dist, args
        self.ctx = self.context_lens(dist.rank)
        bt, self.num_pages = wl.paged_layout(self.ctx, seed=2026 + dist.rank)
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev)
        g.manual_seed(7 + dist.rank)
        self.B, self.Hq, self.Hkv, self.D = wl.PAGED_B, wl.PAGED_HQ, wl.PAGED_HKV, wl.PAGED_D
        shape = (self.num_pages, self.Hkv, wl.PAGE, self.D)
        self.k_pool = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        self.v_pool = torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)
        self.bt_h = torch.from_numpy(bt).pin_memory()
        self.ctx_h = torch.from_numpy(self.ctx).pin_memory()
        self.bt = self.bt_h.to(dev)
        self.ctxd = self.ctx_h.to(dev)
        self.Lq = wl.PAGED_LQ if self.prefill else 1
        qshape = (self.B, self.Hq, self.Lq, self.D) if self.prefill else (self.B, self.Hq, self.D)
        self.q = torch.randn(qshape, generator=g, device=dev).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        self.lse = torch.empty(qshape[:-1], dtype=torch.float32, device=dev)
        self.max_ctx = int(self.ctx.max())
        self.ws = (None if self.prefill else torch.empty(
            paged.decode_workspace_bytes(self.B, self.Hq, self.D, self.max_ctx),
            dtype=torch.uint8, device=dev))

    def units_per_step(self) -> float:
        # K + V of every context token for every kv head, plus q/out/lse/table
        kv = int(self.ctx.sum()) * self.Hkv * self.D * 2 * 2
        return float(kv + 2 * self.q.numel() * 2 + self.lse.numel() * 4 + self.bt.numel() * 4)

    def launches_per_step(self) -> int:
        return 2

    @staticmethod
    def context_lens(rank: int) -> np.ndarray:
        """This rank's seeded context lengths, U[512, 16384] for each of the 8 sequences."""
        from amp_b200 import workloads as wl
        rng = np.random.default_rng(2025 + rank)
        return rng.integers(wl.PAGED_CTX_LO, wl.PAGED_CTX_HI + 1, size=wl.PAGED_B).astype(np.int32)

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        from amp_b200 import workloads as wl
        ctx = cls.context_lens(rank)
        return {"workload": "paged_gqa_decode", "batch": wl.PAGED_B, "q_heads": wl.PAGED_HQ,
                "kv_heads": wl.PAGED_HKV, "head_dim": wl.PAGED_D, "page_tokens": wl.PAGE,
                "context_lens": ctx.tolist(), "total_context": int(ctx.sum()),
                "block_table": "seeded random permutation of the pool",
                "l2": "KV pools exceed L2; L2 flushed before every step",
                "parallelism": "replicas (each rank its own batch)" if world > 1
                else "single"}

    def config(self):
        return self.describe(self.args, self.dist.world, self.dist.rank)

    def kernel_table(self):
        return [("k_paged_decode + k_paged_combine", self.units_per_step())]

    def _launch(self):
        self.paged.paged_attn_decode(self.q, self.k_pool, self.v_pool, self.bt, self.ctxd,
                                     self.max_ctx, out=self.out, lse=self.lse, workspace=self.ws)

    def step(self, ev=None):
        if ev: ev[0].record()
        self._launch()
        if ev: ev[1].record()

    def e2e(self, steps: int, warmup: int):
        """Public Python API with the step's inputs (q, block table, context
        lengths) copied from pinned host memory and the output read back; the KV
        pools are resident cache state."""
        torch = self.torch
        qh = self.q.cpu().pin_memory()
        oh = torch.empty_like(qh).pin_memory()
        dev = self.q.device

        def fn():
            self.q.copy_(qh, non_blocking=True)
            self.bt.copy_(self.bt_h, non_blocking=True)
            self.ctxd.copy_(self.ctx_h, non_blocking=True)
            self._launch()
            oh.copy_(self.out, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
        ms = _e2e_time_stream(torch, fn, steps, warmup)
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms,
                "h2d_bytes_per_step": qh.numel() * 2 + self.bt.numel() * 4 + self.ctx.size * 4,
                "d2h_bytes_per_step": oh.numel() * 2,
                "api": "amp_b200.paged." + ("paged_attn_prefill" if self.prefill
                                            else "paged_attn_decode")}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        """No CPU attention path exists in the reference: the fp64 oracle on one
        sequence of the workload (gather through the block table + attention)."""
        from oracle import attention as ref
        from amp_b200 import workloads as wl
        ctx = np.array([8448], np.int32)   # the mean context of U[512, 16384]
        ctx, bt, npg, kp, vp = wl.paged_inputs(seed=1, B=1, ctx_lens=ctx)
        rng = np.random.default_rng(2)
        Lq = wl.PAGED_LQ if cls.prefill else 1
        q = rng.standard_normal((1, wl.PAGED_HQ, Lq, wl.PAGED_D)).astype(np.float32)

        def run():
            k = ref.paged_gather(kp, bt[0], int(ctx[0]))[None]
            v = ref.paged_gather(vp, bt[0], int(ctx[0]))[None]
            ref.flash_attn_fwd(q, k, v, causal=cls.prefill, causal_offset=int(ctx[0]) - Lq)
        reps, dt = timed_reps(run, budget_s)
        if cls.prefill:
            units = 4.0 * wl.PAGED_HQ * wl.PAGED_D * sum(int(ctx[0]) - Lq + i + 1
                                                         for i in range(Lq))
        else:
            units = float(int(ctx[0]) * wl.PAGED_HKV * wl.PAGED_D * 4)
        return {"value": units * reps / dt / cls.scale, "unit": cls.unit, "cores": threads,
                "kind": "port",
                "sample": f"{reps} sequence(s) of context {int(ctx[0])} in {dt:.1f} s; fp64 "
                          "numpy oracle (the reference has no attention kernel for block tables)"}


class PagedPrefillWorkload(PagedDecodeWorkload):
    """The last 512 tokens of every context as a paged prefill (bottom-right causal)."""
    name = "paged_prefill"
    metric = "paged_gqa_prefill_TFLOPS"
    unit = "TFLOP/s"
    scale = 1e12
    bound = "tensor"
    prefill = True

    def units_per_step(self) -> float:
        Lq = self.Lq
        pairs = sum(Lq * (int(c) - Lq) + Lq * (Lq + 1) // 2 for c in self.ctx)
        return 4.0 * self.Hq * self.D * pairs

    def launches_per_step(self) -> int:
        return 1

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        from amp_b200 import workloads as wl
        c = super().describe(args, world, rank)
        c.update({"workload": "paged_gqa_prefill", "new_tokens_per_seq": wl.PAGED_LQ,
                  "flop_convention": "4*Hq*D*sum(visible (query, key) pairs)"})
        return c

    def kernel_table(self):
        return [("k_flash_fwd<128, paged>", self.units_per_step())]

    def _launch(self):
        self.paged.paged_attn_prefill(self.q, self.k_pool, self.v_pool, self.bt, self.ctxd,
                                      out=self.out, lse=self.lse)


class AttentionBwdWorkload(AttentionWorkload):
    """FA2 backward (dQ, dK, dV from the forward's O and lse) on the same causal
    configuration; FLOPs by the usual convention of 2.5x the forward (five
    S x S x D products), although the two-pass kernels recompute P and dP."""
    name = "fa2_bwd"
    metric = "fa2_bwd_causal_TFLOPS"
    fused_gather = False

    def __init__(self, dist: Dist, args):
        super().__init__(dist, args)
        torch = self.torch
        from amp_b200._lib import lib
        g = torch.Generator(device=self.q.device)
        g.manual_seed(199 + dist.rank)
        self.do = torch.randn(self.q.shape, generator=g, device=self.q.device).to(torch.bfloat16)
        self.att.launch_flash_attn_bf16(self.q, self.k, self.v, self.o, self.lse, 1, self.S,
                                        self.S, self.cfg)
        self.dq, self.dk, self.dv = (torch.empty_like(self.q) for _ in range(3))
        self.ws = torch.empty(int(lib().amp_flash_attn_bwd_workspace_bytes(1, self.bh, self.S)),
                              dtype=torch.uint8, device=self.q.device)

    def units_per_step(self) -> float:
        return 2.5 * super().units_per_step()

    def launches_per_step(self) -> int:
        return 3

    @classmethod
    def describe(cls, args, world: int, rank: int = 0) -> dict:
        c = super().describe(args, world, rank)
        c["workload"] = "flash_attn2_bwd_causal"
        c["flop_convention"] = "2.5 x 4*B*H*D*S*(S+1)/2 (five products over the visible pairs)"
        c["parallelism"] = "single" if world == 1 else f"(batch*head) split over {world} GPUs"
        return c

    def kernel_table(self):
        return [("k_fa_bwd_delta + k_fa_bwd_dkdv + k_fa_bwd_dq", self.units_per_step())]

    def _call(self, q, k, v, o, do, lse, dq, dk, dv):
        from amp_b200._lib import call
        call("amp_flash_attn_bwd_bf16_dev", q.data_ptr(), k.data_ptr(), v.data_ptr(),
             o.data_ptr(), do.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
             dv.data_ptr(), 1, self.bh, self.bh, self.S, self.S, self.D, 1, 0.0,
             self.ws.data_ptr(), self.ws.numel(),
             self.torch.cuda.current_stream(q.device).cuda_stream)

    def step(self, ev=None):
        if ev: ev[0].record()
        self._call(self.q, self.k, self.v, self.o, self.do, self.lse, self.dq, self.dk, self.dv)
        if ev: ev[1].record()

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        hs = [t.cpu().pin_memory() for t in (self.q, self.k, self.v, self.o, self.do, self.lse)]
        outs = [torch.empty_like(t).pin_memory() for t in hs[:3]]
        dev = [torch.empty_like(t) for t in (self.q, self.k, self.v, self.o, self.do, self.lse)]
        grads = [torch.empty_like(self.q) for _ in range(3)]

        def fn():
            for d, h in zip(dev, hs):
                d.copy_(h, non_blocking=True)
            self._call(*dev, *grads)
            for h, d in zip(outs, grads):
                h.copy_(d, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        ms = _e2e_time(torch, fn, steps, warmup)
        h2d = sum(t.numel() * t.element_size() for t in hs)
        d2h = sum(t.numel() * t.element_size() for t in outs)
        return {"value": self.units_per_step() / (ms * 1e-3) / self.scale, "unit": self.unit,
                "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "amp_flash_attn_bwd_bf16_dev (host tensors copied in and out)"}

    @classmethod
    def cpu_reference(cls, args, budget_s: float, threads: int):
        """No CPU backward exists in AMP: the fp64 chain-rule oracle on one head."""
        from oracle import attention as ref
        S, D = args.seq, 128
        rng = np.random.default_rng(0)
        q, k, v, do = (rng.standard_normal((1, 1, S, D)).astype(np.float32) for _ in range(4))
        run = lambda: ref.flash_attn_bwd(q, k, v, do, True)
        reps, dt = timed_reps(run, budget_s)
        flops = 2.5 * 4.0 * D * S * (S + 1) / 2 * reps
        return {"value": flops / dt / cls.scale, "unit": cls.unit, "cores": threads,
                "kind": "port",
                "sample": f"{reps} head(s) of S={S}, D={D} in {dt:.1f} s; fp64 numpy oracle "
                          "(the reference has no backward)"}


WORKLOADS = {w.name: w for w in (QuantWorkload, GemmWorkload, GemmFp8Workload,
                                 AttentionWorkload, AttentionBwdWorkload, PagedDecodeWorkload,
                                 PagedPrefillWorkload, GemmFp32Workload)}
# The default run: the headline (the FP8 quantiser configuration) and then, in
# the same process and JSON line, every other workload of the measured configs.
HEADLINE = "fp8_quant"
SUITE = ("gemm_bf16", "gemm_fp8", "fa2_fwd", "paged_decode", "paged_prefill", "gemm_fp32",
         "fa2_bwd")


def _e2e_time_stream(torch, fn, steps, warmup):
    """Like _e2e_time, for callables that enqueue on torch's current stream."""
    for _ in range(warmup):
        fn()
    st = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        s.record(st)
        fn()
        e.record(st)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return sum(times) / len(times)


def _e2e_time(torch, fn, steps, warmup):
    for _ in range(warmup):
        fn()
    legacy = torch.cuda.default_stream()  # the host-pointer entry points use stream 0
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        s.record(legacy)
        fn()
        e.record(legacy)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return sum(times) / len(times)


def library_bar(W, flush, reps: int = 10, interleave: bool = True):
    """The vendor library's GEMM on the same square shape, timed here in the
    same process (L2 flushed before each launch): torch.matmul (cuBLAS) for
    bf16, torch._scaled_mm with per-tensor scales (cuBLASLt FP8, the call AMP's
    VendorGemm makes, src/gemm_vendor.cpp:226-230) for E4M3.  With `interleave`
    (one GPU) the library's launches alternate with this kernel's, so the two
    means see the same clocks and power state -- these GEMMs run at the 1 kW
    cap, where back-to-back blocks of launches do not.  A measurement bar only;
    nothing of it is on the product path."""
    import torch
    S = W.S
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    a = torch.randn(S, S, generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn(S, S, generator=g, device=dev).to(torch.bfloat16)
    if W.fp8:
        a8 = a.to(torch.float8_e4m3fn)
        b8 = b.t().contiguous().to(torch.float8_e4m3fn).t()   # column-major B, as cuBLASLt wants
        one = torch.ones((), device=dev)
        fn = lambda: torch._scaled_mm(a8, b8, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        what = "cuBLASLt FP8 E4M3 (torch._scaled_mm, per-tensor scales, bf16 out)"
    else:
        fn = lambda: torch.matmul(a, b)
        what = "cuBLAS bf16 (torch.matmul)"

    def timed(f):
        flush()
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        f()
        e0.record()
        e0.synchronize()
        return s0.elapsed_time(e0)
    for _ in range(3):
        fn()
    lib_ms, ours_ms = [], []
    for _ in range(reps):
        lib_ms.append(timed(fn))
        if interleave:
            ours_ms.append(timed(W._launch))
    rate = lambda ms: round(2.0 * S ** 3 / (ms * 1e-3) / 1e12, 1)
    out = {"kernel": what, "shape": [S, S, S], "value": rate(min(lib_ms)),
           "mean": rate(statistics.mean(lib_ms)), "unit": "TFLOP/s",
           "timing": f"value: best of {reps}, mean: their mean; L2 flushed before each"}
    if interleave:
        # this kernel at the same shape, launch for launch beside the library's
        units = 2.0 * S * S * W.Np
        out["ours_interleaved_mean"] = round(units / (statistics.mean(ours_ms) * 1e-3) / 1e12, 1)
        out["ratio_interleaved"] = round(statistics.mean(lib_ms) / statistics.mean(ours_ms)
                                         * (units / (2.0 * S ** 3)), 4)
    return out


def peak_for(W, peaks, live=None):
    """(peak, unit, source) for the roofline of workload W."""
    live = live or {}
    if W.bound == "hbm":
        return peaks["hbm_gbs"], "GB/s", "MEASURED_PEAKS.json hbm_gbs"
    if W.bound == "fp32":
        return (live["fp32_nominal"], "TFLOP/s",
                "nominal FP32 FFMA rate (SMs x 128 lanes x 2 FLOP x max SM clock); no measured "
                "figure exists for the FP32 pipe; the exact form issues FMUL + FADD, so its own "
                "ceiling is half of this")
    bf16 = peaks["bf16_tflops"]
    if getattr(W, "fp8", False):
        if live.get("fp8_library"):
            return (live["fp8_library"], "TFLOP/s",
                    "measured here: cuBLASLt FP8 E4M3 GEMM at the same shape, same run "
                    "(library_bar)")
        return 2 * bf16, "TFLOP/s", "2 x MEASURED_PEAKS.json bf16_tflops (dense FP8 = 2x bf16)"
    return bf16, "TFLOP/s", "MEASURED_PEAKS.json bf16_tflops (burst)"


def make_flush():
    """L2 flush between steps (outside the timed events): write 256 MiB, then
    read 1 GiB (8x L2) so that the flush's own dirty lines are written back
    before the step starts instead of during it.  (Measured: a read of only
    256 MiB after the write left enough dirty lines behind to add 2.7 us of
    write-back to the next 52 us quantise; reads of 1 GiB or more, with or
    without the write, all give the same step time.)"""
    import torch
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    flush_r = torch.ones(1 << 28, dtype=torch.int32, device="cuda")

    def flush():
        flush_w.zero_()
        torch.amax(flush_r)   # a plain read of all 1 GiB (no widened temporary)
    return flush


def measure(W, args, dist: Dist, flush, steps: int, warmup: int, cpu_budget_s: float) -> dict:
    """One workload's full record: device-timed value, per-kernel roofline,
    clocks during the timed region, e2e through the host-pointer API and (rank
    0 at N = 1) the CPU baseline."""
    import torch
    for _ in range(warmup):
        flush()
        W.step()
    nk = len(W.kernel_table())
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(steps)]
    sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    # A GPU-side pause (~1 ms a step, at most 200 ms; outside the events) lets the
    # host queue the steps ahead of the GPU, so the events time GPU execution and
    # not the pace at which each rank's Python enqueues: at N > 1 the steps are
    # coupled by their exchanges, and one rank's host jitter would stall them all.
    if hasattr(torch.cuda, "_sleep"):
        torch.cuda._sleep(int(2e6) * min(steps, 200))
    phys = os.environ.get("CUDA_VISIBLE_DEVICES")
    dev_index = torch.cuda.current_device()
    nvml_index = int(phys.split(",")[dev_index]) if phys else dev_index
    with ClockSampler(nvml_index) as clocks:
        for i in range(steps):
            flush()
            sev[i][0].record()
            W.step(ev[i])
            sev[i][1].record()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    from amp_b200._lib import lib
    if lib().amp_device_status(1) != 0:
        raise SystemExit(f"{W.name}: a kernel reported a device-side timeout in the timed region")
    total_ms = dist.max(sum(a.elapsed_time(b) for a, b in sev))
    ms_per_step = total_ms / steps
    value = W.units_per_step() * dist.world / (ms_per_step * 1e-3) / W.scale

    spans = []
    for k, (kname, units) in enumerate(W.kernel_table()):
        ms = statistics.mean(ev[i][k].elapsed_time(ev[i][k + 1]) for i in range(steps))
        spans.append((ms, kname, units))
    spans.sort(reverse=True)
    dom_ms, dom_name, dom_units = spans[0]
    csum = clocks.summary()
    live = {}
    bar = None
    if isinstance(W, GemmWorkload):
        bar = library_bar(W, flush, interleave=dist.world == 1)
        if W.fp8:
            live["fp8_library"] = bar["value"]
    if W.bound == "fp32":
        sms = torch.cuda.get_device_properties(dev_index).multi_processor_count
        live["fp32_nominal"] = sms * 128 * 2 * (csum["sm_max_mhz"] or 1965) * 1e6 / 1e12
    peaks, peak_src = load_peaks()
    peak, punit, pkey = peak_for(W, peaks, live)
    achieved = dom_units / (dom_ms * 1e-3) / W.scale
    roofline = {"bound": W.bound, "kernel": dom_name, "achieved": round(achieved, 2),
                "peak": round(peak, 1), "unit": punit, "frac": round(achieved / peak, 4),
                "peak_source": pkey if peak_src == "measured" or "MEASURED" not in pkey
                else "fallback figure of the profiling recipe",
                "traffic": traffic_for(W, dist.world, dom_name),
                "algorithmic_units_per_launch": dom_units, "kernel_ms": round(dom_ms, 5),
                "all_kernels": [{"kernel": n, "ms": round(m, 5),
                                 "rate": round(u / (m * 1e-3) / W.scale, 2)}
                                for m, n, u in spans]}
    if getattr(W, "fp8", False) and live.get("fp8_library"):
        roofline["frac_of_2x_bf16_peak"] = round(achieved / (2 * peaks["bf16_tflops"]), 4)
    e2e = None
    if not args.skip_e2e:
        e2e = W.e2e(max(3, min(steps, 10)), 2)
        e2e["ms_per_step"] = dist.max(e2e["ms_per_step"])  # every rank runs it on its shard
        e2e["value"] = W.units_per_step() * dist.world / (e2e["ms_per_step"] * 1e-3) / W.scale
        if "pageable" in e2e:
            pg = e2e["pageable"]
            pg["ms_per_step"] = dist.max(pg["ms_per_step"])
            pg["value"] = W.units_per_step() * dist.world / (pg["ms_per_step"] * 1e-3) / W.scale
    out = {
        "metric": W.metric, "value": round(value, 3), "unit": W.unit, "n_gpus": dist.world,
        "steps": steps, "warmup": warmup, "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True, "scaling": W.scaling, "vs_baseline": None,
        "dtype": W.dtype, "data": "synthetic (seeded)", "config": W.config(),
        "impl": "amp_b200", "gpu_launches": W.launches_per_step() * steps,
        "clocks": csum, "roofline": roofline,
        "e2e": _round(e2e) if e2e else None,
    }
    if bar is not None:
        # this kernel's mean launch in the timed region against the library's mean launch
        bar["ratio"] = round(achieved / bar["mean"], 4)
        out["library_bar"] = bar
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = W.cpu_reference(args, budget_s=cpu_budget_s,
                                              threads=host_threads())
    return out


def _round(d):
    return {k: (round(v, 4) if isinstance(v, float) else _round(v) if isinstance(v, dict) else v)
            for k, v in d.items()}


def run_one(name, args, dist: Dist, flush, steps, warmup, cpu_budget_s):
    import torch
    W = WORKLOADS[name](dist, args)
    try:
        return measure(W, args, dist, flush, steps, warmup, cpu_budget_s)
    finally:
        if hasattr(W, "close"):
            W.close()   # collective: every rank releases its peer resources here
        del W
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def run_amp(args, dist: Dist):
    import torch
    import amp_b200
    from amp_b200 import build as ampbuild
    if not amp_b200.LIB_PATH.exists():
        ampbuild.build()
    torch.cuda.set_device(dist.local_rank)
    flush = make_flush()
    if args.workload != "suite":
        return run_one(args.workload, args, dist, flush, args.steps, args.warmup, 10.0)
    out = run_one(HEADLINE, args, dist, flush, args.steps, args.warmup, 10.0)
    # the other workloads at the same warm-up and (capped) step count
    steps = min(args.steps, args.suite_steps)
    out["workloads"] = [run_one(n, args, dist, flush, steps, args.warmup, 4.0) for n in SUITE]
    return out


def run_reference(args):
    """The reference's own CPU code for the workload (the headline's for the
    suite), on this host (rank 0 only)."""
    W = WORKLOADS[HEADLINE if args.workload == "suite" else args.workload]
    threads = host_threads()
    # each step is one bounded sample of the workload (about a second of CPU work)
    for _ in range(args.warmup):
        W.cpu_reference(args, budget_s=0.0, threads=threads)
    vals = [W.cpu_reference(args, budget_s=1.0, threads=threads) for _ in range(args.steps)]
    v = statistics.mean(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = round(v, 4)
    return {
        "metric": W.metric, "value": round(v, 4), "unit": W.unit,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": W.scaling,
        "vs_baseline": None, "dtype": W.dtype, "data": "synthetic (seeded)",
        "config": W.describe(args, int(os.environ.get("WORLD_SIZE", "1"))),
        "impl": "reference", "cpu_baseline": cb,
        "e2e": {"value": round(v, 4), "unit": W.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--workload", choices=["suite"] + sorted(WORKLOADS), default="suite",
                    help="suite (default): the headline fp8_quant line with every other "
                         "workload in its 'workloads' array; or one workload alone")
    ap.add_argument("--impl", choices=["amp_b200", "reference"], default="amp_b200")
    ap.add_argument("--elements", type=int, default=1 << 26)
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--fp32-size", type=int, default=1024)
    ap.add_argument("--suite-steps", type=int, default=200,
                    help="cap on the timed steps of the suite's non-headline workloads")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="N>1 GEMM: all-gather fused into the epilogue (peer) or NCCL after it")
    return ap


def main():
    args = build_parser().parse_args()
    if args.impl == "reference":
        args.steps = args.steps or 5
        args.warmup = args.warmup if args.warmup is not None else 3
    else:
        heavy = args.workload not in ("fp8_quant", "suite")
        args.steps = args.steps or (200 if heavy else 2000)
        args.warmup = args.warmup if args.warmup is not None else (10 if heavy else 20)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return  # only rank 0 runs the CPU arm; the others exit without work
        print(json.dumps(run_reference(args)), flush=True)
        return
    dist = Dist(args.gpus)
    try:
        out = run_amp(args, dist)
        if dist.rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
