"""bench.py's host side on CPU: every workload's config is built from the
arguments alone, and the reference arm (the reference's CPU code, no GPU)
prints the JSON line of the contract with the same config as the amp_b200 arm."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

import bench

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
@pytest.mark.parametrize("world", [1, 2, 8])
def test_describe_needs_no_device(name, world):
    W = bench.WORKLOADS[name]
    args = bench.build_parser().parse_args(["--workload", name])
    c = W.describe(args, world)
    json.dumps(c)
    assert c["workload"] and c["parallelism"]
    assert (c["parallelism"] == "single") == (world == 1)


def test_gemm_parallelism_follows_gather_mode():
    args = bench.build_parser().parse_args(["--workload", "gemm_bf16", "--gather", "nccl"])
    assert "NCCL" in bench.GemmWorkload.describe(args, 2)["parallelism"]
    args = bench.build_parser().parse_args(["--workload", "gemm_bf16"])
    assert "fused" in bench.GemmWorkload.describe(args, 2)["parallelism"]


def test_paged_context_lengths_are_seeded_per_rank():
    a, b = bench.PagedDecodeWorkload.context_lens(0), bench.PagedDecodeWorkload.context_lens(0)
    assert (a == b).all() and a.min() >= 512 and a.max() <= 16384 and a.size == 8
    assert (a != bench.PagedDecodeWorkload.context_lens(1)).any()


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, timeout=300, env=env, cwd=ROOT)


def test_reference_arm_json_line(oracle_lib):
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    args = bench.build_parser().parse_args([])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.QuantWorkload.metric and d["unit"] == bench.QuantWorkload.unit
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["config"] == bench.QuantWorkload.describe(args, 1)
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port")
    assert cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"],
             {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_warmup_below_three_is_rejected():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "1"])
    assert r.returncode != 0 and "warmup" in (r.stderr + r.stdout)


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_instance_config_is_describe(name):
    """config() of a set-up workload (here without its device buffers) is describe()."""
    class _Dist:
        world, rank = 2, 0
    W = bench.WORKLOADS[name]
    args = bench.build_parser().parse_args(["--workload", name])
    w = object.__new__(W)
    w.args, w.dist = args, _Dist()
    assert w.config() == W.describe(args, 2)


def test_traffic_is_reported_only_for_the_captured_launch():
    t = bench.load_traffic()
    q = "quantise (k_amax_partials + k_quant_encode)"
    assert bench.traffic_for(bench.QuantWorkload, 1, q) == t["fp8_quant"][q]
    assert bench.traffic_for(bench.QuantWorkload, 8, q) == t["fp8_quant"][q]   # weak scaling
    g = "k_gemm_tc2<bf16>"
    assert bench.traffic_for(bench.GemmWorkload, 1, g) == t["gemm_bf16"][g]
    assert bench.traffic_for(bench.GemmWorkload, 2, g) is None                 # strong scaling
    assert bench.traffic_for(bench.AttentionWorkload, 4, "k_flash_fwd<128>") is None


def test_default_run_is_the_suite_over_every_workload():
    args = bench.build_parser().parse_args([])
    assert args.workload == "suite"
    assert bench.HEADLINE == "fp8_quant" and bench.HEADLINE not in bench.SUITE
    assert set(bench.SUITE) | {bench.HEADLINE} == set(bench.WORKLOADS)


def test_roofline_peaks_name_their_source():
    peaks = {"hbm_gbs": 6550.1, "bf16_tflops": 1662.9}
    p, u, src = bench.peak_for(bench.QuantWorkload, peaks)
    assert (p, u) == (6550.1, "GB/s") and "hbm_gbs" in src
    p, u, src = bench.peak_for(bench.GemmWorkload, peaks)
    assert p == 1662.9 and "bf16_tflops" in src
    p, u, src = bench.peak_for(bench.GemmFp8Workload, peaks, {"fp8_library": 3069.0})
    assert p == 3069.0 and "cuBLASLt" in src
    p, u, src = bench.peak_for(bench.GemmFp8Workload, peaks)
    assert p == 2 * 1662.9
    p, u, src = bench.peak_for(bench.GemmFp32Workload, peaks, {"fp32_nominal": 74.4})
    assert p == 74.4 and "nominal" in src


def test_fp32_gemm_units():
    G = object.__new__(bench.GemmFp32Workload)
    G.S = 1024
    assert G.units_per_step() == 2.0 * 1024 ** 3
