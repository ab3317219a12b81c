"""bench.py's command-line contract, on the CPU: the reference arm's JSON line, rank handling under
a two-rank launch, the warm-up floor, the gloo control plane, and our arm refusing to run without a
GPU (no fallback); on a GPU, our arm's full line with its sub-records."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    full_env = dict(os.environ)
    full_env.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=full_env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line() -> None:
    out = run_bench("--impl", "reference", "--steps", "2", "--warmup", "3")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [line for line in out.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["metric"] == "add+RMSNorm achieved HBM GB/s" and d["unit"] == "GB/s" and d["higher_is_better"]
    assert d["value"] > 0 and "workload" in d["config"]
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work() -> None:
    out = run_bench("--impl", "reference", "--gpus", "2", "--steps", "2", "--warmup", "3",
                    env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_warmup_below_three_is_rejected() -> None:
    out = run_bench("--impl", "reference", "--steps", "2", "--warmup", "2")
    assert out.returncode != 0 and "--warmup must be at least 3" in out.stderr


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_our_arm_fails_loudly_without_a_gpu() -> None:
    out = run_bench("--steps", "2", "--warmup", "3")
    assert out.returncode != 0 and out.stdout.strip() == ""
    assert "needs a CUDA device" in out.stderr


@pytest.mark.gpu
def test_our_arm_prints_the_full_contract_line_on_a_gpu() -> None:
    """Our arm on a B200: one JSON line with the roofline, CPU-baseline, end-to-end, launch-count and
    clock keys, the roofline fraction computed from the measured peak, inputs larger than L2."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    out = run_bench("--steps", "20", "--warmup", "3", "--e2e-steps", "5", "--cpu-seconds", "0.5")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [line for line in out.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["metric"] == "add+RMSNorm achieved HBM GB/s" and d["n_gpus"] == 1 and d["steps"] == 20
    assert d["dtype"] == "bf16" and d["config"]["kernel"].startswith("rmsnorm_") and "l2" in d["config"]
    rl = d["roofline"]
    assert rl["bound"] == "hbm" and rl["unit"] == "GB/s" and rl["peak"] > 0
    assert abs(rl["frac"] - rl["achieved"] / rl["peak"]) < 1e-9 and 0.3 < rl["frac"] < 1.2
    assert rl["traffic"] is None or rl["traffic_ratio"] == rl["traffic"] / d["config"]["bytes_per_step_per_rank"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] > 0
    e2e = d["e2e"]
    assert e2e["h2d_bytes_per_step"] == e2e["d2h_bytes_per_step"] == 2048 * 3584 * 2 * 2 and e2e["value"] > 0
    assert d["gpu_launches"] == 20
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])
    # Every launch was queued before the region started, and the host's pace is reported beside it.
    assert d["launch"]["queued_before_start"] and d["launch"]["host_us_per_call"] > 0
    assert d["parity"]["parity_ok"] and d["parity"]["residual_exact"] and d["parity"]["rows_checked"] == 2048
    # The other three workloads, measured in the same run and checked against the oracle.
    for key, kernel_prefix in (("sharded", "rmsnorm_stash_kernel"), ("misaligned", "rmsnorm_shifted_"),
                               ("silu", "silu_wave_kernel")):
        sub = d[key]
        assert sub["kernel"].startswith(kernel_prefix), (key, sub["kernel"])
        assert sub["parity"]["parity_ok"] and sub["parity"]["parity_ok_all_ranks"], (key, sub["parity"])
        assert sub["value"] > 0 and 0.1 < sub["roofline_frac"] < 1.3 and sub["launch"]["queued_before_start"]
        cpu = sub["cpu_baseline"]  # the reference's CPU path beside each record
        assert cpu["value"] > 0 and cpu["cores"] >= 1 and cpu["kind"] == "port" and cpu["rows_per_s"] > 0
    assert d["sharded"]["rows_per_rank"] == 262144 and d["sharded"]["parity"]["rows_checked"] >= 64
    assert d["sharded"]["cpu_baseline"]["sample"].startswith("1024 rows")


@pytest.mark.gpu
def test_reference_arm_times_the_reference_kernels_on_this_gpu() -> None:
    """The reference arm on a B200: its CPU line, plus the reference's own kernels compiled for
    sm_100a timed on the four workloads and checked against the oracle (when they were built)."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    out = run_bench("--impl", "reference", "--steps", "5", "--warmup", "3", "--reference-seconds", "2")
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([line for line in out.stdout.splitlines() if line.strip()][-1])
    assert d["impl"] == "reference" and d["value"] > 0
    kernels = d.get("reference_cuda_kernels")
    if kernels is None or "unavailable" in kernels:
        pytest.skip(f"the reference's kernels were not built: {kernels}")
    for key in ("rmsnorm", "misaligned", "sharded", "silu"):
        assert kernels[key]["parity"]["parity_ok"], (key, kernels[key]["parity"])
        assert kernels[key]["value"] > 0
