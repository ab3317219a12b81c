"""Benchmark of the fused add+RMSNorm hot path (and SiLU-and-mul) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload rmsnorm|rmsnorm-misaligned|silu|rmsnorm-sharded|rmsnorm-plain|rmsnorm-fp8]
                    [--no-subrecords]

Prints ONE JSON line on rank 0. Under torchrun (N > 1) every rank runs its own GPU; each timed
region is bracketed by a device synchronise and a barrier on both sides, and the elapsed time is
the max over ranks. The ranks' control plane (barriers, max over ranks, the parity verdicts) is a
gloo process group on the host: no NCCL, and no collective on the data path.

A step is one call of the op on one batch already resident in HBM:

* ``rmsnorm`` (default): fused_add_rms_norm on bf16 [2048, 3584], eps 1e-6, x/residual ~ N(0,1),
  weight = 1 + 0.1 N(0,1), seed 0 (+ rank). Every rank processes its own batch (weak scaling).
  The batch is 58.7 MB, below the 126 MB L2, so steps rotate over enough batches (>= 4x L2 in
  total) that each step's inputs are cold in L2.
* ``rmsnorm-misaligned``: the same with x and residual as views 2 bytes off 16-byte alignment.
* ``silu``: silu_and_mul on bf16 [128, 37888] ~ N(0, 2), rotated the same way.
* ``rmsnorm-sharded``: bf16 [262144, 8192], eps 1e-5, rows split across the ranks with no
  collective (strong scaling); each rank generates its shard on its own device from seed + rank.

Unless ``--no-subrecords``, the line for the default workload also carries ``sharded``,
``misaligned`` and ``silu`` records: the other three workloads measured the same way in the same
run, each with its kernel, timings, roofline fraction and an oracle check of its outputs, and on
one GPU the reference's CPU path timed on the same workload (1024 rows of the sharded one).

Timing: W warm-up steps; then, while the device is held by a short sleep kernel (NVBench's
blocking-kernel method), the host enqueues W more warm-up steps, the start event, the K timed
steps and the end event. The timed region is the device running the K launches back to back
right after W launches that bring HBM and L2 to their steady state, not the host's pace of
enqueuing them. The host's cost per call, whether all K launches were queued before the region
started, the same K steps launched just in time (no hold) and a CUDA-graph replay of the same
launches are reported beside it.

Metric: algorithmic HBM bytes per step (add+RMSNorm: 4*H*2 per row = read x, r + write x, r;
weight excluded; SiLU: 6 per output element) over the device time, in GB/s, summed over ranks.
``roofline`` relates the kernel's per-launch time to the measured HBM copy peak and carries the
DRAM traffic per launch measured by ncu (profiles/dram_traffic_per_launch.json);
``cpu_baseline`` is the reference's CPU path (its torch fp32 oracle restated, oracle/oracle.py)
timed on this host; ``e2e`` repeats the metric through the public op with the inputs copied from
pinned host memory and the results copied back inside the timed region.

``--impl reference`` times the reference's CPU path alone (rank 0; other ranks exit) on the same
workload and prints the same metric. When the reference's own CUDA kernels have been built for
sm_100a (oracle/build_ref_kernels.py) and a GPU is present, its line also carries
``reference_cuda_kernels``: those kernels timed the same way on the same workloads, on this box.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO_ROOT / "inference-performance-lab_b200"))

L2_BYTES = 126 * 1024 * 1024
MEASURED_PEAKS = REPO_ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = REPO_ROOT / "profiles" / "dram_traffic_per_launch.json"
FALLBACK_HBM_GBS = 6650.0
# Device clock used to size the hold (cycles of torch.cuda._sleep): at or above the B200's
# 1965 MHz maximum, so that the hold lasts at least as long as asked.
HOLD_CLOCK_GHZ = 2.0

WORKLOADS = {
    "rmsnorm": {"op": "fused_add_rms_norm", "rows": 2048, "hidden": 3584, "eps": 1e-6, "offset": 0},
    "rmsnorm-misaligned": {"op": "fused_add_rms_norm", "rows": 2048, "hidden": 3584, "eps": 1e-6, "offset": 1},
    "rmsnorm-sharded": {"op": "fused_add_rms_norm", "rows": 262144, "hidden": 8192, "eps": 1e-5, "offset": 0,
                        "sharded": True},
    "silu": {"op": "silu_and_mul", "rows": 128, "intermediate": 18944, "std": 2.0},
    "rmsnorm-plain": {"op": "rms_norm", "rows": 2048, "hidden": 3584, "eps": 1e-6, "offset": 0},
    "rmsnorm-fp8": {"op": "fused_add_rms_norm_static_fp8_quant", "rows": 2048, "hidden": 3584, "eps": 1e-6,
                    "offset": 0},
}
# Records added to the default workload's line: name -> workload.
SUBRECORDS = {"sharded": "rmsnorm-sharded", "misaligned": "rmsnorm-misaligned", "silu": "silu"}
# Rows of a batch checked against the oracle: every row up to this many, else a sample of at least
# 64 rows that includes the first and the last.
CHECK_ALL_ROWS = 4096
CHECK_SAMPLE_ROWS = 64


def workload_name(spec) -> str:
    if spec["op"] == "rms_norm":
        return f"rms_norm bf16 [{spec['rows']}, {spec['hidden']}] eps {spec['eps']:g} (out of place)"
    if spec["op"] == "fused_add_rms_norm_static_fp8_quant":
        return (f"fused_add_rms_norm_static_fp8_quant bf16 [{spec['rows']}, {spec['hidden']}] -> e4m3, "
                f"eps {spec['eps']:g}")
    if spec["op"] == "silu_and_mul":
        return f"silu_and_mul bf16 [{spec['rows']}, {2 * spec['intermediate']}] -> [{spec['rows']}, {spec['intermediate']}]"
    name = f"fused_add_rms_norm bf16 [{spec['rows']}, {spec['hidden']}] eps {spec['eps']:g}"
    if spec.get("offset"):
        name += f", x/residual offset {2 * spec['offset']} bytes from 16-byte alignment"
    if spec.get("sharded"):
        name += ", rows sharded across ranks"
    return name


def step_bytes(spec, rows: int) -> int:
    """Algorithmic DRAM bytes of one step: every input element read once, every output written once
    (the weight, read once per SM, is not counted)."""
    if spec["op"] == "silu_and_mul":
        return 6 * rows * spec["intermediate"]
    if spec["op"] == "rms_norm":
        return 2 * spec["hidden"] * 2 * rows  # read x, write out
    if spec["op"] == "fused_add_rms_norm_static_fp8_quant":
        return 7 * spec["hidden"] * rows  # read x, r (4 B), write r (2 B), write e4m3 (1 B)
    return 4 * spec["hidden"] * 2 * rows


def load_peak() -> tuple[float, str]:
    try:
        peaks = json.loads(MEASURED_PEAKS.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(workload: str) -> dict | None:
    """ncu's DRAM bytes per launch of this workload's kernel (steady state: the mean over
    back-to-back launches after the first, each launch's write-back of its predecessor's
    outputs included), with the command that measured it."""
    try:
        table = json.loads(TRAFFIC_FILE.read_text())
    except (OSError, ValueError):
        return None
    entry = table.get("workloads", {}).get(workload)
    return entry if isinstance(entry, dict) else None


# ------------------------------------------------------------------------------------------
# clocks (NVML) sampled during the timed region


class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int) -> None:
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self.error = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            handle = None
            try:
                import torch

                props = torch.cuda.get_device_properties(device_index)
                handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{props.uuid}")
            except Exception:
                visible = os.environ.get("CUDA_VISIBLE_DEVICES")
                index = int(visible.split(",")[device_index]) if visible else device_index
                handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._handle = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # NVML missing: report, do not fail the bench
            self.error = f"{type(exc).__name__}: {exc}"
            self._nvml = None

    def _sample(self) -> None:
        nv = self._nvml
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
        try:
            self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        except AttributeError:
            self.reasons |= nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._handle)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception as exc:
                self.error = f"{type(exc).__name__}: {exc}"
                return
            time.sleep(0.002)

    def __enter__(self):
        self._stop.clear()
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
            self._thread = None
            try:
                self._sample()  # one sample after the region ends, so that short regions have one
            except Exception:
                pass

    def summary(self) -> dict:
        reasons = [name for bit, name in self.REASONS.items() if self.reasons & bit and name != "gpu_idle"]
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(self.samples),
            **({"error": self.error} if self.error else {}),
        }


# ------------------------------------------------------------------------------------------
# distributed plumbing: a gloo group on the host (barriers, max over ranks, verdicts)


class Dist:
    def __init__(self, timeout_s: float = 300.0, single: bool = False) -> None:
        # The timeout bounds every collective: a rank that failed or left ends the others' next
        # barrier with an error instead of a hang (300 s covers a fresh box's first torch import).
        self.world = 1 if single else int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = 0 if single else int(os.environ.get("RANK", "0"))
        self.local_rank = 0 if single else int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
            self.pg = dist

    def barrier(self) -> None:
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def all(self, flag: bool) -> bool:
        if self.pg is None:
            return bool(flag)
        import torch

        t = torch.tensor([1 if flag else 0], dtype=torch.int64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MIN)
        return bool(t.item())

    def gather(self, value) -> list:
        if self.pg is None:
            return [value]
        out = [None] * self.world
        self.pg.all_gather_object(out, value)
        return out

    def close(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()


# ------------------------------------------------------------------------------------------
# per-op workload: inputs, the call, the oracle check, host buffers for the e2e leg


class OpWorkload:
    """Everything op-specific: device batches, the op call, its kernel plan, the check of one call
    against the oracle, the reference's CPU call on a sample, and which tensors an end-to-end step
    uploads and downloads."""

    def __init__(self, spec, namespace: str = "inference_performance_lab") -> None:
        self.spec = spec
        self.op = spec["op"]
        self.namespace = namespace

    def make_sets(self, rows: int, seed: int, device, sets: int):
        """`sets` batches (dicts of device tensors) and the tensors they share (weight, scale)."""
        import torch

        spec = self.spec
        generator = torch.Generator(device=device).manual_seed(seed)
        batches = []
        if self.op == "silu_and_mul":
            inter = spec["intermediate"]
            for _ in range(sets):
                x = (torch.randn(rows, 2 * inter, device=device, generator=generator) * spec["std"]).to(torch.bfloat16)
                batches.append({"x": x, "out": torch.empty(rows, inter, device=device, dtype=torch.bfloat16)})
            return batches, {}
        hidden, offset = spec["hidden"], spec.get("offset", 0)

        def row_view(buf):
            return buf[offset: offset + rows * hidden].view(rows, hidden)

        for _ in range(sets):
            batch = {"x": row_view(torch.randn(rows * hidden + 8, device=device, dtype=torch.bfloat16,
                                               generator=generator))}
            if self.op != "rms_norm":
                batch["r"] = row_view(torch.randn(rows * hidden + 8, device=device, dtype=torch.bfloat16,
                                                  generator=generator))
            if self.op == "rms_norm":
                batch["out"] = torch.empty(rows, hidden, device=device, dtype=torch.bfloat16)
            if self.op == "fused_add_rms_norm_static_fp8_quant":
                batch["out"] = torch.empty(rows, hidden, device=device, dtype=torch.float8_e4m3fn)
            batches.append(batch)
        shared = {"w": (torch.randn(hidden, device=device, generator=generator) * 0.1 + 1.0).to(torch.bfloat16)}
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            shared["scale"] = torch.tensor([0.05], dtype=torch.float32, device=device)
        return batches, shared

    def bind(self, batch, shared):
        """A no-argument callable that runs the op on `batch` through the public torch op (bound
        once, so that the timed loop adds no Python work of its own beyond the op call)."""
        import functools

        import torch

        ops = getattr(torch.ops, self.namespace)
        eps = self.spec.get("eps")
        if self.op == "silu_and_mul":
            # The reference's own library has the vectorised kernel under the packed op name only.
            name = "silu_and_mul_packed" if self.namespace != "inference_performance_lab" else "silu_and_mul"
            return functools.partial(getattr(ops, name).default, batch["out"], batch["x"])
        if self.op == "rms_norm":
            return functools.partial(ops.rms_norm.default, batch["out"], batch["x"], shared["w"], eps)
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            return functools.partial(ops.fused_add_rms_norm_static_fp8_quant.default, batch["out"], batch["x"],
                                     batch["r"], shared["w"], shared["scale"], eps)
        return functools.partial(ops.fused_add_rms_norm.default, batch["x"], batch["r"], shared["w"], eps)

    def plan(self, batch, shared, rows: int) -> str:
        from inference_performance_lab.kernels import capi

        if self.op == "silu_and_mul":
            return capi.silu_and_mul_plan(batch["out"].data_ptr(), batch["x"].data_ptr(), rows,
                                          self.spec["intermediate"])
        hidden, w = self.spec["hidden"], shared["w"].data_ptr()
        if self.op == "rms_norm":
            return capi.rms_norm_plan(batch["out"].data_ptr(), batch["x"].data_ptr(), w, rows, hidden)
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            return capi.fused_add_rms_norm_static_fp8_quant_plan(
                batch["out"].data_ptr(), batch["x"].data_ptr(), batch["r"].data_ptr(), w, rows, hidden)
        return capi.fused_add_rms_norm_plan(batch["x"].data_ptr(), batch["r"].data_ptr(), w, rows, hidden)

    def check(self, batch, shared, rows: int) -> dict:
        """One op call on `batch` (fresh inputs), with its rows compared against the C oracle: every
        row up to CHECK_ALL_ROWS rows, else CHECK_SAMPLE_ROWS spread over the batch including the
        first and last. Residuals must match bit for bit; bf16 outputs must be within rtol = atol =
        1e-2 and one bf16 ulp of the oracle; e4m3 outputs within one e4m3 step. Outside every timed
        region: the oracle is the checker here, never the thing measured."""
        import numpy as np
        import torch

        from oracle import oracle

        if rows <= CHECK_ALL_ROWS:
            index = list(range(rows))
        else:
            step = (rows - 1) / (CHECK_SAMPLE_ROWS - 1)
            index = sorted({round(i * step) for i in range(CHECK_SAMPLE_ROWS)} | {0, rows - 1})
        idx = torch.tensor(index, dtype=torch.int64, device=batch["x"].device)

        def take(t):
            return t.index_select(0, idx).contiguous()

        before = {k: take(v) for k, v in batch.items() if k in ("x", "r")}
        self.bind(batch, shared)()
        torch.cuda.synchronize()
        result = {"rows_checked": len(index), "residual_exact": None, "max_ulp": None, "max_abs_err": None}

        def compare_bf16(got_t, want_bits) -> bool:
            got = oracle.tensor_bits(got_t)
            g, w = oracle.bf16_bits_to_f32(got), oracle.bf16_bits_to_f32(want_bits)
            finite = np.isfinite(w)
            err = np.abs(g - w)
            result["max_abs_err"] = float(err[finite].max(initial=0.0))
            ordered = [np.where(a.astype(np.int32) & 0x8000, 0x8000 - a.astype(np.int32), a.astype(np.int32))
                       for a in (got, want_bits)]
            result["max_ulp"] = int(np.abs(ordered[0] - ordered[1]).max(initial=0))
            close = np.all((err <= 1e-2 + 1e-2 * np.abs(w)) | ~finite) and np.array_equal(np.isnan(g), np.isnan(w))
            return bool(close) and result["max_ulp"] <= 1

        if self.op == "silu_and_mul":
            want = oracle.c_silu_and_mul(oracle.tensor_bits(before["x"]))
            ok = compare_bf16(take(batch["out"]), want)
        elif self.op == "rms_norm":
            want = oracle.c_rms_norm(oracle.tensor_bits(before["x"]), oracle.tensor_bits(shared["w"]), self.spec["eps"])
            ok = compare_bf16(take(batch["out"]), want)
        elif self.op == "fused_add_rms_norm_static_fp8_quant":
            want8, want_res = oracle.c_fused_add_rms_norm_static_fp8_quant(
                oracle.tensor_bits(before["x"]), oracle.tensor_bits(before["r"]), oracle.tensor_bits(shared["w"]),
                float(shared["scale"].item()), self.spec["eps"])
            result["residual_exact"] = bool(np.array_equal(oracle.tensor_bits(take(batch["r"])), want_res))
            got8 = take(batch["out"]).view(torch.uint8).cpu().numpy().astype(np.int32)
            ordered = [np.where(a & 0x80, 0x80 - a, a) for a in (got8, want8.astype(np.int32))]
            result["max_ulp"] = int(np.abs(ordered[0] - ordered[1]).max(initial=0))
            ok = result["residual_exact"] and result["max_ulp"] <= 1
        else:
            want_out, want_res = oracle.c_fused_add_rms_norm(
                oracle.tensor_bits(before["x"]), oracle.tensor_bits(before["r"]), oracle.tensor_bits(shared["w"]),
                self.spec["eps"])
            result["residual_exact"] = bool(np.array_equal(oracle.tensor_bits(take(batch["r"])), want_res))
            ok = compare_bf16(take(batch["x"]), want_out) and result["residual_exact"]
        result["parity_ok"] = bool(ok)
        return result

    def e2e_inputs(self, batch):
        """Device tensors an end-to-end step fills from pinned host memory."""
        return [batch["x"]] if self.op in ("silu_and_mul", "rms_norm") else [batch["x"], batch["r"]]

    def e2e_outputs(self, batch):
        """Device tensors an end-to-end step reads back into pinned host memory."""
        if self.op == "fused_add_rms_norm":
            return [batch["x"], batch["r"]]
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            return [batch["out"], batch["r"]]
        return [batch["out"]]

    def cpu_call(self, rows: int):
        """The reference's CPU path (its torch fp32 oracle, restated in oracle/) on `rows` rows."""
        import torch

        from oracle import oracle

        spec = self.spec
        generator = torch.Generator().manual_seed(0)
        if self.op == "silu_and_mul":
            x = (torch.randn(rows, 2 * spec["intermediate"], generator=generator) * spec["std"]).to(torch.bfloat16)
            return lambda: oracle.torch_silu_and_mul(x)
        x = torch.randn(rows, spec["hidden"], generator=generator).to(torch.bfloat16)
        r = torch.randn(rows, spec["hidden"], generator=generator).to(torch.bfloat16)
        w = (torch.randn(spec["hidden"], generator=generator) * 0.1 + 1).to(torch.bfloat16)
        eps = spec["eps"]
        if self.op == "rms_norm":
            return lambda: oracle.torch_rms_norm(x, w, eps)
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            return lambda: oracle.torch_fused_add_rms_norm_static_fp8_quant(x, r, w, 0.05, eps)
        return lambda: oracle.torch_fused_add_rms_norm(x, r, w, eps)

    def metric(self) -> str:
        return {
            "silu_and_mul": "SiLU-and-mul achieved GB/s",
            "rms_norm": "RMSNorm achieved HBM GB/s",
            "fused_add_rms_norm_static_fp8_quant": "add+RMSNorm (fp8 out) achieved HBM GB/s",
        }.get(self.op, "add+RMSNorm achieved HBM GB/s")

    def traffic_elems(self, rows: int) -> tuple[int, int]:
        """(bf16 elements read, bf16 elements written) of a torch op with the same DRAM bytes."""
        if self.op == "silu_and_mul":
            return 2 * rows * self.spec["intermediate"], rows * self.spec["intermediate"]
        hidden = self.spec["hidden"]
        if self.op == "rms_norm":
            return rows * hidden, rows * hidden
        if self.op == "fused_add_rms_norm_static_fp8_quant":
            return 2 * rows * hidden, (3 * rows * hidden) // 2
        return 2 * rows * hidden, 2 * rows * hidden


# ------------------------------------------------------------------------------------------
# device timing


def time_calls(calls, steps: int, warmup: int, stream, dist, clocks: ClockSampler | None) -> dict:
    """W warm-up calls, then K calls timed on the device.

    The device is held by a short sleep kernel while the host enqueues W more warm-up calls, the
    start event and the K timed calls (NVBench's blocking-kernel method): the events then bracket
    the device running the K launches back to back, right after W launches that bring the memory
    system to its steady state, and the host's enqueue pace is reported separately
    (``host_us_per_call``). ``queued_before_start`` says whether every timed launch was in the
    queue before the start event fired. The same K calls are then run again without the hold, as
    a caller that launches just in time would: ``unqueued_us_per_step``, and ``idle_us_per_step``,
    the device time per step that the host's pace adds."""
    import torch

    n = len(calls)
    t0 = time.perf_counter()
    for i in range(warmup):
        calls[i % n]()
    host_warm = (time.perf_counter() - t0) / max(warmup, 1)
    pre = [calls[i % n] for i in range(warmup)]
    order = [calls[(warmup + i) % n] for i in range(steps)]
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    hold_s = min(max(50e-6, 2.0 * (steps + warmup) * host_warm + 20e-6), 0.2)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks is not None:
        clocks.__enter__()
    try:
        torch.cuda._sleep(int(hold_s * HOLD_CLOCK_GHZ * 1e9))
        for call in pre:
            call()
        start.record(stream)
        # Host cost per call over the first calls only: a long run fills CUDA's launch queue
        # during the hold, after which enqueuing waits for the device.
        sampled = min(steps, 200)
        h0 = time.perf_counter()
        for call in order[:sampled]:
            call()
        host_s = time.perf_counter() - h0
        for call in order[sampled:]:
            call()
        queued = not start.query()
        end.record(stream)
        end.synchronize()
    finally:
        if clocks is not None:
            clocks.__exit__(None, None, None)
    torch.cuda.synchronize()
    dist.barrier()
    local_ms = start.elapsed_time(end)
    elapsed_ms = dist.max(local_ms)

    # Just in time: the same calls with no hold (the host's pace included).
    torch.cuda.synchronize()
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    u0.record(stream)
    for call in order:
        call()
    u1.record(stream)
    u1.synchronize()
    unqueued_ms = u0.elapsed_time(u1)
    return {
        "local_ms": local_ms,
        "elapsed_ms": elapsed_ms,
        "us_per_step": elapsed_ms / steps * 1e3,
        "host_us_per_call": host_s / sampled * 1e6,
        "queued_before_start": bool(queued),
        "hold_us": hold_s * 1e6,
        "unqueued_us_per_step": unqueued_ms / steps * 1e3,
        "idle_us_per_step": max(0.0, (unqueued_ms - local_ms) / steps * 1e3),
    }


def graph_replay_us(calls, stream) -> float:
    """Per-launch device time of the same launches replayed from a CUDA graph of at least 100 of
    them (launch cost gone), timed on a replay that directly follows an untimed one."""
    import torch

    sets = len(calls)
    graph_steps = max(sets, -(-100 // sets) * sets)
    graph = torch.cuda.CUDAGraph()
    capture_stream = torch.cuda.Stream()
    capture_stream.wait_stream(stream)
    with torch.cuda.stream(capture_stream):
        with torch.cuda.graph(graph, stream=capture_stream):
            for i in range(graph_steps):
                calls[i % sets]()
    stream.wait_stream(capture_stream)
    graph.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graph.replay()
    g0.record(stream)
    graph.replay()
    g1.record(stream)
    g1.synchronize()
    us = g0.elapsed_time(g1) / graph_steps * 1e3
    del graph
    return us


def rotation_sets(per_step: int) -> int:
    """Batches to rotate over so that each step's inputs are cold in L2 (>= 4x L2 in total)."""
    return max(1, math.ceil(4 * L2_BYTES / per_step)) if per_step < 4 * L2_BYTES else 1


def measure_workload(name: str, spec, dist, device, stream, steps: int, warmup: int, *, graph: bool,
                     namespace: str = "inference_performance_lab", with_plan: bool = True) -> dict:
    """Inputs for this rank, one checked call, then the timing of K steps (see time_calls)."""
    import torch

    from inference_performance_lab.kernels.sharding import row_shard, shard_seed

    workload = OpWorkload(spec, namespace)
    if spec.get("sharded"):
        shard = row_shard(spec["rows"], dist.world, dist.rank)
        rows, total_rows = shard.rows, spec["rows"]
    else:
        rows, total_rows = spec["rows"], spec["rows"] * dist.world
    per_step = step_bytes(spec, rows)
    sets = rotation_sets(per_step)
    batches, shared = workload.make_sets(rows, shard_seed(0, dist.rank), device, sets)
    parity = workload.check(batches[0], shared, rows)
    calls = [workload.bind(batch, shared) for batch in batches]
    clocks = ClockSampler(dist.local_rank)
    timing = time_calls(calls, steps, warmup, stream, dist, clocks)
    graph_us = graph_replay_us(calls, stream) if graph else None
    kernel = workload.plan(batches[0], shared, rows) if with_plan else None
    peak, peak_kind = load_peak()
    local_us = timing["local_ms"] / steps * 1e3
    total_bytes = step_bytes(spec, total_rows)
    clock_summary = clocks.summary()
    result = {
        "workload": workload_name(spec),
        "metric": workload.metric(),
        "rows_per_rank": rows,
        "bytes_per_step_per_rank": per_step,
        "l2": (f"inputs rotate over {sets} batches ({sets * per_step / 1e6:.0f} MB per rank, > 4x the 126 MB L2)"
               if sets > 1 else "inputs larger than the 126 MB L2"),
        "kernel": kernel,
        "steps": steps,
        "warmup": warmup,
        "value": total_bytes / (timing["us_per_step"] * 1e-6) / 1e9,
        "unit": "GB/s",
        "rows_per_s": total_rows / (timing["us_per_step"] * 1e-6),
        "us_per_step": timing["us_per_step"],
        "roofline_frac": per_step / (local_us * 1e-6) / 1e9 / peak,
        "graph_replay_us_per_launch": graph_us,
        "graph_replay_frac": (per_step / (graph_us * 1e-6) / 1e9 / peak) if graph_us else None,
        "launch": {k: timing[k] for k in ("host_us_per_call", "queued_before_start", "hold_us",
                                          "unqueued_us_per_step", "idle_us_per_step")},
        "parity": parity,
        "clocks": clock_summary,
        # Device time per step times the median SM clock under load: comparable across boxes
        # whose clocks differ (cycles per step, in microsecond-megahertz).
        "us_x_median_sm_mhz": (timing["us_per_step"] * clock_summary["sm_mhz"]) if clock_summary["sm_mhz"] else None,
        "_local_us": local_us,
        "_peak": (peak, peak_kind),
        "_calls": calls,
        "_batches": batches,
        "_shared": shared,
        "_workload": workload,
        "_rows": rows,
    }
    return result


def public(record: dict) -> dict:
    return {k: v for k, v in record.items() if not k.startswith("_")}


# ------------------------------------------------------------------------------------------
# CPU path of the reference (the oracle's torch restatement of reference.py)


def cpu_reference_rate(spec, seconds: float, sample_rows: int | None = None) -> dict:
    """Times the reference's CPU path on a bounded sample of the workload; GB/s of the metric."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = spec["rows"] if sample_rows is None else sample_rows
    call = OpWorkload(spec).cpu_call(rows)
    call()
    times = []
    start = time.perf_counter()
    while (time.perf_counter() - start < seconds and len(times) < 10000) or len(times) < 3:
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    median = statistics.median(times)
    return {
        "value": step_bytes(spec, rows) / median / 1e9,
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{rows} rows of the workload per call, median of {len(times)} calls "
                  f"({median * 1e3:.2f} ms/call, {rows / median:.0f} rows/s), torch fp32 on CPU",
        "ms_per_call": median * 1e3,
        "rows_per_s": rows / median,
    }


def reference_cuda_kernels(args) -> dict | None:
    """The reference's own CUDA kernels, built for sm_100a from its sources (oracle/_ref), timed on
    this GPU exactly as our arm times ours, on the same workloads, each checked against the oracle.
    None when the library is absent or there is no GPU."""
    import torch

    from oracle import build_ref_kernels

    if not torch.cuda.is_available():
        return None
    if not build_ref_kernels.load():
        return {"unavailable": "oracle/_ref/libref_kernels.so not built (oracle/build_ref_kernels.py)"}
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    dist = Dist(single=True)
    records = {}
    kernels = {
        "rmsnorm": "fused_add_rms_norm_bf16_packed_cached_kernel<3584>",
        "misaligned": "fused_add_rms_norm_bf16_cached_kernel<3584>",
        "silu": "silu_and_mul_bf16_packed_kernel (op silu_and_mul_packed)",
        "sharded": "fused_add_rms_norm_bf16_generic_kernel",
    }
    names = {"rmsnorm": "rmsnorm", **SUBRECORDS}
    with torch.inference_mode():
        for key, workload in names.items():
            spec = dict(WORKLOADS[workload])
            if spec.get("sharded"):
                steps, warmup = min(args.steps, 40), max(3, min(args.warmup, 5))
            else:
                steps, warmup = min(args.steps, 1000), args.warmup
            rec = measure_workload(workload, spec, dist, device, stream, steps, warmup,
                                   graph=not spec.get("sharded"), namespace="inference_performance_lab_ref",
                                   with_plan=False)
            rec["kernel"] = kernels[key]
            records[key] = public(rec)
            del rec
            torch.cuda.empty_cache()
    return {
        "what": "the reference's csrc kernels compiled for sm_100a from its unmodified sources "
                "(oracle/build_ref_kernels.py), run through its own op wrappers on this GPU, timed as our arm",
        **records,
    }


def run_reference(args, spec) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # Size each step's sample so that warm-up + K steps end within the budget (a minute by default).
    probe = cpu_reference_rate(spec, 0.5, sample_rows=min(spec["rows"], 256))
    per_row = probe["ms_per_call"] / 1e3 / min(spec["rows"], 256)
    budget = args.reference_seconds / max(args.steps + args.warmup, 1)
    rows = int(max(1, min(spec["rows"], budget / per_row)))
    workload = OpWorkload(spec)
    call = workload.cpu_call(rows)
    for _ in range(args.warmup):
        call()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call()
    elapsed = time.perf_counter() - t0
    value = step_bytes(spec, rows) * args.steps / elapsed / 1e9
    sample = f"{rows} of {spec['rows']} rows per step, torch fp32 on CPU ({threads} threads)"
    line = {
        "impl": "reference",
        "metric": workload.metric(),
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if spec.get("sharded") else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": workload_name(spec), "rows_per_step": rows},
        "rows_per_s": rows * args.steps / elapsed,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload == "rmsnorm" and not args.no_subrecords:
        try:
            kernels = reference_cuda_kernels(args)
        except Exception as exc:  # the CPU arm's line stands on its own
            kernels = {"unavailable": f"{type(exc).__name__}: {exc}"}
        if kernels is not None:
            line["reference_cuda_kernels"] = kernels
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------
# our implementation


def run_ours(args, spec) -> None:
    import torch

    from inference_performance_lab.kernels import capi, extension

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU fallback)")
    dist = Dist()
    torch.cuda.set_device(dist.local_rank)
    device = torch.device("cuda", dist.local_rank)
    extension.load_extension()
    stream = torch.cuda.current_stream()

    with torch.inference_mode():
        main = measure_workload(args.workload, spec, dist, device, stream, args.steps, args.warmup, graph=True)
        workload, rows = main["_workload"], main["_rows"]
        e2e = run_e2e(args, spec, workload, rows, main["_batches"], main["_shared"], stream, dist)
        same_traffic = copy_same_traffic(workload, rows, device, args.steps)
        for key in [k for k in main if k.startswith("_") and k not in ("_local_us", "_peak", "_rows")]:
            del main[key]
        torch.cuda.empty_cache()

        subrecords = {}
        if args.workload == "rmsnorm" and not args.no_subrecords:
            for key, name in SUBRECORDS.items():
                sub_spec = dict(WORKLOADS[name])
                if sub_spec.get("sharded"):
                    steps, warmup = min(args.steps, 40), max(3, min(args.warmup, 5))
                else:
                    steps, warmup = min(args.steps, 1000), args.warmup
                rec = measure_workload(name, sub_spec, dist, device, stream, steps, warmup,
                                       graph=not sub_spec.get("sharded"))
                rec["parity"]["parity_ok_all_ranks"] = dist.all(rec["parity"]["parity_ok"])
                per_rank = dist.gather({"rank": dist.rank, "us_per_step": rec["_local_us"],
                                        "roofline_frac": rec["roofline_frac"], "rows": rec["rows_per_rank"],
                                        "parity_ok": rec["parity"]["parity_ok"]})
                rec["per_rank"] = per_rank
                traffic = load_traffic(name)
                if traffic is not None:
                    scaled = traffic["bytes_per_launch"] * rec["rows_per_rank"] / traffic["rows"]
                    rec["traffic"] = {"bytes_per_launch": scaled,
                                      "ratio": scaled / rec["bytes_per_step_per_rank"],
                                      "source": traffic["command"]}
                else:
                    rec["traffic"] = None
                # The reference's CPU path beside each record (one GPU only, like the line's own):
                # the full batch, or 1024 rows of the row-sharded workload; a quarter of the time.
                if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
                    rec["cpu_baseline"] = cpu_reference_rate(
                        sub_spec, max(0.5, args.cpu_seconds / 4),
                        sample_rows=1024 if sub_spec.get("sharded") else sub_spec["rows"])
                subrecords[key] = public(rec)
                del rec
                torch.cuda.empty_cache()

    # Every bounded wait of the staged kernel must have completed: a nonzero fault word means a
    # kernel gave up and its outputs are incomplete, so the run is not a measurement.
    fault_flags = int(dist.max(float(capi.device_fault_flags(dist.local_rank))))
    if fault_flags:
        raise SystemExit(f"device fault word {fault_flags:#x}: a kernel gave up on a wait")
    parity_ok = dist.all(main["parity"]["parity_ok"])

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        sample_rows = spec["rows"] if not spec.get("sharded") else 1024
        cpu = cpu_reference_rate(spec, args.cpu_seconds, sample_rows=sample_rows)

    peak, peak_kind = main["_peak"]
    local_us = main["_local_us"]
    per_step = main["bytes_per_step_per_rank"]
    achieved = per_step / (local_us * 1e-6) / 1e9
    traffic = load_traffic(args.workload)
    traffic_bytes = None
    if traffic is not None:
        traffic_bytes = traffic["bytes_per_launch"] * main["rows_per_rank"] / traffic["rows"]
    line = {
        "metric": main["metric"],
        "value": main["value"],
        "unit": "GB/s",
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": main["us_per_step"] / 1e3,
        "higher_is_better": True,
        "scaling": "strong" if spec.get("sharded") else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) inputs on device, the reference's recipe)",
        "config": {
            "workload": main["workload"],
            "rows_per_rank": main["rows_per_rank"],
            "bytes_per_step_per_rank": per_step,
            "l2": main["l2"],
            "kernel": main["kernel"],
            "launch": "K launches enqueued behind a device-side hold before the start event: "
                      "the device runs them back to back",
        },
        "pct_of_peak": 100.0 * achieved / peak,
        "rows_per_s": main["rows_per_s"],
        # The reference's own microbenchmark counts 10 B per add+RMSNorm element (the weight
        # read for every row as well); the same time at that count, for comparison with it.
        "gbs_at_reference_byte_count": (main["value"] * 10 / 8 if spec["op"] == "fused_add_rms_norm" else main["value"]),
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic_bytes,
            "traffic_ratio": (traffic_bytes / per_step) if traffic_bytes else None,
            "traffic_source": traffic["command"] if traffic else None,
            "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback 6.65 TB/s",
            "graph_replay_us_per_launch": main["graph_replay_us_per_launch"],
            "graph_replay_frac": main["graph_replay_frac"],
            "same_traffic_torch_op": same_traffic,
            "frac_of_same_traffic_torch_op": achieved / same_traffic["achieved"],
        },
        "launch": main["launch"],
        "us_x_median_sm_mhz": main["us_x_median_sm_mhz"],
        "parity": {**main["parity"], "parity_ok_all_ranks": parity_ok},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "fault_flags": fault_flags,
        "clocks": main["clocks"],
        **subrecords,
    }
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()
    if not parity_ok:
        raise SystemExit("oracle check of the measured workload failed")


def copy_same_traffic(workload, rows: int, device, steps: int) -> dict:
    """A torch elementwise op moving the same DRAM bytes as one step (an add of two halves when the
    step reads twice what it writes, as SiLU does, else a copy of half the step's bytes), timed
    the same way (back-to-back over rotating buffers > 4x L2, CUDA events): the practical
    bandwidth at this transfer size, beside the large-copy peak."""
    import torch

    read_elems, write_elems = workload.traffic_elems(rows)
    per = 2 * (read_elems + write_elems)
    use_add = read_elems == 2 * write_elems
    n = write_elems if use_add else (read_elems + write_elems) // 2
    sets = rotation_sets(per)
    src = [torch.empty(2 * n if use_add else n, dtype=torch.bfloat16, device=device).normal_() for _ in range(sets)]
    dst = [torch.empty(n, dtype=torch.bfloat16, device=device) for _ in range(sets)]
    if use_add:
        def one(i: int) -> None:
            torch.add(src[i % sets][:n], src[i % sets][n:], out=dst[i % sets])
    else:
        def one(i: int) -> None:
            dst[i % sets].copy_(src[i % sets])
    steps = max(3, min(steps, int(20e9 // per)))
    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        one(i)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) / steps * 1e3
    return {"op": "torch add" if use_add else "torch copy", "us_per_launch": us,
            "achieved": per / (us * 1e-6) / 1e9}


E2E_MIN_WARMUP = 30
E2E_MIN_WARMUP_S = 0.15


def run_e2e(args, spec, workload, rows: int, batches, shared, stream, dist) -> dict:
    """The metric through the public op, with each step's inputs copied from pinned host memory
    and its results copied back inside the timed region.

    Steps are double-buffered across three streams, as a host-fed pipeline would run them: step
    k's upload (pinned host -> set k % 2), its op on the compute stream once uploaded, and its
    download (set k % 2 -> pinned host) once computed; the upload of step k + 2 waits for the
    download of step k, which frees the set. PCIe is full duplex, so step k + 1's upload overlaps
    step k's download."""
    import torch

    per_step = step_bytes(spec, rows)
    # Bounded: a step moves 2x its bytes over PCIe; keep the region to a few seconds.
    steps = max(3, min(args.steps, args.e2e_steps, int(20e9 // per_step)))
    sets = list(batches[:2])
    if len(sets) < 2:
        extra, _ = workload.make_sets(rows, 0x5EED, sets[0]["x"].device, 1)
        sets.append(extra[0])
    if workload.op == "fused_add_rms_norm" and not spec.get("offset"):
        # x and residual of a set side by side in one device buffer (and one pinned host buffer): a
        # step uploads its inputs with one copy and downloads its results with one.
        packed = []
        for b in sets:
            buf = torch.empty(2, rows, spec["hidden"], dtype=torch.bfloat16, device=b["x"].device)
            buf[0].copy_(b["x"])
            buf[1].copy_(b["r"])
            packed.append({"x": buf[0], "r": buf[1], "packed": buf})
        sets = packed
        plan = [([b["packed"]], [b["packed"]], workload.bind(b, shared)) for b in sets]
    else:
        plan = [(workload.e2e_inputs(b), workload.e2e_outputs(b), workload.bind(b, shared)) for b in sets]
    inputs_h = [t.cpu().pin_memory() for t in plan[0][0]]
    # One host destination serves both sets: downloads run in order on one stream.
    outputs_h = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in plan[0][1]]
    h2d = sum(t.numel() * t.element_size() for t in inputs_h)
    d2h = sum(t.numel() * t.element_size() for t in outputs_h)
    upload, download = torch.cuda.Stream(), torch.cuda.Stream()

    def pipeline(n: int, first: "torch.cuda.Event | None" = None) -> "torch.cuda.Event":
        freed = [None, None]  # per set: the event of its last download
        if first is not None:
            first.record(upload)
        for k in range(n):
            ins, outs, call = plan[k % 2]
            if freed[k % 2] is not None:
                upload.wait_event(freed[k % 2])
            with torch.cuda.stream(upload):
                for d, h in zip(ins, inputs_h):
                    d.copy_(h, non_blocking=True)
            uploaded = torch.cuda.Event()
            uploaded.record(upload)
            stream.wait_event(uploaded)
            with torch.cuda.stream(stream):
                call()
            computed = torch.cuda.Event()
            computed.record(stream)
            download.wait_event(computed)
            with torch.cuda.stream(download):
                for d, h in zip(outs, outputs_h):
                    h.copy_(d, non_blocking=True)
            freed[k % 2] = torch.cuda.Event(enable_timing=True)
            freed[k % 2].record(download)
        return freed[(n - 1) % 2]

    # Untimed steps first: W, at least E2E_MIN_WARMUP, and repeated until E2E_MIN_WARMUP_S has
    # passed. The copy pipeline reaches its steady pace only some time after its pinned buffers
    # are allocated (measured on B200, K = 20 timed steps: 0.675-0.732 ms a step after 5 warm-up
    # steps, 0.646 after 30, 0.616 over 200; fresh buffers in one process ran 1.07 ms a step for
    # their first ~40 ms of copies and 0.62-0.65 from ~75 ms on).
    warm_steps = max(3, args.warmup, E2E_MIN_WARMUP)
    warm_total = 0
    warm_until = time.perf_counter() + E2E_MIN_WARMUP_S
    while warm_total == 0 or time.perf_counter() < warm_until:
        pipeline(warm_steps).synchronize()
        warm_total += warm_steps
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    e1 = pipeline(steps, first=e0)
    e1.synchronize()
    wall = time.perf_counter() - wall0
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1))
    return {
        "value": per_step * dist.world * steps / (ms * 1e-3) / 1e9,
        "unit": "GB/s",
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": d2h,
        "steps": steps,
        "warmup_steps": warm_total,
        "ms_per_step": ms / steps,
        "wall_ms_per_step": wall / steps * 1e3,
        "api": "torch.ops.inference_performance_lab (pinned host buffers, non_blocking copies; "
               "two device buffer sets, upload / op / download on three streams, so step k + 1's "
               "upload overlaps step k's download; x and residual packed side by side, one copy "
               "each way per step)" if workload.op == "fused_add_rms_norm" and not spec.get("offset") else
               "torch.ops.inference_performance_lab (pinned host buffers, non_blocking copies; "
               "two device buffer sets, upload / op / download on three streams, so step k + 1's "
               "upload overlaps step k's download)",
    }


def _reserve_stdout_for_the_result() -> None:
    """Only the result line goes to stdout: libraries that print from C are sent to stderr by
    pointing file descriptor 1 there, and Python's stdout is re-opened on a private duplicate of
    the original descriptor."""
    sys.stdout.flush()
    result_fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(result_fd, "w", buffering=1)


def main() -> None:
    _reserve_stdout_for_the_result()
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=3000)
    parser.add_argument("--warmup", type=int, default=50)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="rmsnorm")
    parser.add_argument("--e2e-steps", type=int, default=200)
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--reference-seconds", type=float, default=60.0,
                        help="--impl reference: CPU time budget of warm-up + timed steps")
    parser.add_argument("--no-subrecords", action="store_true",
                        help="measure the chosen workload only (no sharded / misaligned / silu records)")
    parser.add_argument("--rows", type=int, default=None,
                        help="override the workload's row count (small cases for profiling)")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    spec = dict(WORKLOADS[args.workload])
    if args.rows is not None:
        spec["rows"] = args.rows
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, spec)
    else:
        run_ours(args, spec)


if __name__ == "__main__":
    main()
