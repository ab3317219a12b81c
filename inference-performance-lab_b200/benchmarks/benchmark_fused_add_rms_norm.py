"""Head-to-head of these RMSNorm kernels and vLLM's CUDA kernels on B200, per token count.

    python inference-performance-lab_b200/benchmarks/benchmark_fused_add_rms_norm.py
        [--op fused|plain|fp8] [--hidden 3584] [--tokens 1,8,128,2048] [--cold]

Follows the reference's microbenchmark protocol (benchmarks/benchmark_fused_add_rms_norm.py:12-
52): hidden 3584, seed 0, x and residual N(0, 1), weight 1 + 0.1 N(0, 1), eps 1e-6, token counts
1 / 8 / 128 / 2048 with 2000 / 1000 / 300 / 50 timed calls after 25 warm-up calls, the same
buffers every call (L2-warm), CUDA events around the loop, and GB/s at its 10 bytes per element
(x, residual and weight read, x and residual written). It prints the same table and adds two
columns per implementation: the same calls replayed from one CUDA graph (device time without
the host's per-call cost, which is what vLLM's captured decode steps see).

``--op plain`` compares ``rms_norm(out, x, w, eps)`` (6 B/elem: x and weight read, out
written) and ``--op fp8`` the add+RMSNorm with a static e4m3 output
(``fused_add_rms_norm_static_fp8_quant``; 9 B/elem) against vLLM's ops of the same names.

``--cold`` measures the HBM-bound case instead: consecutive calls cycle through enough buffer
sets to exceed four times the 126 MB L2 (or one set larger than that), and GB/s count only the
bytes that must cross HBM (weight excluded: 8 / 4 / 7 B/elem).
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from inference_performance_lab.kernels.extension import load_extension  # noqa: E402

EPSILON = 1e-6
ITERATIONS = {1: 2000, 8: 1000, 128: 300, 2048: 50}
WARMUP_ITERATIONS = 25
BYTES_PER_ELEMENT = {"fused": 10, "plain": 6, "fp8": 9}
HBM_BYTES_PER_ELEMENT = {"fused": 8, "plain": 4, "fp8": 7}
L2_BYTES = 126 * 2**20


def _iterations(tokens: int) -> int:
    return ITERATIONS.get(tokens, max(20, min(2000, 100_000_000 // max(1, tokens * 3584 * 10))))


def make_call(impl: str, op: str, tokens: int, hidden: int):
    x = torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    residual = torch.randn_like(x)
    weight = torch.randn(hidden, device="cuda", dtype=torch.bfloat16) * 0.1 + 1.0
    ours = torch.ops.inference_performance_lab
    theirs = torch.ops._C
    if op == "fused":
        fn = ours.fused_add_rms_norm if impl == "custom" else theirs.fused_add_rms_norm
        return lambda: fn(x, residual, weight, EPSILON)
    if op == "plain":
        out = torch.empty_like(x)
        fn = ours.rms_norm if impl == "custom" else theirs.rms_norm
        return lambda: fn(out, x, weight, EPSILON)
    result = torch.empty(tokens, hidden, device="cuda", dtype=torch.float8_e4m3fn)
    scale = torch.tensor([0.05], device="cuda", dtype=torch.float32)
    fn = ours.fused_add_rms_norm_static_fp8_quant if impl == "custom" else theirs.fused_add_rms_norm_static_fp8_quant
    return lambda: fn(result, x, residual, weight, scale, EPSILON)


MAX_SETS = 1024  # cold mode needs tokens * hidden * B/elem >= 4 x L2 / 1024 (~0.5 MB) to be cold


def make_calls(impl: str, op: str, tokens: int, hidden: int, cold: bool) -> list:
    """One call (L2-warm), or calls over enough buffer sets to exceed 4x L2 (cold)."""
    torch.manual_seed(0)
    sets = 1
    if cold:
        per_set = tokens * hidden * HBM_BYTES_PER_ELEMENT[op]
        sets = min(MAX_SETS, max(1, math.ceil(4 * L2_BYTES / per_set))) if per_set < 4 * L2_BYTES else 1
    return [make_call(impl, op, tokens, hidden) for _ in range(sets)]


def time_stream(calls, iterations: int) -> float:
    calls = calls if isinstance(calls, list) else [calls]
    for i in range(WARMUP_ITERATIONS):
        calls[i % len(calls)]()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(iterations):
        calls[i % len(calls)]()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) * 1e3 / iterations


def time_graph(calls, iterations: int) -> float:
    calls = calls if isinstance(calls, list) else [calls]
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        calls[0]()  # warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(iterations):
                calls[i % len(calls)]()
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    graph.replay()
    end.record()
    end.synchronize()
    elapsed = start.elapsed_time(end) * 1e3 / iterations
    del graph
    return elapsed


@torch.inference_mode()
def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--op", choices=sorted(BYTES_PER_ELEMENT), default="fused")
    parser.add_argument("--hidden", type=int, default=3584)
    parser.add_argument("--tokens", default="1,8,128,2048")
    parser.add_argument("--cold", action="store_true")
    args = parser.parse_args()
    token_counts = [int(t) for t in args.tokens.split(",")]

    load_extension()
    import vllm._custom_ops  # noqa: F401  (registers torch.ops._C)

    results = {}
    for impl in ("vLLM", "custom"):
        for tokens in token_counts:
            calls = make_calls("custom" if impl == "custom" else "vllm", args.op, tokens, args.hidden, args.cold)
            iterations = max(_iterations(tokens), 2 * len(calls))
            results[impl, tokens] = (time_stream(calls, iterations), time_graph(calls, iterations))
            del calls
            torch.cuda.empty_cache()

    per_element = (HBM_BYTES_PER_ELEMENT if args.cold else BYTES_PER_ELEMENT)[args.op]
    regime = "cold L2, HBM bytes" if args.cold else "L2-warm"
    print(f"op={args.op} hidden={args.hidden} {regime}, {per_element} B/elem ({torch.cuda.get_device_name()})")
    print("| Tokens | vLLM (us) | Custom (us) | Speedup | vLLM GB/s | Custom GB/s "
          "| vLLM graph (us) | Custom graph (us) | Graph speedup |")
    print("|---:|---:|---:|---:|---:|---:|---:|---:|---:|")
    for tokens in token_counts:
        (v_us, v_graph), (c_us, c_graph) = results["vLLM", tokens], results["custom", tokens]
        nbytes = tokens * args.hidden * per_element
        print(f"| {tokens} | {v_us:.3f} | {c_us:.3f} | {v_us / c_us:.3f}x | {nbytes / v_us / 1e3:.1f} "
              f"| {nbytes / c_us / 1e3:.1f} | {v_graph:.3f} | {c_graph:.3f} | {v_graph / c_graph:.3f}x |")


if __name__ == "__main__":
    main()
