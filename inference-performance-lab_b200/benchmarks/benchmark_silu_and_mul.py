"""Head-to-head of these SiLU-and-mul kernels and vLLM's CUDA kernel on B200, per token count.

    python inference-performance-lab_b200/benchmarks/benchmark_silu_and_mul.py
        [--intermediate 18944] [--tokens 1,8,128,2048]

Follows the reference's microbenchmark protocol (benchmarks/benchmark_silu_and_mul.py:10-53):
intermediate 18944, seed 0, input N(0, 1) of shape [T, 2 * 18944], token counts 1 / 8 / 128 /
2048 with 2000 / 1000 / 300 / 50 timed calls after 25 warm-up calls on the same buffers
(L2-warm), CUDA events around the loop, GB/s at 6 bytes per output element, and the three
implementations vLLM (``torch.ops._C.silu_and_mul``), custom scalar and custom packed (here both
names reach the same dispatcher). Adds the same calls replayed from one CUDA graph.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from benchmark_fused_add_rms_norm import _iterations, time_graph, time_stream  # noqa: E402
from inference_performance_lab.kernels.extension import load_extension  # noqa: E402

BYTES_PER_OUTPUT = 6


def make_call(impl: str, tokens: int, intermediate: int):
    torch.manual_seed(0)
    x = torch.randn(tokens, 2 * intermediate, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(tokens, intermediate, device="cuda", dtype=torch.bfloat16)
    fn = {
        "vLLM": torch.ops._C.silu_and_mul,
        "Custom scalar": torch.ops.inference_performance_lab.silu_and_mul,
        "Custom packed": torch.ops.inference_performance_lab.silu_and_mul_packed,
    }[impl]
    return lambda: fn(out, x)


@torch.inference_mode()
def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--intermediate", type=int, default=18944)
    parser.add_argument("--tokens", default="1,8,128,2048")
    args = parser.parse_args()
    token_counts = [int(t) for t in args.tokens.split(",")]

    load_extension()
    import vllm._custom_ops  # noqa: F401  (registers torch.ops._C)

    impls = ("vLLM", "Custom scalar", "Custom packed")
    results = {}
    for impl in impls:
        for tokens in token_counts:
            call = make_call(impl, tokens, args.intermediate)
            iterations = _iterations(tokens)
            results[impl, tokens] = (time_stream(call, iterations), time_graph(call, iterations))

    print(f"silu_and_mul intermediate={args.intermediate} ({torch.cuda.get_device_name()})")
    print("| Tokens | vLLM (us) | Custom scalar (us) | Custom packed (us) | Packed speedup | vLLM GB/s "
          "| Packed GB/s | vLLM graph (us) | Packed graph (us) | Graph speedup |")
    print("|---:|---:|---:|---:|---:|---:|---:|---:|---:|---:|")
    for tokens in token_counts:
        v, s, p = (results[i, tokens] for i in impls)
        nbytes = tokens * args.intermediate * BYTES_PER_OUTPUT
        print(f"| {tokens} | {v[0]:.3f} | {s[0]:.3f} | {p[0]:.3f} | {v[0] / p[0]:.3f}x "
              f"| {nbytes / v[0] / 1e3:.1f} | {nbytes / p[0] / 1e3:.1f} | {v[1]:.3f} | {p[1]:.3f} "
              f"| {v[1] / p[1]:.3f}x |")


if __name__ == "__main__":
    main()
