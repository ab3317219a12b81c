"""Offline vLLM serving of a Qwen2.5-7B-architecture decoder with a chosen RMSNorm provider.

    python inference-performance-lab_b200/vllm_serving_bench.py \
        --provider inference_lab|vllm_c|native [--concurrency 1,8,32] [--layers 28]
        [--requests 64] [--input-len 2048] [--output-len 32] [--profile]

The reference measures its provider end to end in vLLM serving (scripts/serve.sh,
scripts/benchmark.sh; results/a100-qwen2.5-7b-custom-rmsnorm-analysis.md): `vllm bench serve`
with the synthetic "random" dataset at several concurrencies, reporting tok/s, TTFT and TPOT.
There is no network here, so the model is the Qwen2.5-7B architecture (28 layers, hidden 3584,
intermediate 18944, 28 query / 4 KV heads, head_dim 128, vocab 152064, RMSNorm eps 1e-6) with
vLLM's dummy (random) weights, and the requests are uniform-random token ids. Greedy decoding,
prefix caching off, decode steps replayed from full CUDA graphs, no torch.compile. The engine
runs in this process so that the plugin registered here is the one the model uses.

Providers: ``inference_lab`` = this library for fused_add_rms_norm, rms_norm and SiluAndMul;
``vllm_c`` = vLLM's own CUDA kernels for all three (the reference's comparison arm);
``native`` = vLLM's PyTorch RMSNorm (eager, several kernels per call) and vLLM's SiLU kernel.

Concurrency c is emulated offline: the requests are submitted in waves of c (every request of
a wave has the same input and output length, so the waves keep c requests in flight, like
`--max-concurrency c`). Prints one JSON line with, per c, total and output tok/s, mean TTFT
(engine arrival to first token) and mean TPOT (first to last token over the tokens after the
first), and with --profile the norm and activation CUDA kernels of one short run (8 requests,
4 output tokens) by name with their launch count and total / mean device time, showing which
kernels ran inside the CUDA graphs and what they cost there.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

QWEN25_7B = {
    "architectures": ["Qwen2ForCausalLM"],
    "model_type": "qwen2",
    "hidden_size": 3584,
    "intermediate_size": 18944,
    "num_hidden_layers": 28,
    "num_attention_heads": 28,
    "num_key_value_heads": 4,
    "vocab_size": 152064,
    "max_position_embeddings": 32768,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "hidden_act": "silu",
    "torch_dtype": "bfloat16",
    "tie_word_embeddings": False,
    "use_sliding_window": False,
    "sliding_window": None,
    "bos_token_id": 151643,
    "eos_token_id": 151645,
}

PROVIDERS = ("inference_lab", "vllm_c", "native")


def _wave_stats(outputs) -> tuple[list[float], list[float]]:
    ttft, tpot = [], []
    for out in outputs:
        stats = out.metrics
        if stats is None:
            continue
        ttft.append(stats.first_token_latency)
        n = len(out.outputs[0].token_ids)
        if n > 1:
            tpot.append((stats.last_token_ts - stats.first_token_ts) / (n - 1))
    return ttft, tpot


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--provider", choices=PROVIDERS, default="inference_lab")
    parser.add_argument("--concurrency", default="1,8,32")
    parser.add_argument("--layers", type=int, default=28)
    parser.add_argument("--requests", type=int, default=64)
    parser.add_argument("--input-len", type=int, default=2048)
    parser.add_argument("--output-len", type=int, default=32)
    parser.add_argument("--profile", action="store_true")
    args = parser.parse_args()
    concurrencies = [int(c) for c in args.concurrency.split(",")]

    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    import torch
    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    from inference_performance_lab.kernels import vllm_plugin

    if args.provider == "inference_lab":
        vllm_plugin.register()
        vllm_plugin.register_silu_and_mul()
    priority = {"fused_add_rms_norm": [args.provider], "rms_norm": [args.provider]}

    model_dir = Path(tempfile.mkdtemp(prefix="qwen25_7b_arch_"))
    config = dict(QWEN25_7B, num_hidden_layers=args.layers)
    (model_dir / "config.json").write_text(json.dumps(config))
    llm = LLM(
        model=str(model_dir),
        load_format="dummy",
        skip_tokenizer_init=True,
        dtype="bfloat16",
        max_model_len=args.input_len + args.output_len + 16,
        max_num_seqs=max(concurrencies),
        max_num_batched_tokens=max(8192, args.input_len),
        enable_prefix_caching=False,
        gpu_memory_utilization=0.85,
        seed=0,
        disable_log_stats=False,
        compilation_config={"mode": 0, "cudagraph_mode": "FULL_DECODE_ONLY"},
        ir_op_priority=priority,
    )
    generator = torch.Generator().manual_seed(0)
    prompts = [
        TokensPrompt(prompt_token_ids=torch.randint(0, 150000, (args.input_len,), generator=generator).tolist())
        for _ in range(args.requests)
    ]
    params = SamplingParams(max_tokens=args.output_len, temperature=0.0, ignore_eos=True, detokenize=False)
    llm.generate(prompts[: min(4, len(prompts))], params, use_tqdm=False)  # warm-up

    runs = {}
    for c in concurrencies:
        ttft, tpot, generated = [], [], 0
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for start in range(0, len(prompts), c):
            outputs = llm.generate(prompts[start:start + c], params, use_tqdm=False)
            generated += sum(len(o.outputs[0].token_ids) for o in outputs)
            wave_ttft, wave_tpot = _wave_stats(outputs)
            ttft += wave_ttft
            tpot += wave_tpot
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        runs[str(c)] = {
            "wall_s": round(wall, 4),
            "output_tokens_per_s": round(generated / wall, 1),
            "total_tokens_per_s": round((generated + len(prompts) * args.input_len) / wall, 1),
            "mean_ttft_ms": round(1e3 * sum(ttft) / len(ttft), 3) if ttft else None,
            "mean_tpot_ms": round(1e3 * sum(tpot) / len(tpot), 3) if tpot else None,
        }

    kernels = None
    if args.profile:
        from torch.profiler import ProfilerActivity, profile

        short = SamplingParams(max_tokens=4, temperature=0.0, ignore_eos=True, detokenize=False)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            llm.generate(prompts[:8], short, use_tqdm=False)
            torch.cuda.synchronize()
        kernels = {}
        for event in prof.events():
            if event.device_type.name == "CUDA":
                name = event.name
                if any(k in name for k in ("rms", "norm", "silu", "Silu", "act_and_mul")):
                    entry = kernels.setdefault(name[:90], {"launches": 0, "total_us": 0.0})
                    entry["launches"] += 1
                    entry["total_us"] += event.device_time_total
        for entry in kernels.values():
            entry["mean_us"] = round(entry["total_us"] / entry["launches"], 3)
            entry["total_us"] = round(entry["total_us"], 1)

    line = {
        "provider": args.provider,
        "model": f"Qwen2.5-7B architecture, {args.layers} layers, dummy bf16 weights",
        "requests": args.requests,
        "input_len": args.input_len,
        "output_len": args.output_len,
        "by_concurrency": runs,
        "norm_and_activation_kernels": kernels,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
