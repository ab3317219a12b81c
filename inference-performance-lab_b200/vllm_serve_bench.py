"""vLLM serving of a Qwen2.5-7B-architecture decoder the reference's way: `vllm serve` plus
`vllm bench serve`, vLLM's default compilation, one provider per server.

    python inference-performance-lab_b200/vllm_serve_bench.py --provider inference_lab|vllm_c
        [--concurrency 1,8,32] [--num-prompts 64] [--input-len 2048] [--output-len 32]
        [--custom-ops +silu_and_mul] [--profile] [--port 8011] [--workdir DIR]

It follows the reference's scripts: scripts/serve.sh:10-41 (the provider chosen with
VLLM_PLUGINS and --ir-op-priority; bf16, --max-model-len 4096, --gpu-memory-utilization 0.90,
--no-enable-prefix-caching, --generation-config vllm, --seed 0) and scripts/benchmark.sh:37-53
(`vllm bench serve --backend openai --endpoint /v1/completions --dataset-name random
--random-range-ratio 0 --ignore-eos --request-rate inf --max-concurrency c --seed 0
--temperature 0 --num-warmups 2`). The plugin is found through this package's installed
``vllm.general_plugins`` entry points, as `vllm serve` finds the reference's: the package is
installed (offline) into a directory of the work tree first.

What cannot be had offline is replaced, and nothing else: the checkpoint by vLLM's dummy weights
of the same architecture (28 layers, hidden 3584, intermediate 18944, 28 query / 4 KV heads,
head_dim 128, vocab 152064, eps 1e-6), and Qwen's tokenizer by a word-level tokenizer of the same
vocabulary size (token i is the word "t<i>", so the random dataset's decode / re-encode round trip
keeps every prompt at exactly --input-len tokens).

Providers: ``vllm_c`` = vLLM's own CUDA kernels, the reference's comparison arm
(VLLM_PLUGINS=""); ``inference_lab`` = this library for fused_add_rms_norm and rms_norm (IR
providers, lowered into the compiled graph) and SiluAndMul (the second entry point). Under vLLM's
default compilation custom ops are off and SiLU-and-mul is fused by Inductor into a Triton kernel
for either provider; --custom-ops +silu_and_mul turns vLLM's SiluAndMul op on, which then runs
this library's kernel (inference_lab) or vLLM's (vllm_c). With --profile, a short extra run is traced
with vLLM's torch profiler and the norm and activation kernels are listed by name with launch
counts and device time, which shows what ran inside the compiled, CUDA-graphed model.

Prints one JSON line per provider run.
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import shutil
import signal
import subprocess
import sys
import time
import urllib.request
from pathlib import Path

HERE = Path(__file__).resolve().parent

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
# Qwen2.5's tokenizer: 151643 regular tokens, then its special tokens from id 151643.
REGULAR_TOKENS = 151643
SPECIAL_TOKENS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
SERVED_NAME = "qwen2.5-7b-arch"


def write_model_dir(path: Path) -> Path:
    """config.json of the architecture and a word-level tokenizer of Qwen's vocabulary size."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers

    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(QWEN25_7B))
    vocab = {f"t{i}": i for i in range(REGULAR_TOKENS)}
    for k, token in enumerate(SPECIAL_TOKENS):
        vocab[token] = REGULAR_TOKENS + k
    tokenizer = Tokenizer(models.WordLevel(vocab, unk_token="<|endoftext|>"))
    tokenizer.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tokenizer.decoder = decoders.WordPiece(prefix="##", cleanup=False)  # joins words with spaces
    tokenizer.add_special_tokens(SPECIAL_TOKENS)
    tokenizer.save(str(path / "tokenizer.json"))
    (path / "tokenizer_config.json").write_text(json.dumps({
        "tokenizer_class": "PreTrainedTokenizerFast",
        "bos_token": None,
        "eos_token": "<|im_end|>",
        "pad_token": "<|endoftext|>",
        "unk_token": "<|endoftext|>",
        "model_max_length": 32768,
        "clean_up_tokenization_spaces": False,
    }))
    (path / "generation_config.json").write_text(json.dumps({"eos_token_id": 151645, "do_sample": False}))
    return path


def install_package(site: Path) -> None:
    """This package (with its built native libraries) installed offline into `site`, so that the
    server process finds its vllm.general_plugins entry points."""
    if (site / "inference_performance_lab").exists():
        return
    subprocess.run([sys.executable, str(HERE / "build.py"), "-q"], check=True)
    source = site.parent / "package_src"
    if source.exists():
        shutil.rmtree(source)
    source.mkdir(parents=True)
    shutil.copy(HERE / "pyproject.toml", source / "pyproject.toml")
    shutil.copytree(HERE / "inference_performance_lab", source / "inference_performance_lab",
                    ignore=shutil.ignore_patterns("__pycache__", "test", "*.stamp", "*.txt", ".build.lock"))
    subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "--no-build-isolation",
                    "--quiet", "--target", str(site), str(source)], check=True)


def provider_env(provider: str, site: Path) -> tuple[dict, dict]:
    env = dict(os.environ)
    env["PYTHONPATH"] = str(site)
    if provider == "vllm_c":
        env["VLLM_PLUGINS"] = ""  # as the reference's serve.sh: no general plugin loads
        priority = {"fused_add_rms_norm": ["vllm_c"], "rms_norm": ["vllm_c"]}
    else:
        env["VLLM_PLUGINS"] = "inference_performance_lab,inference_performance_lab_silu"
        priority = {"fused_add_rms_norm": ["inference_lab"], "rms_norm": ["inference_lab"]}
    return env, priority


def wait_healthy(port: int, server: subprocess.Popen, limit_s: float) -> None:
    deadline = time.monotonic() + limit_s
    while time.monotonic() < deadline:
        if server.poll() is not None:
            raise RuntimeError(f"vllm serve exited with {server.returncode} before it was ready")
        try:
            with urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=5) as reply:
                if reply.status == 200:
                    return
        except OSError:
            pass
        time.sleep(5)
    raise RuntimeError(f"vllm serve not ready after {limit_s:.0f} s")


def stop(server: subprocess.Popen) -> None:
    if server.poll() is None:
        os.killpg(server.pid, signal.SIGINT)
        try:
            server.wait(timeout=60)
        except subprocess.TimeoutExpired:
            os.killpg(server.pid, signal.SIGKILL)
            server.wait(timeout=60)


def bench_serve(args, model_dir: Path, env: dict, concurrency: int, result_dir: Path, *, num_prompts: int,
                output_len: int, profile: bool = False) -> dict:
    name = f"c{concurrency}{'-profile' if profile else ''}.json"
    command = [
        sys.executable, "-m", "vllm.entrypoints.cli.main", "bench", "serve",
        "--backend", "openai", "--base-url", f"http://127.0.0.1:{args.port}", "--endpoint", "/v1/completions",
        "--model", SERVED_NAME, "--tokenizer", str(model_dir), "--dataset-name", "random",
        "--num-prompts", str(num_prompts), "--random-input-len", str(args.input_len),
        "--random-output-len", str(output_len), "--random-range-ratio", "0", "--ignore-eos",
        "--request-rate", "inf", "--max-concurrency", str(concurrency), "--seed", "0", "--temperature", "0",
        "--num-warmups", "2", "--percentile-metrics", "ttft,tpot,itl,e2el", "--metric-percentiles", "50,90,95,99",
        "--save-result", "--result-dir", str(result_dir), "--result-filename", name,
    ]
    if profile:
        command.append("--profile")
    log = result_dir / (name + ".log")
    with open(log, "w") as out:
        subprocess.run(command, env=env, stdout=out, stderr=subprocess.STDOUT, check=True, timeout=1800)
    return json.loads((result_dir / name).read_text())


def profiled_kernels(trace_dir: Path) -> dict:
    """Norm and activation kernels in the torch-profiler traces the server wrote."""
    kernels: dict[str, dict] = {}
    for path in sorted(trace_dir.rglob("*.json*")):
        opener = gzip.open if path.suffix == ".gz" else open
        try:
            with opener(path, "rt") as f:
                trace = json.load(f)
        except (OSError, ValueError):
            continue
        for event in trace.get("traceEvents", []):
            if event.get("cat") != "kernel":
                continue
            name = event.get("name", "")
            if any(k in name for k in ("rms", "norm", "silu", "Silu", "act_and_mul")):
                entry = kernels.setdefault(name[:100], {"launches": 0, "total_us": 0.0})
                entry["launches"] += 1
                entry["total_us"] += float(event.get("dur", 0.0))
    for entry in kernels.values():
        entry["mean_us"] = round(entry["total_us"] / entry["launches"], 3)
        entry["total_us"] = round(entry["total_us"], 1)
    return kernels


def run(args, provider: str, work: Path) -> dict:
    model_dir = write_model_dir(work / "model")
    site = work / "site"
    install_package(site)
    env, priority = provider_env(provider, site)
    result_dir = work / f"results_{provider}"
    result_dir.mkdir(parents=True, exist_ok=True)
    trace_dir = work / f"traces_{provider}"
    command = [
        sys.executable, "-m", "vllm.entrypoints.cli.main", "serve", str(model_dir),
        "--load-format", "dummy", "--tokenizer", str(model_dir), "--served-model-name", SERVED_NAME,
        "--dtype", "bfloat16", "--max-model-len", "4096", "--gpu-memory-utilization", "0.90",
        "--no-enable-prefix-caching", "--generation-config", "vllm", "--seed", "0",
        "--ir-op-priority", json.dumps(priority), "--host", "127.0.0.1", "--port", str(args.port),
    ]
    if args.custom_ops:
        command += ["--compilation-config", json.dumps({"custom_ops": args.custom_ops.split(",")})]
    if args.profile:
        command += ["--profiler-config", json.dumps({
            "profiler": "torch", "torch_profiler_dir": str(trace_dir), "torch_profiler_with_stack": False,
            "torch_profiler_use_gzip": False})]
    server_log = open(work / f"server_{provider}.log", "w")
    started = time.monotonic()
    server = subprocess.Popen(command, env=env, stdout=server_log, stderr=subprocess.STDOUT, start_new_session=True)
    try:
        wait_healthy(args.port, server, args.startup_timeout)
        startup_s = time.monotonic() - started
        runs = {}
        for c in [int(c) for c in args.concurrency.split(",")]:
            r = bench_serve(args, model_dir, env, c, result_dir, num_prompts=args.num_prompts,
                            output_len=args.output_len)
            runs[str(c)] = {k: (round(r[k], 3) if isinstance(r.get(k), float) else r.get(k)) for k in (
                "completed", "total_input_tokens", "total_output_tokens", "duration", "request_throughput",
                "output_throughput", "total_token_throughput", "mean_ttft_ms", "median_ttft_ms", "p99_ttft_ms",
                "mean_tpot_ms", "median_tpot_ms", "p99_tpot_ms", "mean_itl_ms", "mean_e2el_ms")}
        kernels = None
        if args.profile:
            bench_serve(args, model_dir, env, 8, result_dir, num_prompts=8, output_len=4, profile=True)
            time.sleep(10)  # the trace is written after /stop_profile returns
            kernels = profiled_kernels(trace_dir)
    finally:
        stop(server)
        server_log.close()
    return {
        "provider": provider,
        "model": "Qwen2.5-7B architecture, 28 layers, dummy bf16 weights, word-level tokenizer of its vocabulary size",
        "server": "vllm serve, default compilation (torch.compile + CUDA graphs), prefix caching off"
                  + (f", custom ops {args.custom_ops}" if args.custom_ops else ""),
        "ir_op_priority": priority,
        "vllm_plugins": env["VLLM_PLUGINS"],
        "startup_s": round(startup_s, 1),
        "num_prompts": args.num_prompts,
        "input_len": args.input_len,
        "output_len": args.output_len,
        "by_concurrency": runs,
        "norm_and_activation_kernels": kernels,
    }


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--provider", choices=("inference_lab", "vllm_c"), action="append")
    parser.add_argument("--concurrency", default="1,8,32")
    parser.add_argument("--num-prompts", type=int, default=64)
    parser.add_argument("--input-len", type=int, default=2048)
    parser.add_argument("--output-len", type=int, default=32)
    parser.add_argument("--profile", action="store_true")
    parser.add_argument("--port", type=int, default=8011)
    parser.add_argument("--startup-timeout", type=float, default=1200.0)
    parser.add_argument("--workdir", type=Path, default=Path("vllm_serve_work"))
    parser.add_argument("--custom-ops", default=None,
                        help='vLLM custom ops to enable under compilation, e.g. "+silu_and_mul" (default: vLLM\'s)')
    args = parser.parse_args()
    args.workdir.mkdir(parents=True, exist_ok=True)
    for provider in args.provider or ["vllm_c", "inference_lab"]:
        print(json.dumps(run(args, provider, args.workdir.resolve())), flush=True)


if __name__ == "__main__":
    main()
