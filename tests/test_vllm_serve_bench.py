"""The serving driver (inference-performance-lab_b200/vllm_serve_bench.py) on the CPU, the way the
reference tests its serving scripts (tests/test_serving_scripts.py: a fake CLI records argv; the
flags of `vllm serve` and `vllm bench serve` are asserted; a failing exit code must propagate):

* the server is started with the reference's serve flags (scripts/serve.sh:10-41) and the
  provider's VLLM_PLUGINS / --ir-op-priority, and each benchmark with the reference's
  `vllm bench serve` flags (scripts/benchmark.sh:37-53);
* the stand-in tokenizer keeps every prompt of vLLM's own random dataset at exactly the input length;
* a server that exits before it is ready ends the run with an error (no hang, no result line).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "inference-performance-lab_b200"))

import vllm_serve_bench as serve  # noqa: E402


class _Args:
    concurrency = "1,8"
    num_prompts = 16
    input_len = 2048
    output_len = 32
    profile = False
    port = 8099
    startup_timeout = 30.0
    custom_ops = None


def test_commands_follow_the_reference_protocol(tmp_path: Path, monkeypatch) -> None:
    calls = {"popen": [], "run": []}

    class FakeServer:
        pid = 4242
        returncode = None

        def __init__(self, argv, env=None, **kwargs):
            calls["popen"].append((argv, env))

        def poll(self):
            return None

        def wait(self, timeout=None):
            return 0

    def fake_run(argv, env=None, stdout=None, **kwargs):
        calls["run"].append((argv, env))
        if "bench" in argv:
            result_dir = Path(argv[argv.index("--result-dir") + 1])
            name = argv[argv.index("--result-filename") + 1]
            (result_dir / name).write_text(json.dumps({"completed": 16, "output_throughput": 100.0,
                                                       "mean_ttft_ms": 1.0, "mean_tpot_ms": 1.0}))

    monkeypatch.setattr(serve, "install_package", lambda site: site.mkdir(parents=True, exist_ok=True))
    monkeypatch.setattr(serve.subprocess, "Popen", FakeServer)
    monkeypatch.setattr(serve.subprocess, "run", fake_run)
    monkeypatch.setattr(serve, "wait_healthy", lambda port, server, limit: None)
    monkeypatch.setattr(serve, "stop", lambda server: None)

    line = serve.run(_Args(), "inference_lab", tmp_path)
    (server_argv, server_env), = calls["popen"]
    for flag, value in (("--dtype", "bfloat16"), ("--max-model-len", "4096"), ("--gpu-memory-utilization", "0.90"),
                        ("--generation-config", "vllm"), ("--seed", "0"), ("--load-format", "dummy"),
                        ("--host", "127.0.0.1"), ("--port", "8099")):
        assert server_argv[server_argv.index(flag) + 1] == value, flag
    assert "--no-enable-prefix-caching" in server_argv
    assert json.loads(server_argv[server_argv.index("--ir-op-priority") + 1]) == {
        "fused_add_rms_norm": ["inference_lab"], "rms_norm": ["inference_lab"]}
    assert server_env["VLLM_PLUGINS"] == "inference_performance_lab,inference_performance_lab_silu"

    benches = [argv for argv, _ in calls["run"] if "bench" in argv]
    assert [b[b.index("--max-concurrency") + 1] for b in benches] == ["1", "8"]
    for b in benches:
        for flag, value in (("--backend", "openai"), ("--endpoint", "/v1/completions"), ("--dataset-name", "random"),
                            ("--random-input-len", "2048"), ("--random-output-len", "32"),
                            ("--random-range-ratio", "0"), ("--request-rate", "inf"), ("--seed", "0"),
                            ("--temperature", "0"), ("--num-warmups", "2"), ("--num-prompts", "16"),
                            ("--percentile-metrics", "ttft,tpot,itl,e2el")):
            assert b[b.index(flag) + 1] == value, flag
        assert "--ignore-eos" in b and "--save-result" in b
    assert set(line["by_concurrency"]) == {"1", "8"} and line["provider"] == "inference_lab"

    calls["popen"].clear()
    serve.run(_Args(), "vllm_c", tmp_path)
    (server_argv, server_env), = calls["popen"]
    assert server_env["VLLM_PLUGINS"] == ""  # as the reference's serve.sh: no general plugin
    assert json.loads(server_argv[server_argv.index("--ir-op-priority") + 1])["fused_add_rms_norm"] == ["vllm_c"]


def test_stand_in_tokenizer_keeps_random_prompts_at_the_input_length(tmp_path: Path) -> None:
    pytest.importorskip("vllm.benchmarks.datasets")
    from transformers import AutoTokenizer
    from vllm.benchmarks.datasets import RandomDataset

    model = serve.write_model_dir(tmp_path / "model")
    assert json.loads((model / "config.json").read_text())["num_hidden_layers"] == 28
    tokenizer = AutoTokenizer.from_pretrained(str(model))
    assert tokenizer.num_special_tokens_to_add() == 0
    requests = RandomDataset(random_seed=0).sample(tokenizer=tokenizer, num_requests=3, input_len=2048,
                                                   output_len=32, range_ratio=0.0)
    assert [r.prompt_len for r in requests] == [2048, 2048, 2048]
    assert all(len(tokenizer.encode(r.prompt, add_special_tokens=False)) == 2048 for r in requests)


def test_a_server_that_dies_at_startup_ends_the_run(tmp_path: Path, monkeypatch) -> None:
    class DeadServer:
        pid = 4243
        returncode = 1

        def __init__(self, *args, **kwargs):
            pass

        def poll(self):
            return 1

    monkeypatch.setattr(serve, "install_package", lambda site: site.mkdir(parents=True, exist_ok=True))
    monkeypatch.setattr(serve.subprocess, "Popen", DeadServer)
    monkeypatch.setattr(serve, "stop", lambda server: None)
    with pytest.raises(RuntimeError, match="exited with 1 before it was ready"):
        serve.run(_Args(), "inference_lab", tmp_path)
