"""GPU parity of SiLU-and-mul against the oracle and the reference's golden vectors.

Mirrors the reference's tests/test_silu_and_mul.py (seed 0, I = 18944, T in {1, 8, 128, 2048},
rtol = atol = 1e-2, input unmodified, both op names) and extends it: golden vectors of
reference.py, widths and alignments that exercise every kernel with canary guards, the packed
op's rejection of what it cannot vectorise, the N(0, 2) [128, 37888] workload, and the C ABI.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from inference_performance_lab.kernels.extension import silu_and_mul as custom_silu_and_mul
from inference_performance_lab.kernels.extension import silu_and_mul_packed as custom_packed_silu_and_mul
from oracle import oracle
from parity import Guarded, assert_close_to_oracle, require_cuda

INTERMEDIATE_SIZE = 18944
TOKEN_COUNTS = [1, 8, 128, 2048]

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN = np.load(GOLDEN_DIR / "golden.npz")
CASES = json.loads((GOLDEN_DIR / "golden.json").read_text())["cases"]
SILU_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "silu_and_mul")

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


@pytest.mark.parametrize(
    "implementation",
    [
        pytest.param(custom_silu_and_mul, id="custom-scalar"),
        pytest.param(custom_packed_silu_and_mul, id="custom-packed"),
    ],
)
@pytest.mark.parametrize("num_tokens", TOKEN_COUNTS)
@torch.inference_mode()
def test_custom_matches_reference(implementation, num_tokens: int) -> None:
    torch.manual_seed(0)
    x = torch.randn((num_tokens, 2 * INTERMEDIATE_SIZE), device="cuda", dtype=torch.bfloat16)
    original = x.clone()

    expected = oracle.torch_silu_and_mul(x.cpu())
    actual = implementation(x)

    torch.testing.assert_close(actual.cpu(), expected, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(x, original, rtol=0, atol=0)
    assert_close_to_oracle(actual, oracle.c_silu_and_mul(oracle.tensor_bits(x)), f"T={num_tokens}")


@pytest.mark.parametrize("num_tokens", TOKEN_COUNTS)
@torch.inference_mode()
def test_vllm_matches_reference(num_tokens: int) -> None:
    """The comparison arm of the head-to-head benchmarks (vLLM's kernel) meets the same oracle, as
    the reference's own test of it does (tests/test_silu_and_mul.py:52-61 of the reference)."""
    pytest.importorskip("vllm._custom_ops")
    torch.manual_seed(0)
    x = torch.randn((num_tokens, 2 * INTERMEDIATE_SIZE), device="cuda", dtype=torch.bfloat16)
    output = torch.empty((num_tokens, INTERMEDIATE_SIZE), device="cuda", dtype=torch.bfloat16)
    torch.ops._C.silu_and_mul(output, x)
    torch.testing.assert_close(output.cpu(), oracle.torch_silu_and_mul(x.cpu()), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("name", SILU_CASES)
@torch.inference_mode()
def test_golden_vectors(name: str) -> None:
    meta = CASES[name]
    rows, inter = meta["rows"], meta["intermediate"]
    gi, go = Guarded((rows, 2 * inter), 0), Guarded((rows, inter), 0)
    x = gi.load(GOLDEN[f"{name}.input"])
    torch.ops.inference_performance_lab.silu_and_mul(go.tensor, x)
    # Saturated gates (|g| near 88, where e^-g approaches the fp32 limit) are compared by the
    # reference tests' tolerance only; everywhere else within one bf16 ulp of the reference.
    assert_close_to_oracle(go.tensor, GOLDEN[f"{name}.out"], name,
                           max_ulp=1 if name != "silu_extremes" else 1 << 16)
    assert torch.equal(oracle.bits_tensor(GOLDEN[f"{name}.input"], "cuda"), x)
    gi.assert_guards_intact()
    go.assert_guards_intact()


SWEEP = [
    # rows, intermediate, output offset, input offset (elements)
    *[(rows, inter, 0, 0) for rows in (1, 5, 300) for inter in
      (1, 2, 3, 7, 8, 9, 15, 16, 17, 24, 1000, 1001, 4096, 14336, 18944, 18952)],
    *[(33, 18944, oo, io) for oo in (0, 1, 8, 16) for io in (0, 1, 8, 16)],
    (4097, 16, 0, 0),
    (70000, 16, 0, 0),
    (2, 1 << 20, 0, 0),
]


@pytest.mark.parametrize("rows, inter, out_off, in_off", SWEEP)
@torch.inference_mode()
def test_sweep_against_oracle(rows: int, inter: int, out_off: int, in_off: int) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows * 7 + inter)
    x = (torch.randn(rows, 2 * inter, device="cuda", generator=generator) * 2).to(torch.bfloat16)
    gi, go = Guarded(x.shape, in_off), Guarded((rows, inter), out_off)
    xin = gi.load(oracle.tensor_bits(x))
    torch.ops.inference_performance_lab.silu_and_mul(go.tensor, xin)
    assert_close_to_oracle(go.tensor, oracle.c_silu_and_mul(oracle.tensor_bits(x)),
                           f"rows={rows} I={inter} offsets={out_off},{in_off}")
    assert torch.equal(xin, x)
    gi.assert_guards_intact()
    go.assert_guards_intact()


@torch.inference_mode()
def test_silu_workload_128x37888_normal_std2() -> None:
    torch.manual_seed(0)
    x = (torch.randn(128, 37888, device="cuda") * 2.0).to(torch.bfloat16)
    out = torch.empty(128, 18944, device="cuda", dtype=torch.bfloat16)
    torch.ops.inference_performance_lab.silu_and_mul(out, x)
    assert_close_to_oracle(out, oracle.c_silu_and_mul(oracle.tensor_bits(x)), "128x37888")
    out2 = torch.empty_like(out)
    torch.ops.inference_performance_lab.silu_and_mul_packed(out2, x)
    assert torch.equal(out, out2)


@torch.inference_mode()
def test_three_dimensional_input() -> None:
    torch.manual_seed(1)
    x = torch.randn(4, 6, 2 * 4096, device="cuda", dtype=torch.bfloat16)
    out = custom_silu_and_mul(x)
    assert out.shape == (4, 6, 4096)
    assert_close_to_oracle(out, oracle.c_silu_and_mul(oracle.tensor_bits(x)), "3-D")


@torch.inference_mode()
def test_packed_rejects_what_it_cannot_vectorise() -> None:
    x = torch.randn(4, 2 * 18, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="the output width must be divisible by 8"):
        custom_packed_silu_and_mul(x)
    buf = torch.randn(4 * 2 * 16 + 1, device="cuda", dtype=torch.bfloat16)
    x = buf[1:].view(4, 32)
    with pytest.raises(RuntimeError, match="input and output must be 16-byte aligned"):
        custom_packed_silu_and_mul(x)
    # The general op takes the same input.
    out = custom_silu_and_mul(x)
    assert_close_to_oracle(out, oracle.c_silu_and_mul(oracle.tensor_bits(x)), "misaligned general")


@torch.inference_mode()
def test_shape_and_dtype_errors() -> None:
    x = torch.randn(4, 32, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="input and output must use bfloat16"):
        torch.ops.inference_performance_lab.silu_and_mul(torch.empty(4, 16, device="cuda"), x)
    with pytest.raises(RuntimeError, match="the output width must be half the input width"):
        torch.ops.inference_performance_lab.silu_and_mul(
            torch.empty(4, 15, device="cuda", dtype=torch.bfloat16), x
        )
    with pytest.raises(RuntimeError, match="leading dimensions must match"):
        torch.ops.inference_performance_lab.silu_and_mul(
            torch.empty(3, 16, device="cuda", dtype=torch.bfloat16), x
        )
    with pytest.raises(RuntimeError, match="the final input dimension must be even"):
        torch.ops.inference_performance_lab.silu_and_mul(
            torch.empty(4, 16, device="cuda", dtype=torch.bfloat16), x[:, :31].contiguous()
        )
    empty = torch.empty(0, 32, device="cuda", dtype=torch.bfloat16)
    assert custom_silu_and_mul(empty).shape == (0, 16)


@torch.inference_mode()
def test_c_abi_entry_points_match_torch_op() -> None:
    torch.manual_seed(2)
    x = torch.randn(128, 37888, device="cuda", dtype=torch.bfloat16)
    expected = custom_silu_and_mul(x)
    for packed in (False, True):
        out = torch.empty_like(expected)
        capi.silu_and_mul_tensors(out, x, packed=packed)
        torch.cuda.synchronize()
        assert torch.equal(out, expected)


@torch.inference_mode()
def test_graph_capture() -> None:
    torch.manual_seed(3)
    x = torch.randn(128, 37888, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(128, 18944, device="cuda", dtype=torch.bfloat16)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        torch.ops.inference_performance_lab.silu_and_mul(out, x)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert_close_to_oracle(out, oracle.c_silu_and_mul(oracle.tensor_bits(x)), "graph")
    del graph


@pytest.mark.vllm
@torch.inference_mode()
def test_vllm_silu_and_mul_layer_runs_the_b200_kernel() -> None:
    """vLLM's SiluAndMul layer, replaced through its out-of-tree custom-op registry, returns these
    kernels' result (bit-identical to the op) and matches the oracle and vLLM's native path."""
    pytest.importorskip("vllm.model_executor.layers.activation")
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.model_executor.layers.activation import SiluAndMul

    from inference_performance_lab.kernels import vllm_plugin

    from vllm.config import CompilationConfig

    vllm_plugin.register_silu_and_mul()
    vllm_plugin.register_silu_and_mul()  # idempotent
    with set_current_vllm_config(VllmConfig()):
        layer = SiluAndMul()
    assert type(layer).__name__ == "InferenceLabSiluAndMul"
    # vLLM's own switch for the op under compilation turns the replacement on.
    assert type(layer).name == SiluAndMul.name == "silu_and_mul"
    with set_current_vllm_config(VllmConfig(compilation_config=CompilationConfig(custom_ops=["+silu_and_mul"]))):
        assert type(layer).enabled()
    torch.manual_seed(4)
    x = (torch.randn(128, 37888, device="cuda") * 2).to(torch.bfloat16)
    y = layer.forward_cuda(x)
    assert torch.equal(y, custom_silu_and_mul(x))
    assert_close_to_oracle(y, oracle.c_silu_and_mul(oracle.tensor_bits(x)), "vLLM SiluAndMul")
    torch.testing.assert_close(y, SiluAndMul.forward_native(x), rtol=1e-2, atol=1e-2)
    # Inputs the kernels do not take go to vLLM's own kernel.
    x16 = x.to(torch.float16)
    torch.testing.assert_close(layer.forward_cuda(x16), SiluAndMul.forward_native(x16), rtol=1e-2, atol=1e-2)
