"""GPU parity of plain RMSNorm (no residual) against the oracle, the reference oracle's golden
vectors (its arithmetic with a zero residual) and vLLM's native rms_norm.

Not an op of the reference library: it is the plain rms_norm of the vLLM IR the reference's
plugin targets, built on the same row kernels. Outputs within rtol = atol = 1e-2 and one bf16
ulp of the oracle; canary guards around every tensor; in place and out of place.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from inference_performance_lab.kernels.extension import rms_norm as custom_rms_norm
from oracle import oracle
from parity import Guarded, assert_close_to_oracle, require_cuda

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN = np.load(GOLDEN_DIR / "golden.npz")
CASES = json.loads((GOLDEN_DIR / "golden.json").read_text())["cases"]
PLAIN_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "rms_norm")

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


@pytest.mark.parametrize("name", PLAIN_CASES)
@torch.inference_mode()
def test_golden_vectors(name: str) -> None:
    meta = CASES[name]
    gx, go = Guarded((meta["rows"], meta["hidden"]), 0), Guarded((meta["rows"], meta["hidden"]), 0)
    x = gx.load(GOLDEN[f"{name}.x"])
    w = oracle.bits_tensor(GOLDEN[f"{name}.weight"], "cuda")
    torch.ops.inference_performance_lab.rms_norm(go.tensor, x, w, meta["epsilon"])
    assert_close_to_oracle(go.tensor, GOLDEN[f"{name}.out"], name)
    assert torch.equal(x, oracle.bits_tensor(GOLDEN[f"{name}.x"], "cuda"))
    gx.assert_guards_intact()
    go.assert_guards_intact()


SWEEP = [
    *[(rows, hidden, 0, 0) for rows in (1, 5, 300) for hidden in (1, 7, 8, 64, 1001, 3584, 4096, 8192, 16384)],
    *[(37, 3584, off, off) for off in range(8)],
    *[(9, 3584, xo, oo) for xo, oo in ((0, 1), (1, 0), (3, 5))],
    (2048, 3584, 0, 0),
    (5, 40000, 0, 0),
]


@pytest.mark.parametrize("rows, hidden, x_off, out_off", SWEEP)
@torch.inference_mode()
def test_sweep_against_oracle(rows: int, hidden: int, x_off: int, out_off: int) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows * 17 + hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    gx, go = Guarded(x.shape, x_off), Guarded(x.shape, out_off)
    xin = gx.load(oracle.tensor_bits(x))
    torch.ops.inference_performance_lab.rms_norm(go.tensor, xin, w, 1e-6)
    expected = oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6)
    assert_close_to_oracle(go.tensor, expected, f"rows={rows} H={hidden} offsets={x_off},{out_off}")
    assert torch.equal(xin, x)
    gx.assert_guards_intact()
    go.assert_guards_intact()


@torch.inference_mode()
def test_in_place_and_c_abi() -> None:
    torch.manual_seed(1)
    x = torch.randn(2048, 3584, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3584, device="cuda", dtype=torch.bfloat16) * 0.1 + 1
    expected = custom_rms_norm(x, w, 1e-6)
    inplace = x.clone()
    torch.ops.inference_performance_lab.rms_norm(inplace, inplace, w, 1e-6)
    assert torch.equal(inplace, expected)
    via_c = torch.empty_like(x)
    capi.rms_norm_tensors(via_c, x, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(via_c, expected)
    assert_close_to_oracle(expected, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6), "2048x3584")


@torch.inference_mode()
def test_errors() -> None:
    x = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="identical shapes"):
        torch.ops.inference_performance_lab.rms_norm(torch.empty(4, 32, device="cuda", dtype=torch.bfloat16), x, w, 1e-6)
    with pytest.raises(RuntimeError, match="must use bfloat16"):
        torch.ops.inference_performance_lab.rms_norm(torch.empty(4, 64, device="cuda"), x, w, 1e-6)
    with pytest.raises(RuntimeError, match="epsilon must be positive"):
        torch.ops.inference_performance_lab.rms_norm(torch.empty_like(x), x, w, -1.0)
    empty = torch.empty(0, 64, device="cuda", dtype=torch.bfloat16)
    assert custom_rms_norm(empty, w, 1e-6).shape == (0, 64)


# ---- vLLM IR providers -----------------------------------------------------------------------


@pytest.mark.vllm
@torch.inference_mode()
def test_vllm_providers_dispatch_to_the_b200_kernels() -> None:
    """The reference's production caller: vLLM's IR ops with the inference_lab provider first
    in the priority list dispatch to these kernels and match the oracle; vLLM's own native
    implementation agrees within tolerance."""
    pytest.importorskip("vllm.ir")
    from vllm import ir

    from inference_performance_lab.kernels import vllm_plugin

    vllm_plugin.register()
    torch.manual_seed(2)
    x = torch.randn(512, 3584, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(3584, device="cuda", dtype=torch.bfloat16) * 0.1 + 1
    eps = 1e-6

    fused = ir.ops.fused_add_rms_norm
    with fused.set_priority([vllm_plugin.PROVIDER, "native"]):
        assert fused.dispatch(x, r, w, eps, None).provider == vllm_plugin.PROVIDER
        # variance_size is not supported: vLLM falls back to its native implementation.
        assert fused.dispatch(x, r, w, eps, 1024).provider == "native"
        xk, rk = x.clone(), r.clone()
        out, res = fused.maybe_inplace(xk, rk, w, eps, None)
    expected_out, expected_res = oracle.c_fused_add_rms_norm(
        oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), eps
    )
    np.testing.assert_array_equal(oracle.tensor_bits(res), expected_res)
    assert_close_to_oracle(out, expected_out, "vLLM fused_add_rms_norm")
    native_out, native_res = fused.impls["native"].impl_fn(x.clone(), r.clone(), w, eps, None)
    torch.testing.assert_close(out, native_out, rtol=1e-2, atol=1e-2)
    assert torch.equal(res, native_res)

    plain = ir.ops.rms_norm
    with plain.set_priority([vllm_plugin.PROVIDER, "native"]):
        assert plain.dispatch(x, w, eps, None).provider == vllm_plugin.PROVIDER
        y = plain(x, w, eps, None)
    assert_close_to_oracle(y, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), eps), "vLLM rms_norm")
    torch.testing.assert_close(y, plain.impls["native"].impl_fn(x, w, eps, None), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("tokens, hidden", [(8, 8192), (16, 16384), (4, 65536)])
@torch.inference_mode()
def test_vllm_provider_runs_the_cluster_kernel_on_long_decode_rows(tokens: int, hidden: int) -> None:
    """Decode batches of long rows through vLLM's IR ops reach the cluster kernel (each row split
    over a thread-block cluster) and match the oracle."""
    pytest.importorskip("vllm.ir")
    from vllm import ir

    from inference_performance_lab.kernels import vllm_plugin

    vllm_plugin.register()
    generator = torch.Generator(device="cuda").manual_seed(tokens + hidden)
    x = torch.randn(tokens, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(tokens, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    eps = 1e-6
    assert capi.fused_add_rms_norm_plan(x.data_ptr(), r.data_ptr(), w.data_ptr(), tokens, hidden).startswith(
        "rmsnorm_cluster_kernel")
    fused = ir.ops.fused_add_rms_norm
    with fused.set_priority([vllm_plugin.PROVIDER, "native"]):
        assert fused.dispatch(x, r, w, eps, None).provider == vllm_plugin.PROVIDER
        out, res = fused.maybe_inplace(x.clone(), r.clone(), w, eps, None)
    expected_out, expected_res = oracle.c_fused_add_rms_norm(
        oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), eps
    )
    np.testing.assert_array_equal(oracle.tensor_bits(res), expected_res)
    assert_close_to_oracle(out, expected_out, f"vLLM fused_add_rms_norm {tokens}x{hidden}")

    plain = ir.ops.rms_norm
    out_plan = torch.empty_like(x)
    assert capi.rms_norm_plan(out_plan.data_ptr(), x.data_ptr(), w.data_ptr(), tokens, hidden).startswith(
        "rmsnorm_cluster_kernel")
    with plain.set_priority([vllm_plugin.PROVIDER, "native"]):
        assert plain.dispatch(x, w, eps, None).provider == vllm_plugin.PROVIDER
        y = plain(x, w, eps, None)
    assert_close_to_oracle(y, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), eps),
                           f"vLLM rms_norm {tokens}x{hidden}")
