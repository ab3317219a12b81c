"""The reference's own CUDA kernels, built for sm_100a from its sources (oracle/build_ref_kernels.py),
as a second pin of parity on the GPU.

* On the golden inputs (made by the reference's own ``reference.py``), the reference's kernels
  reproduce the golden outputs: residual bit for bit, outputs within the reference tests'
  tolerance (rtol = atol = 1e-2) - the same bar our kernels meet in test_fused_add_rms_norm.py and
  test_silu_and_mul.py.
* On the benchmark workloads (the aligned [2048, 3584] batch of the packed kernel, the same batch
  2 bytes off 16 of the cached kernel, [1024, 8192] of the generic kernel, SiLU [128, 37888] of the
  packed SiLU kernel), ours and theirs agree: residuals bit for bit, outputs within one bf16 ulp
  of each other.

Skipped when the library has not been built (the reference checkout was absent at build time).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import build_ref_kernels, oracle
from parity import assert_bits_equal, assert_close_to_oracle, bf16_ulp_distance, require_cuda

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def ref_ops():
    require_cuda()
    if not build_ref_kernels.load():
        pytest.skip("the reference's kernels were not built (oracle/build_ref_kernels.py)")
    return torch.ops.inference_performance_lab_ref


def _golden():
    cases = json.loads((GOLDEN / "golden.json").read_text())["cases"]
    return cases, np.load(GOLDEN / "golden.npz")


@pytest.mark.parametrize("name", ["rms_config0", "rms_h8192", "rms_odd_width", "rms_tiny", "rms_one_element",
                                  "rms_large_magnitude", "rms_small_magnitude"])
def test_reference_kernels_reproduce_the_golden_rmsnorm(ref_ops, name: str) -> None:
    cases, golden = _golden()
    case = cases[name]
    x = oracle.bits_tensor(golden[f"{name}.x"], "cuda")
    r = oracle.bits_tensor(golden[f"{name}.residual"], "cuda")
    w = oracle.bits_tensor(golden[f"{name}.weight"], "cuda")
    ref_ops.fused_add_rms_norm(x, r, w, case["epsilon"])
    torch.cuda.synchronize()
    assert_bits_equal(r, golden[f"{name}.residual_out"], f"{name} residual (reference kernel)")
    assert_close_to_oracle(x, golden[f"{name}.out"], f"{name} output (reference kernel)", max_ulp=2)


@pytest.mark.parametrize("name", ["silu_width18944", "silu_reference_recipe", "silu_odd_width", "silu_tiny"])
def test_reference_kernels_reproduce_the_golden_silu(ref_ops, name: str) -> None:
    _, golden = _golden()
    xin = oracle.bits_tensor(golden[f"{name}.input"], "cuda")
    inter = xin.shape[-1] // 2
    out = torch.empty(*xin.shape[:-1], inter, dtype=torch.bfloat16, device="cuda")
    ref_ops.silu_and_mul(out, xin)  # the reference's scalar kernel: any width
    torch.cuda.synchronize()
    assert_close_to_oracle(out, golden[f"{name}.out"], f"{name} (reference kernel)", max_ulp=2)


def _fused_inputs(rows: int, hidden: int, offset: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    bufs = [torch.randn(rows * hidden + 8, device="cuda", dtype=torch.bfloat16, generator=generator) for _ in range(2)]
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    x, r = (b[offset: offset + rows * hidden].view(rows, hidden) for b in bufs)
    return x, r, w


@pytest.mark.parametrize(("rows", "hidden", "offset", "eps"),
                         [(2048, 3584, 0, 1e-6), (2048, 3584, 1, 1e-6), (1024, 8192, 0, 1e-5)],
                         ids=["packed-3584", "cached-3584-misaligned", "generic-8192"])
def test_ours_and_the_reference_kernels_agree(ref_ops, rows: int, hidden: int, offset: int, eps: float) -> None:
    x, r, w = _fused_inputs(rows, hidden, offset, seed=rows + offset)
    x2, r2 = x.clone(), r.clone()
    torch.ops.inference_performance_lab.fused_add_rms_norm(x, r, w, eps)
    ref_ops.fused_add_rms_norm(x2, r2, w, eps)
    torch.cuda.synchronize()
    assert np.array_equal(oracle.tensor_bits(r), oracle.tensor_bits(r2)), "residuals differ"
    distance = bf16_ulp_distance(oracle.tensor_bits(x).reshape(-1), oracle.tensor_bits(x2).reshape(-1))
    assert int(distance.max()) <= 1, f"outputs {int(distance.max())} ulps apart"


def test_ours_and_the_reference_silu_kernels_agree(ref_ops) -> None:
    generator = torch.Generator(device="cuda").manual_seed(7)
    xin = (torch.randn(128, 37888, device="cuda", generator=generator) * 2.0).to(torch.bfloat16)
    ours = torch.empty(128, 18944, dtype=torch.bfloat16, device="cuda")
    theirs = torch.empty_like(ours)
    torch.ops.inference_performance_lab.silu_and_mul(ours, xin)
    ref_ops.silu_and_mul_packed(theirs, xin)
    torch.cuda.synchronize()
    distance = bf16_ulp_distance(oracle.tensor_bits(ours).reshape(-1), oracle.tensor_bits(theirs).reshape(-1))
    assert int(distance.max()) <= 1, f"outputs {int(distance.max())} ulps apart"
