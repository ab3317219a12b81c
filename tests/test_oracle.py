"""The CPU oracle, pinned against golden vectors produced by the reference's own reference.py.

The golden file (tests/golden/golden.npz, made by tests/golden/make_golden.py) holds inputs and
outputs of src/inference_performance_lab/kernels/reference.py evaluated on CPU. Both oracle
restatements must reproduce them bit for bit; the kernels are then checked against the oracle.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN = np.load(GOLDEN_DIR / "golden.npz")
CASES = json.loads((GOLDEN_DIR / "golden.json").read_text())["cases"]
RMS_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "fused_add_rms_norm")
SILU_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "silu_and_mul")
PLAIN_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "rms_norm")


def test_golden_covers_the_reference_cpu_configuration() -> None:
    meta = CASES["rms_config0"]
    assert (meta["rows"], meta["hidden"], meta["epsilon"]) == (8, 3584, 1e-6)
    assert CASES["silu_width18944"]["intermediate"] == 18944


@pytest.mark.parametrize("name", RMS_CASES)
def test_c_oracle_matches_reference_rms(name: str) -> None:
    out, res = oracle.c_fused_add_rms_norm(
        GOLDEN[f"{name}.x"], GOLDEN[f"{name}.residual"], GOLDEN[f"{name}.weight"],
        CASES[name]["epsilon"],
    )
    np.testing.assert_array_equal(res, GOLDEN[f"{name}.residual_out"])
    np.testing.assert_array_equal(out, GOLDEN[f"{name}.out"])


@pytest.mark.parametrize("name", PLAIN_CASES)
def test_oracles_match_reference_plain_rms_norm(name: str) -> None:
    x, w, eps = GOLDEN[f"{name}.x"], GOLDEN[f"{name}.weight"], CASES[name]["epsilon"]
    np.testing.assert_array_equal(oracle.c_rms_norm(x, w, eps), GOLDEN[f"{name}.out"])
    out = oracle.torch_rms_norm(oracle.bits_tensor(x), oracle.bits_tensor(w), eps)
    np.testing.assert_array_equal(oracle.tensor_bits(out), GOLDEN[f"{name}.out"])


@pytest.mark.parametrize("name", SILU_CASES)
def test_c_oracle_matches_reference_silu(name: str) -> None:
    out = oracle.c_silu_and_mul(GOLDEN[f"{name}.input"])
    np.testing.assert_array_equal(out, GOLDEN[f"{name}.out"])


@pytest.mark.parametrize("name", RMS_CASES)
def test_torch_port_matches_reference_rms(name: str) -> None:
    out, res = oracle.torch_fused_add_rms_norm(
        oracle.bits_tensor(GOLDEN[f"{name}.x"]),
        oracle.bits_tensor(GOLDEN[f"{name}.residual"]),
        oracle.bits_tensor(GOLDEN[f"{name}.weight"]),
        CASES[name]["epsilon"],
    )
    np.testing.assert_array_equal(oracle.tensor_bits(res), GOLDEN[f"{name}.residual_out"])
    np.testing.assert_array_equal(oracle.tensor_bits(out), GOLDEN[f"{name}.out"])


@pytest.mark.parametrize("name", SILU_CASES)
def test_torch_port_matches_reference_silu(name: str) -> None:
    out = oracle.torch_silu_and_mul(oracle.bits_tensor(GOLDEN[f"{name}.input"]))
    np.testing.assert_array_equal(oracle.tensor_bits(out), GOLDEN[f"{name}.out"])


def test_oracles_agree_on_fresh_seeded_inputs() -> None:
    generator = torch.Generator().manual_seed(1234)
    for rows, hidden in [(3, 4096), (2, 5120), (7, 33)]:
        x = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        r = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        w = (torch.randn(hidden, generator=generator) * 0.1 + 1).to(torch.bfloat16)
        t_out, t_res = oracle.torch_fused_add_rms_norm(x, r, w, 1e-6)
        c_out, c_res = oracle.c_fused_add_rms_norm(
            oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6
        )
        np.testing.assert_array_equal(c_res, oracle.tensor_bits(t_res))
        # The mean may differ in the last fp32 bit (torch sums in fp32, the C oracle in double):
        # at most one bf16 ulp, in few elements.
        diff = np.abs(oracle.bf16_bits_to_f32(c_out) - t_out.float().numpy())
        assert float(diff.max()) <= 2.0 ** -7 * float(np.abs(t_out.float().numpy()).max())


def test_bf16_rounding_matches_torch() -> None:
    generator = torch.Generator().manual_seed(7)
    values = torch.cat(
        [
            torch.randn(100000, generator=generator) * 10,
            torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 1e-40, -1e-40, 3.4e38, 1.0 + 2**-8,
                          1.0 + 2**-7 + 2**-8, 1.0 + 2**-8 + 2**-20]),
        ]
    )
    expected = oracle.tensor_bits(values.to(torch.bfloat16))
    np.testing.assert_array_equal(oracle.f32_to_bf16_bits(values.numpy()), expected)
    # Every NaN narrows to the canonical 0x7FC0, as c10::BFloat16 does.
    assert oracle.f32_to_bf16_bits(np.array([np.nan], dtype=np.float32))[0] == 0x7FC0


def test_reference_rejects_odd_final_dimension() -> None:
    with pytest.raises(ValueError, match="final tensor dimension must be even"):
        oracle.torch_silu_and_mul(torch.empty((2, 7)))
    with pytest.raises(ValueError, match="final tensor dimension must be even"):
        oracle.c_silu_and_mul(np.zeros((2, 7), dtype=np.uint16))


def test_oracle_rejects_mismatched_shapes() -> None:
    x = np.zeros((2, 8), dtype=np.uint16)
    with pytest.raises(ValueError, match="identical shapes"):
        oracle.c_fused_add_rms_norm(x, np.zeros((2, 9), dtype=np.uint16), np.zeros(8, np.uint16), 1e-6)
    with pytest.raises(ValueError, match="final tensor dimension"):
        oracle.c_fused_add_rms_norm(x, x, np.zeros(9, np.uint16), 1e-6)


def test_oracle_empty_batch() -> None:
    out, res = oracle.c_fused_add_rms_norm(
        np.zeros((0, 16), np.uint16), np.zeros((0, 16), np.uint16), np.zeros(16, np.uint16), 1e-6
    )
    assert out.shape == res.shape == (0, 16)


def test_e4m3_conversion_matches_torch() -> None:
    generator = torch.Generator().manual_seed(11)
    values = torch.cat(
        [torch.randn(5000, generator=generator) * s for s in (1e-4, 1e-2, 1.0, 30.0, 200.0)]
        + [torch.tensor([0.0, -0.0, 448.0, -448.0, 447.9, 2.0**-9, 2.0**-10, 1.5 * 2.0**-9, 2.0**-6,
                         0.0146484375, 240.0, 232.0, 248.0, 1.0625, 1.1875])]
    ).clamp(-448.0, 448.0)
    expected = values.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(oracle.c_f32_to_e4m3(values.numpy()), expected)
    # Saturation (torch would give NaN beyond 448; the op saturates, as vLLM's does) and NaN.
    np.testing.assert_array_equal(
        oracle.c_f32_to_e4m3(np.array([1e6, -1e6, 464.0, np.nan], dtype=np.float32)),
        np.array([0x7E, 0xFE, 0x7E, 0x7F], dtype=np.uint8),
    )


def test_fp8_quant_oracles_agree() -> None:
    generator = torch.Generator().manual_seed(12)
    for rows, hidden, scale in [(16, 1024, 0.05), (3, 3584, 0.01), (4, 1001, 1.0)]:
        x = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        r = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        w = (torch.randn(hidden, generator=generator) * 0.1 + 1).to(torch.bfloat16)
        c_out, c_res = oracle.c_fused_add_rms_norm_static_fp8_quant(
            oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), scale, 1e-6
        )
        t_out, t_res = oracle.torch_fused_add_rms_norm_static_fp8_quant(x, r, w, scale, 1e-6)
        np.testing.assert_array_equal(c_res, oracle.tensor_bits(t_res))
        mismatches = int((c_out != t_out.view(torch.uint8).numpy()).sum())
        assert mismatches <= c_out.size // 1000  # the fp32 mean may differ in its last bit
