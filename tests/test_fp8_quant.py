"""GPU parity of add+RMSNorm with a static fp8 (e4m3) output against the oracle.

Not an op of the reference library (its scope lists it next: the fused variant feeding an fp8
GEMM). The residual is bit-exact; the e4m3 output is within one e4m3 step of the oracle (the
fp32 mean may differ in its last bit) and all but a few per mille of its bytes are identical.
Byte canaries guard the fp8 output, bf16 canaries the inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from inference_performance_lab.kernels.extension import fused_add_rms_norm_static_fp8_quant
from oracle import oracle
from parity import Guarded, assert_bits_equal, require_cuda

pytestmark = pytest.mark.gpu

BYTE_CANARY = 0x5A


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


def e4m3_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Steps between e4m3 codes on the ordered number line (sign-magnitude to offset)."""
    def ordered(v: np.ndarray) -> np.ndarray:
        v = v.astype(np.int32)
        return np.where(v & 0x80, -(v & 0x7F), v)

    return np.abs(ordered(a) - ordered(b))


def check(out8: np.ndarray, expected: np.ndarray, what: str) -> None:
    distance = e4m3_distance(out8.reshape(-1), expected.reshape(-1))
    assert int(distance.max(initial=0)) <= 1, f"{what}: {int(distance.max())} e4m3 steps from the oracle"
    assert int((distance > 0).sum()) <= max(2, out8.size // 200), f"{what}: {(distance > 0).sum()} bytes differ"


CASES = [
    # rows, hidden, x/residual offset (elements), output offset (bytes), scale
    (2048, 3584, 0, 0, 0.05),     # stash kernel (a CTA per row, chunks in registers)
    (7, 3584, 0, 0, 1.0),         # CTA-per-row kernel
    (3000, 8192, 0, 0, 0.02),     # stash kernel, 256 threads a row
    (600, 16384, 0, 0, 0.05),     # stash kernel, 512 threads a row
    (300, 16392, 0, 0, 0.05),     # stash kernel, eight chunks a thread, 96 registers
    (100, 24576, 0, 0, 0.05),     # stash kernel, eight chunks a thread, 128 registers
    (1000, 1024, 0, 0, 0.05),     # CTA-per-row kernel (every CTA resident at once)
    (5000, 512, 0, 0, 0.05),      # warp-per-row kernel (3.5 KiB a row)
    (3000, 1024, 0, 0, 0.05),     # stash kernel (7 KiB a row)
    (5, 256, 0, 0, 0.5),
    (64, 3584, 1, 0, 0.05),       # rows not 16-byte aligned: general row kernel
    (64, 3584, 0, 3, 0.05),       # output not 8-byte aligned
    (9, 1001, 0, 0, 0.05),        # odd width
    (3, 40000, 0, 0, 0.05),       # two-pass row kernel
]


@pytest.mark.parametrize("rows, hidden, in_off, out_off, scale", CASES)
@torch.inference_mode()
def test_against_oracle(rows: int, hidden: int, in_off: int, out_off: int, scale: float) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows + hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    gx, gr = Guarded(x.shape, in_off), Guarded(x.shape, in_off)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    storage = torch.full((4096 + out_off + rows * hidden + 4096,), BYTE_CANARY, dtype=torch.uint8, device="cuda")
    out = storage[4096 + out_off: 4096 + out_off + rows * hidden].view(torch.float8_e4m3fn).view(rows, hidden)
    scale_t = torch.tensor([scale], dtype=torch.float32, device="cuda")
    torch.ops.inference_performance_lab.fused_add_rms_norm_static_fp8_quant(out, ax, ar, w, scale_t, 1e-6)
    expected8, expected_res = oracle.c_fused_add_rms_norm_static_fp8_quant(
        oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), scale, 1e-6
    )
    assert_bits_equal(ar, expected_res, f"{rows}x{hidden} residual")
    check(out.view(torch.uint8).cpu().numpy(), expected8, f"{rows}x{hidden}")
    assert torch.equal(ax, x), "input must not be modified"
    assert bool((storage[: 4096 + out_off] == BYTE_CANARY).all())
    assert bool((storage[4096 + out_off + rows * hidden:] == BYTE_CANARY).all())
    gx.assert_guards_intact()
    gr.assert_guards_intact()


@torch.inference_mode()
def test_saturation_and_wrapper() -> None:
    torch.manual_seed(3)
    x = torch.randn(64, 4096, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.ones(4096, device="cuda", dtype=torch.bfloat16)
    # A tiny scale pushes most outputs past 448: they saturate to +-448 (0x7E / 0xFE), never NaN.
    scale = torch.tensor([1e-3], device="cuda")
    out = fused_add_rms_norm_static_fp8_quant(x, r.clone(), w, scale, 1e-6)
    codes = out.view(torch.uint8)
    assert not bool(((codes & 0x7F) == 0x7F).any())
    assert bool(((codes == 0x7E) | (codes == 0xFE)).float().mean() > 0.5)
    # The same call through the C ABI.
    r2 = r.clone()
    out2 = torch.empty_like(out)
    capi.fused_add_rms_norm_static_fp8_quant(
        out2.data_ptr(), x.data_ptr(), r2.data_ptr(), w.data_ptr(), scale.data_ptr(), 64, 4096, 1e-6,
        torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    assert torch.equal(out2.view(torch.uint8), codes)


@torch.inference_mode()
def test_errors() -> None:
    x = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    scale = torch.ones(1, device="cuda")
    op = torch.ops.inference_performance_lab.fused_add_rms_norm_static_fp8_quant
    with pytest.raises(RuntimeError, match="result must use float8_e4m3fn"):
        op(torch.empty_like(x), x, x.clone(), w, scale, 1e-6)
    with pytest.raises(RuntimeError, match="scale must be a single float32"):
        op(torch.empty(4, 64, device="cuda", dtype=torch.float8_e4m3fn), x, x.clone(), w, torch.ones(2, device="cuda"), 1e-6)
