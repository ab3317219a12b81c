"""GPU parity of short rows (H <= 1024, 16-byte aligned) for the fused op and plain RMSNorm, against
the oracle, with canary guards: a CTA per row while every row's CTA is resident at once (here up
to 1000 rows), then a warp per row (eight rows a CTA) for rows that move under 7 KiB through HBM,
and the stash kernel for add+RMSNorm rows of 896 and more."""

from __future__ import annotations

import pytest
import torch

from inference_performance_lab.kernels import capi
from oracle import oracle
from parity import Guarded, assert_bits_equal, assert_close_to_oracle, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


CASES = [(rows, hidden) for hidden in (8, 248, 256, 264, 512, 1000, 1024) for rows in (1, 7, 1000, 20000)]


def expected_kernel(rows: int, hidden: int, bytes_per_element: int) -> str:
    if rows <= 1000:
        return "rmsnorm_cta_kernel"
    return "rmsnorm_warp_kernel" if bytes_per_element * hidden < 7168 else "rmsnorm_stash_kernel"


@pytest.mark.parametrize("rows, hidden", CASES)
@torch.inference_mode()
def test_fused_short_rows(rows: int, hidden: int) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows + 3 * hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, 1)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan.startswith(expected_kernel(rows, hidden, 8)), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", CASES)
@torch.inference_mode()
def test_plain_short_rows(rows: int, hidden: int) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows + 5 * hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    gx, go = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax = gx.load(oracle.tensor_bits(x))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), w.data_ptr(), rows, hidden)
    assert plan.startswith(expected_kernel(rows, hidden, 4)), plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, w, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}")
    # In place.
    torch.ops.inference_performance_lab.rms_norm(ax, ax, w, 1e-6)
    assert torch.equal(ax, go.tensor)
    gx.assert_guards_intact()
    go.assert_guards_intact()
