"""GPU parity of the few-rows kernel (a CTA per row, values in registers; H % 8 == 0, 16-byte
aligned rows, 1024 < H <= 16384, decode-sized row counts, and with one chunk a thread as many rows
as have their CTAs resident at once) for the fused op, plain RMSNorm and the fp8-output op,
against the oracle, with canary guards and a misaligned weight."""

from __future__ import annotations

import pytest
import torch

from inference_performance_lab.kernels import capi
from oracle import oracle
from parity import Guarded, assert_bits_equal, assert_close_to_oracle, require_cuda
from test_fp8_quant import BYTE_CANARY, check

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


HIDDEN = (1032, 1536, 2048, 3584, 4096, 5120, 8192, 12288, 16384)
# Rows of 8192+ elements: row counts the planner keeps on this kernel (fewer rows, and at 12288+
# more rows than SMs, go to the cluster kernel).
ROWS = {hidden: (1, 3, 64, 256) if hidden < 8192 else (33, 64, 256) if hidden < 12288 else (33, 64, 148)
        for hidden in HIDDEN}
CASES = [(rows, hidden, w_off) for hidden in HIDDEN for rows in ROWS[hidden] for w_off in (0, 1)
         if w_off == 0 or rows == ROWS[hidden][1]]
# One chunk a thread: up to the rows whose CTAs an SM holds at once (148 SMs x 8 / 8 / 6 / 3 / 3);
# from H = 1536 with a weight off 16 bytes (the 256-bit stash kernel takes an aligned one).
CASES += [(1184, 1032, 0), (1184, 1536, 1), (888, 2048, 1), (444, 3584, 1), (400, 3584, 1), (444, 4096, 1)]


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize("rows, hidden, w_off", CASES)
@torch.inference_mode()
def test_fused_few_rows(rows: int, hidden: int, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 3 * hidden + w_off)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_cta_kernel"), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden, w_off", CASES)
@torch.inference_mode()
def test_plain_few_rows(rows: int, hidden: int, w_off: int) -> None:
    x, _, w = _inputs(rows, hidden, rows + 5 * hidden + w_off)
    gx, go, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, aw = gx.load(oracle.tensor_bits(x)), gw.load(oracle.tensor_bits(w))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_cta_kernel"), plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, aw, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}")
    torch.ops.inference_performance_lab.rms_norm(ax, ax, aw, 1e-6)  # in place
    assert torch.equal(ax, go.tensor)
    for g in (gx, go, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(1, 3584), (7, 3584), (256, 4096), (33, 16384), (5, 1032), (296, 3576),
                                         (592, 2040)])
@torch.inference_mode()
def test_fp8_few_rows(rows: int, hidden: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 7 * hidden)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    storage = torch.full((4096 + rows * hidden + 4096,), BYTE_CANARY, dtype=torch.uint8, device="cuda")
    out = storage[4096: 4096 + rows * hidden].view(torch.float8_e4m3fn).view(rows, hidden)
    plan = capi.fused_add_rms_norm_static_fp8_quant_plan(out.data_ptr(), ax.data_ptr(), ar.data_ptr(),
                                                         w.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_cta_kernel"), plan
    scale = 0.05
    scale_t = torch.tensor([scale], dtype=torch.float32, device="cuda")
    torch.ops.inference_performance_lab.fused_add_rms_norm_static_fp8_quant(out, ax, ar, w, scale_t, 1e-6)
    expected8, expected_res = oracle.c_fused_add_rms_norm_static_fp8_quant(
        oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), scale, 1e-6
    )
    assert_bits_equal(ar, expected_res, f"{rows}x{hidden} residual")
    check(out.view(torch.uint8).cpu().numpy(), expected8, f"{rows}x{hidden}")
    assert torch.equal(ax, x), "input must not be modified"
    assert bool((storage[:4096] == BYTE_CANARY).all())
    assert bool((storage[4096 + rows * hidden:] == BYTE_CANARY).all())


@torch.inference_mode()
def test_graph_capture_and_chained_launches() -> None:
    """Back-to-back dependent launches (each reads what the previous one wrote) replayed from a
    CUDA graph give the bits of the same launches run eagerly; the first matches the oracle."""
    rows, hidden = 8, 3584
    x, r, w = _inputs(rows, hidden, 11)
    ex, er = x.clone(), r.clone()
    for step in range(3):
        torch.ops.inference_performance_lab.fused_add_rms_norm(ex, er, w, 1e-6)
        if step == 0:
            out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r),
                                                   oracle.tensor_bits(w), 1e-6)
            assert_bits_equal(er, res, "residual after one launch")
            assert_close_to_oracle(ex, out, "output after one launch")
    gx, gr = x.clone(), r.clone()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(3):
                torch.ops.inference_performance_lab.fused_add_rms_norm(gx, gr, w, 1e-6)
    gx.copy_(x)
    gr.copy_(r)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gx, ex) and torch.equal(gr, er)
    del graph
