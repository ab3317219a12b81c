"""GPU parity of the stash kernel with 256-bit accesses (a CTA for every row, one 32-byte pair of
chunks a thread; H % 16 == 0, 32-byte aligned rows, a 16-byte aligned weight, 1536 <= H <= 5120,
257-4096 rows) for the fused op and the fp8-output op, against the oracle, with canary guards and
chained launches replayed from a CUDA graph; the same shapes with a misaligned weight, which the
planner gives to the other kernels."""

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


# (rows, hidden): the bench workload, the edges of the width and row ranges, odd thread counts
# (H / 16 not a multiple of 32: 1552 -> 97 pairs, 5104 -> 319), one to several resident waves.
CASES = [(2048, 3584), (257, 3584), (445, 3584), (1024, 3584), (4096, 3584), (2048, 2048), (4096, 1536),
         (300, 1552), (3000, 2560), (2000, 3072), (2000, 4096), (1500, 5120), (700, 5104)]


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize("w_off", [0, 1])
@pytest.mark.parametrize("rows, hidden", CASES)
@torch.inference_mode()
def test_fused_v8_rows(rows: int, hidden: int, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 3 * hidden + w_off)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    if w_off == 0:
        assert plan == "rmsnorm_stash_v8_kernel", plan
    else:
        assert plan.startswith(("rmsnorm_stash_kernel<4>", "rmsnorm_cta_kernel")), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(2048, 3584), (300, 1536), (4096, 2048), (1000, 5120), (700, 5104)])
@torch.inference_mode()
def test_fp8_v8_rows(rows: int, hidden: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 7 * hidden)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    storage = torch.full((4096 + rows * hidden + 4096,), BYTE_CANARY, dtype=torch.uint8, device="cuda")
    out = storage[4096: 4096 + rows * hidden].view(torch.float8_e4m3fn).view(rows, hidden)
    plan = capi.fused_add_rms_norm_static_fp8_quant_plan(out.data_ptr(), ax.data_ptr(), ar.data_ptr(),
                                                         w.data_ptr(), rows, hidden)
    assert plan == "rmsnorm_stash_v8_kernel<fp8>", plan
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
def test_chained_launches_queued_and_in_a_graph() -> None:
    """Three dependent launches: one at a time, each matches the oracle on the bits it was given;
    queued back to back and replayed from a CUDA graph they give the same bits."""
    rows, hidden = 2048, 3584
    x, r, w = _inputs(rows, hidden, 17)
    sx, sr = x.clone(), r.clone()
    for step in range(3):
        bx, br = oracle.tensor_bits(sx), oracle.tensor_bits(sr)
        torch.ops.inference_performance_lab.fused_add_rms_norm(sx, sr, w, 1e-6)
        torch.cuda.synchronize()
        out, res = oracle.c_fused_add_rms_norm(bx, br, oracle.tensor_bits(w), 1e-6)
        assert_bits_equal(sr, res, f"residual after launch {step + 1}")
        assert_close_to_oracle(sx, out, f"output after launch {step + 1}")
    qx, qr = x.clone(), r.clone()
    for _ in range(3):
        torch.ops.inference_performance_lab.fused_add_rms_norm(qx, qr, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(qx, sx) and torch.equal(qr, sr)
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
    assert torch.equal(gx, sx) and torch.equal(gr, sr)
    del graph
