"""GPU parity of the cluster kernel (a row split over a thread-block cluster of 2-8 CTAs that
exchange their partial sums of squares through distributed shared memory; H % 8 == 0, 16-byte
aligned rows): aligned rows longer than 32768 elements, which the stash kernel cannot hold, and
launches of a few long rows. Fused op, plain RMSNorm (out of place and in place) and the fp8-output
op against the oracle, with canary guards, a misaligned weight, slices that do not divide the row
evenly, the widest row (131072), and chained launches queued back to back and from a CUDA graph."""

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


# (rows, hidden, the plan's chunks a thread). Cluster sizes by the planner: 8 CTAs a row up to
# 16 rows and beyond H = 32768; otherwise fewer as the launch grows (see the comments).
CASES = [
    (1, 8192, 1),       # 8 CTAs of 128 threads, one chunk each
    (32, 8192, 2),      # 4 CTAs a row
    (16, 6144, 1),      # 8 CTAs of 96 threads
    (8, 12288, 1),
    (200, 12288, 4),    # more rows than SMs: 2 CTAs a row of 768 chunks, 192 threads of four
    (256, 16384, 4),    # 2 CTAs a row of 1024 chunks, 256 threads of four
    (1, 20480, 2),
    (256, 32768, 4),    # 2 CTAs a row, 512 threads of four chunks
    (7, 32776, 4),      # 4097 chunks: the last CTA's slice is shorter
    (3, 40000, 4),
    (5, 65544, 4),      # 8193 chunks over 8 CTAs of 288 threads
    (64, 65536, 4),
    (600, 49152, 4),    # many rows of a long width: 4800 clusters
    (1, 131072, 4),     # the widest: 8 CTAs of 512 threads x 4 chunks
    (2, 131064, 4),
]


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize("w_off", [0, 1])
@pytest.mark.parametrize("rows, hidden, per_thread", CASES)
@torch.inference_mode()
def test_fused_cluster_rows(rows: int, hidden: int, per_thread: int, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 3 * hidden + w_off)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan == f"rmsnorm_cluster_kernel<{per_thread}>", plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(1, 8192), (8, 16384), (100, 32768), (5, 65544), (300, 40960),
                                         (1, 131072)])
@torch.inference_mode()
def test_plain_cluster_rows(rows: int, hidden: int) -> None:
    # Out of place, then in place (each thread reads its chunks before it writes them).
    x, _, w = _inputs(rows, hidden, rows + 5 * hidden)
    gx, go = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax = gx.load(oracle.tensor_bits(x))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), w.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_cluster_kernel") and plan.endswith(", plain>"), plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, w, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}")
    torch.ops.inference_performance_lab.rms_norm(ax, ax, w, 1e-6)  # in place
    assert torch.equal(ax, go.tensor)
    gx.assert_guards_intact()
    go.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(1, 8192), (200, 16384), (64, 32768), (7, 32776), (96, 65536)])
@torch.inference_mode()
def test_fp8_cluster_rows(rows: int, hidden: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 7 * hidden)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    storage = torch.full((4096 + rows * hidden + 4096,), BYTE_CANARY, dtype=torch.uint8, device="cuda")
    out = storage[4096: 4096 + rows * hidden].view(torch.float8_e4m3fn).view(rows, hidden)
    plan = capi.fused_add_rms_norm_static_fp8_quant_plan(out.data_ptr(), ax.data_ptr(), ar.data_ptr(),
                                                         w.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_cluster_kernel") and plan.endswith(", fp8>"), plan
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


@pytest.mark.parametrize("rows, hidden", [(8, 16384), (64, 65536)])
@torch.inference_mode()
def test_chained_launches_queued_and_in_a_graph(rows: int, hidden: int) -> None:
    """Three dependent launches (each reads what the previous one wrote). One at a time with a
    synchronize between them, each matches the oracle on the bits it was given; queued back to
    back (the next launch's CTAs may start while the previous drains) and replayed from a CUDA
    graph they give the same bits."""
    x, r, w = _inputs(rows, hidden, rows + hidden)
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


@torch.inference_mode()
def test_every_cta_of_a_row_normalises_with_the_same_scale() -> None:
    """A row whose slices differ wildly in magnitude (each CTA's partial sum is different): the
    output of every slice must use the one inverse RMS of the whole row."""
    rows, hidden = 4, 65536
    x, r, w = _inputs(rows, hidden, 5)
    x = x * torch.linspace(0.01, 100.0, hidden, device="cuda").to(torch.bfloat16)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    assert capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), w.data_ptr(), rows, hidden) == \
        "rmsnorm_cluster_kernel<4>"
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, w, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, "residual")
    assert_close_to_oracle(ax, out, "output")
    gx.assert_guards_intact()
    gr.assert_guards_intact()


@pytest.mark.parametrize("scale", [300.0, 1e-4])
@pytest.mark.parametrize("rows, hidden", [(2, 65536), (8, 16384)])
@torch.inference_mode()
def test_extreme_magnitudes(rows: int, hidden: int, scale: float) -> None:
    """The golden vectors' large- and small-magnitude recipes (x and residual scaled by 300 and by
    1e-4, where eps dominates the mean of squares) at widths the cluster kernel takes."""
    x, r, w = _inputs(rows, hidden, int(scale * 7) + hidden)
    x = (x.float() * scale).to(torch.bfloat16)
    r = (r.float() * scale).to(torch.bfloat16)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    assert capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), w.data_ptr(), rows, hidden).startswith(
        "rmsnorm_cluster_kernel")
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, w, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} x{scale:g} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} x{scale:g} output")
    gx.assert_guards_intact()
    gr.assert_guards_intact()
