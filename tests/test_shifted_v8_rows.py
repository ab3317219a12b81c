"""GPU parity of the shifted kernel with 256-bit accesses (add+RMSNorm rows that start P = 1..7
elements into a 32-byte block, x and residual alike, so that the aligned chunks covering each row
pair up into 32-byte blocks; H % 16 == 0, 1536 <= H <= 4080, 257-4096 rows, a 16-byte aligned
weight) against the oracle: every phase, the edges of the width and row ranges, canary guards
around every tensor (the first and last chunk of each row are shared with the neighbouring rows
and the guards), and dependent launches queued back to back and replayed from a CUDA graph."""

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


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


# (rows, hidden, phase): the bench's misaligned workload, every phase, the width and row edges,
# odd thread counts (H / 16 + 1 pairs: 3584 -> 225, 1552 -> 98, 4064 -> 255, 4080 -> 256).
CASES = ([(2048, 3584, 1)] + [(700, 3584, off) for off in range(2, 8)] +
         [(257, 1536, 3), (4096, 2048, 5), (300, 1552, 1), (1000, 4080, 7), (600, 4064, 2), (1500, 2560, 4)])


@pytest.mark.parametrize("rows, hidden, off", CASES)
@torch.inference_mode()
def test_fused_shifted_v8_rows(rows: int, hidden: int, off: int) -> None:
    x, r, w = _inputs(rows, hidden, 5 * rows + hidden + 13 * off)
    gx, gr = Guarded(x.shape, off), Guarded(x.shape, off)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), w.data_ptr(), rows, hidden)
    assert plan == f"rmsnorm_shifted_v8_kernel<{off}>", plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, w, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden}+{off} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden}+{off} output")
    gx.assert_guards_intact()
    gr.assert_guards_intact()


@torch.inference_mode()
def test_chained_launches_queued_and_in_a_graph() -> None:
    """Three dependent launches on the misaligned workload's views: one at a time, each matches
    the oracle on the bits it was given; queued back to back and from a CUDA graph, the same bits."""
    rows, hidden, off = 2048, 3584, 1
    x, r, w = _inputs(rows, hidden, 29)
    gx, gr = Guarded(x.shape, off), Guarded(x.shape, off)
    sx, sr = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    for step in range(3):
        bx, br = oracle.tensor_bits(sx), oracle.tensor_bits(sr)
        torch.ops.inference_performance_lab.fused_add_rms_norm(sx, sr, w, 1e-6)
        torch.cuda.synchronize()
        out, res = oracle.c_fused_add_rms_norm(bx, br, oracle.tensor_bits(w), 1e-6)
        assert_bits_equal(sr, res, f"residual after launch {step + 1}")
        assert_close_to_oracle(sx, out, f"output after launch {step + 1}")
    qx_g, qr_g = Guarded(x.shape, off), Guarded(x.shape, off)
    qx, qr = qx_g.load(oracle.tensor_bits(x)), qr_g.load(oracle.tensor_bits(r))
    for _ in range(3):
        torch.ops.inference_performance_lab.fused_add_rms_norm(qx, qr, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(qx, sx) and torch.equal(qr, sr)
    hx_g, hr_g = Guarded(x.shape, off), Guarded(x.shape, off)
    hx, hr = hx_g.load(oracle.tensor_bits(x)), hr_g.load(oracle.tensor_bits(r))
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(3):
                torch.ops.inference_performance_lab.fused_add_rms_norm(hx, hr, w, 1e-6)
    hx.copy_(x)
    hr.copy_(r)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(hx, sx) and torch.equal(hr, sr)
    for g in (gx, gr, qx_g, qr_g, hx_g, hr_g):
        g.assert_guards_intact()
    del graph
