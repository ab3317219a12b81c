"""GPU parity of the many-rows kernel (a small CTA for every row whose threads keep their chunks
in registers; H % 8 == 0, 16-byte aligned rows, 1024 < H <= 12288, more than 256 rows) for the
fused op, plain RMSNorm (four chunks a thread, and eight for 4096+ rows of 8192+ elements) and
the fp8-output op, against the oracle, with canary guards and a misaligned weight. The fused and
fp8 cases of 1536-5120 elements use more than 4096 rows (fewer go to the 256-bit kernel,
tests/test_stash_v8_rows.py) or a misaligned weight."""

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


# (rows, hidden): one, two and four chunks a thread, odd thread counts (H / 32 not a power of 2),
# the largest width the planner gives this kernel.
CASES = [(1600, 1032), (4100, 1536), (4200, 2560), (4500, 3584), (5000, 4096), (4200, 5120), (800, 8192),
         (500, 12288), (2100, 3592), (2200, 1032)]


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize("w_off", [0, 1])
@pytest.mark.parametrize("rows, hidden", CASES)
@torch.inference_mode()
def test_fused_many_rows(rows: int, hidden: int, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 3 * hidden + w_off)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_stash_kernel"), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(1600, 1032), (3000, 1536), (5000, 2048), (2100, 3584), (700, 8192),
                                         (300, 12288), (4100, 8192), (4096, 12288)])
@torch.inference_mode()
def test_plain_many_rows(rows: int, hidden: int) -> None:
    # Out of place, then in place (each thread reads its chunks before it writes them).
    x, _, w = _inputs(rows, hidden, rows + 5 * hidden)
    gx, go = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax = gx.load(oracle.tensor_bits(x))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), w.data_ptr(), rows, hidden)
    wide = hidden >= 8192 and rows >= 4096
    assert plan == ("rmsnorm_stash_kernel<8, plain>" if wide else "rmsnorm_stash_kernel<4, plain>"), plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, w, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}")
    torch.ops.inference_performance_lab.rms_norm(ax, ax, w, 1e-6)  # in place
    assert torch.equal(ax, go.tensor)
    gx.assert_guards_intact()
    go.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(4500, 3584), (800, 8192), (4200, 1536), (1000, 1032), (500, 12288),
                                         (297, 3576)])
@torch.inference_mode()
def test_fp8_many_rows(rows: int, hidden: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + 7 * hidden)
    gx, gr = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax, ar = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    storage = torch.full((4096 + rows * hidden + 4096,), BYTE_CANARY, dtype=torch.uint8, device="cuda")
    out = storage[4096: 4096 + rows * hidden].view(torch.float8_e4m3fn).view(rows, hidden)
    plan = capi.fused_add_rms_norm_static_fp8_quant_plan(out.data_ptr(), ax.data_ptr(), ar.data_ptr(),
                                                         w.data_ptr(), rows, hidden)
    assert plan.startswith("rmsnorm_stash_kernel"), plan
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
def test_graph_replay_matches_eager() -> None:
    rows, hidden = 2100, 3584
    x, r, w = _inputs(rows, hidden, 13)
    ex, er = x.clone(), r.clone()
    for _ in range(2):
        torch.ops.inference_performance_lab.fused_add_rms_norm(ex, er, w, 1e-6)
    gx, gr = x.clone(), r.clone()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(2):
                torch.ops.inference_performance_lab.fused_add_rms_norm(gx, gr, w, 1e-6)
    gx.copy_(x)
    gr.copy_(r)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gx, ex) and torch.equal(gr, er)
    del graph


# Rows of 16384 < H <= 32768: eight chunks a thread (up to 512 threads); add+RMSNorm at 96
# registers ("capped", two CTAs an SM) up to H = 20480 for more than 256 rows, else at 128.
# 256 rows or fewer go to the cluster kernel.
LONG = [(1000, 16392, "capped"), (300, 18432, "capped"), (257, 20480, "capped"), (300, 24576, ""),
        (257, 32768, "")]


@pytest.mark.parametrize("w_off", [0, 1])
@pytest.mark.parametrize("rows, hidden, variant", LONG)
@torch.inference_mode()
def test_fused_long_rows(rows: int, hidden: int, variant: str, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, rows + hidden + w_off)
    gx, gr, gw = Guarded(x.shape, 0), Guarded(x.shape, 0), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    assert plan == ("rmsnorm_stash_kernel<8, capped>" if variant else "rmsnorm_stash_kernel<8>"), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden", [(1000, 18432), (300, 32768)])
@torch.inference_mode()
def test_plain_long_rows(rows: int, hidden: int) -> None:
    x, _, w = _inputs(rows, hidden, rows + 9 * hidden)
    gx, go = Guarded(x.shape, 0), Guarded(x.shape, 0)
    ax = gx.load(oracle.tensor_bits(x))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), w.data_ptr(), rows, hidden)
    assert plan == "rmsnorm_stash_kernel<8, plain>", plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, w, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}")
    gx.assert_guards_intact()
    go.assert_guards_intact()


# Rows off 16 bytes, x and residual alike, every phase (H % 8 == 0): the shifted kernel works on
# the H / 8 + 1 aligned chunks that cover each row, masks the elements of its neighbours and shifts
# gamma by the phase (two aligned loads, or element by element for a misaligned weight).
SHIFTED = [(300, 3584, off) for off in range(1, 8)] + [(2048, 3584, 1), (600, 1032, 5), (300, 1536, 2),
                                                         (500, 8192, 3), (400, 12288, 7), (257, 5120, 4)]


@pytest.mark.parametrize("w_off", [0, 3])
@pytest.mark.parametrize("rows, hidden, off", SHIFTED)
@torch.inference_mode()
def test_fused_shifted_rows(rows: int, hidden: int, off: int, w_off: int) -> None:
    x, r, w = _inputs(rows, hidden, 7 * rows + hidden + 11 * off + w_off)
    gx, gr, gw = Guarded(x.shape, off), Guarded(x.shape, off), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    plan = capi.fused_add_rms_norm_plan(ax.data_ptr(), ar.data_ptr(), aw.data_ptr(), rows, hidden)
    # With a 16-byte aligned weight, rows of 1536-4080 elements (H % 16 == 0) go to the 256-bit
    # variant (tests/test_shifted_v8_rows.py).
    v8 = w_off == 0 and hidden % 16 == 0 and 1536 <= hidden <= 4080 and rows <= 4096
    assert plan == (f"rmsnorm_shifted_v8_kernel<{off}>" if v8 else f"rmsnorm_shifted_kernel<{off}>"), plan
    torch.ops.inference_performance_lab.fused_add_rms_norm(ax, ar, aw, 1e-6)
    out, res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-6)
    assert_bits_equal(ar, res, f"{rows}x{hidden}+{off} residual")
    assert_close_to_oracle(ax, out, f"{rows}x{hidden}+{off} output")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


@pytest.mark.parametrize("rows, hidden, off", [(300, 3584, 1), (700, 4096, 6), (400, 2048, 3), (2000, 1536, 2)])
@torch.inference_mode()
def test_plain_shifted_rows(rows: int, hidden: int, off: int) -> None:
    x, _, w = _inputs(rows, hidden, 3 * rows + hidden + off)
    gx, go = Guarded(x.shape, off), Guarded(x.shape, off)
    ax = gx.load(oracle.tensor_bits(x))
    plan = capi.rms_norm_plan(go.tensor.data_ptr(), ax.data_ptr(), w.data_ptr(), rows, hidden)
    assert plan == f"rmsnorm_shifted_kernel<{off}, plain>", plan
    torch.ops.inference_performance_lab.rms_norm(go.tensor, ax, w, 1e-6)
    assert_close_to_oracle(go.tensor, oracle.c_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(w), 1e-6),
                           f"{rows}x{hidden}+{off}")
    torch.ops.inference_performance_lab.rms_norm(ax, ax, w, 1e-6)  # in place
    assert torch.equal(ax, go.tensor)
    gx.assert_guards_intact()
    go.assert_guards_intact()


@torch.inference_mode()
def test_shifted_graph_replay_matches_eager() -> None:
    rows, hidden, off = 2100, 3584, 3
    x, r, w = _inputs(rows, hidden, 17)
    gx, gr = Guarded(x.shape, off), Guarded(x.shape, off)
    ex, er = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r))
    assert capi.fused_add_rms_norm_plan(ex.data_ptr(), er.data_ptr(), w.data_ptr(), rows, hidden) == (
        "rmsnorm_shifted_v8_kernel<3>"
    )
    for _ in range(2):
        torch.ops.inference_performance_lab.fused_add_rms_norm(ex, er, w, 1e-6)
    hx, hr = Guarded(x.shape, off), Guarded(x.shape, off)
    gxt, grt = hx.load(oracle.tensor_bits(x)), hr.load(oracle.tensor_bits(r))
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(2):
                torch.ops.inference_performance_lab.fused_add_rms_norm(gxt, grt, w, 1e-6)
    gxt.copy_(x)
    grt.copy_(r)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gxt, ex) and torch.equal(grt, er)
    for g in (gx, gr, hx, hr):
        g.assert_guards_intact()
    del graph
