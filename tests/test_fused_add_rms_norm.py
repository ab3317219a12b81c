"""GPU parity of fused add+RMSNorm against the oracle and the reference's golden vectors.

Mirrors the reference's tests/test_fused_add_rms_norm.py (seed 0, H = 3584, T in {1, 8, 128, 2048},
residual bit-exact, output within rtol = atol = 1e-2; x, residual or weight misaligned in turn) and
extends them: golden vectors of reference.py, a sweep of widths and alignments with canary
guards around every tensor, the misaligned 2048 x 3584 workload, the full [262144, 8192] row-sharded
workload checked through size-independent properties, the C-ABI entry point, CUDA-graph
capture, and the device fault word.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from inference_performance_lab.kernels.extension import fused_add_rms_norm as custom_fused_add_rms_norm
from oracle import oracle
from parity import Guarded, assert_bits_equal, assert_close_to_oracle, require_cuda

HIDDEN_SIZE = 3584
EPSILON = 1e-6
TOKEN_COUNTS = [1, 8, 128, 2048]

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN = np.load(GOLDEN_DIR / "golden.npz")
CASES = json.loads((GOLDEN_DIR / "golden.json").read_text())["cases"]
RMS_CASES = sorted(name for name, meta in CASES.items() if meta["op"] == "fused_add_rms_norm")

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


def oracle_bits(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    return oracle.c_fused_add_rms_norm(
        oracle.tensor_bits(x), oracle.tensor_bits(residual), oracle.tensor_bits(weight), eps
    )


def check(x_in, r_in, w, eps, x_out, r_out, what: str) -> None:
    expected_out, expected_res = oracle_bits(x_in, r_in, w, eps)
    assert_bits_equal(r_out, expected_res, f"{what} residual")
    assert_close_to_oracle(x_out, expected_out, f"{what} output")


# ---- the reference's own cases ---------------------------------------------------------------


@pytest.mark.parametrize("num_tokens", TOKEN_COUNTS)
@torch.inference_mode()
def test_custom_matches_reference(num_tokens: int) -> None:
    torch.manual_seed(0)
    x = torch.randn(num_tokens, HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16)
    residual = torch.randn_like(x)
    weight = torch.randn(HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16) * 0.1 + 1.0

    expected_output, expected_residual = oracle.torch_fused_add_rms_norm(
        x.cpu(), residual.cpu(), weight.cpu(), EPSILON
    )
    actual_output = x.clone()
    actual_residual = residual.clone()
    custom_fused_add_rms_norm(actual_output, actual_residual, weight, EPSILON)

    torch.testing.assert_close(actual_residual.cpu(), expected_residual, rtol=0, atol=0)
    torch.testing.assert_close(actual_output.cpu(), expected_output, rtol=1e-2, atol=1e-2)
    check(x, residual, weight, EPSILON, actual_output, actual_residual, f"T={num_tokens}")


@pytest.mark.parametrize("num_tokens", TOKEN_COUNTS)
@torch.inference_mode()
def test_vllm_matches_reference(num_tokens: int) -> None:
    """The comparison arm of the head-to-head benchmarks (vLLM's kernel) meets the same oracle, as
    the reference's own test of it does (tests/test_fused_add_rms_norm.py:46-51 of the reference);
    aligned tensors only."""
    vllm_ops = pytest.importorskip("vllm._custom_ops")
    torch.manual_seed(0)
    x = torch.randn(num_tokens, HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16)
    residual = torch.randn_like(x)
    weight = torch.randn(HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16) * 0.1 + 1.0
    expected_output, expected_residual = oracle.torch_fused_add_rms_norm(x.cpu(), residual.cpu(), weight.cpu(), EPSILON)
    actual_output, actual_residual = x.clone(), residual.clone()
    vllm_ops.fused_add_rms_norm(actual_output, actual_residual, weight, EPSILON)
    torch.testing.assert_close(actual_residual.cpu(), expected_residual, rtol=0, atol=0)
    torch.testing.assert_close(actual_output.cpu(), expected_output, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("misaligned_argument", ["x", "residual", "weight"])
@torch.inference_mode()
def test_custom_handles_misaligned_contiguous_tensors(misaligned_argument: str) -> None:
    torch.manual_seed(0)
    x = torch.randn(8, HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16)
    residual = torch.randn_like(x)
    weight = torch.randn(HIDDEN_SIZE, device="cuda", dtype=torch.bfloat16) * 0.1 + 1.0

    gx = Guarded(x.shape, 1 if misaligned_argument == "x" else 0)
    gr = Guarded(x.shape, 1 if misaligned_argument == "residual" else 0)
    gw = Guarded(weight.shape, 1 if misaligned_argument == "weight" else 0)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(residual)), gw.load(
        oracle.tensor_bits(weight)
    )
    custom_fused_add_rms_norm(ax, ar, aw, EPSILON)
    check(x, residual, weight, EPSILON, ax, ar, f"misaligned {misaligned_argument}")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


# ---- golden vectors of reference.py ---------------------------------------------------------


@pytest.mark.parametrize("name", RMS_CASES)
@torch.inference_mode()
def test_golden_vectors(name: str) -> None:
    meta = CASES[name]
    gx = Guarded((meta["rows"], meta["hidden"]), 0)
    gr = Guarded((meta["rows"], meta["hidden"]), 0)
    w = oracle.bits_tensor(GOLDEN[f"{name}.weight"], "cuda")
    x, r = gx.load(GOLDEN[f"{name}.x"]), gr.load(GOLDEN[f"{name}.residual"])
    custom_fused_add_rms_norm(x, r, w, meta["epsilon"])
    assert_bits_equal(r, GOLDEN[f"{name}.residual_out"], f"{name} residual")
    assert_close_to_oracle(x, GOLDEN[f"{name}.out"], f"{name} output")
    gx.assert_guards_intact()
    gr.assert_guards_intact()


# ---- widths x alignments x row counts, every kernel of the dispatch --------------------------

SWEEP = [
    # rows, hidden, x offset, residual offset, weight offset (elements)
    *[(rows, hidden, 0, 0, 0) for rows in (1, 3, 150) for hidden in
      (1, 2, 7, 8, 9, 15, 16, 17, 64, 127, 1000, 1001, 1024, 3584, 4096, 4097, 5120, 8192, 12288, 16384)],
    *[(37, 3584, off, off, woff) for off in range(8) for woff in (0, 3)],
    *[(37, 1001, off, off, 0) for off in range(8)],
    *[(9, 3584, xo, ro, 0) for xo, ro in ((0, 1), (1, 0), (3, 5), (7, 2))],
    (300, 3584, 0, 0, 0),
    (600, 3584, 0, 0, 0),
    (1200, 3584, 0, 0, 0),
    (400, 16384, 0, 0, 0),
    (300, 16392, 0, 0, 0),
    (5, 27000, 0, 0, 0),
    (5, 40000, 0, 0, 0),
    (5, 40000, 1, 0, 0),
    (3, 100003, 0, 0, 0),
]


@pytest.mark.parametrize("rows, hidden, x_off, r_off, w_off", SWEEP)
@torch.inference_mode()
def test_sweep_against_oracle(rows: int, hidden: int, x_off: int, r_off: int, w_off: int) -> None:
    generator = torch.Generator(device="cuda").manual_seed(rows * 131 + hidden)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    gx, gr, gw = Guarded(x.shape, x_off), Guarded(x.shape, r_off), Guarded(w.shape, w_off)
    ax, ar, aw = gx.load(oracle.tensor_bits(x)), gr.load(oracle.tensor_bits(r)), gw.load(oracle.tensor_bits(w))
    custom_fused_add_rms_norm(ax, ar, aw, EPSILON)
    check(x, r, w, EPSILON, ax, ar, f"rows={rows} H={hidden} offsets={x_off},{r_off},{w_off}")
    for g in (gx, gr, gw):
        g.assert_guards_intact()


# ---- the benchmark workloads ------------------------------------------------------------------


@torch.inference_mode()
def test_misaligned_2048x3584_workload() -> None:
    """x and residual as views one element (2 bytes) into [2048*3584 + 8] buffers."""
    rows, hidden = 2048, 3584
    torch.manual_seed(0)
    x_buf = torch.randn(rows * hidden + 8, device="cuda", dtype=torch.bfloat16)
    r_buf = torch.randn(rows * hidden + 8, device="cuda", dtype=torch.bfloat16)
    weight = torch.randn(hidden, device="cuda", dtype=torch.bfloat16) * 0.1 + 1.0
    x = x_buf[1: 1 + rows * hidden].view(rows, hidden)
    r = r_buf[1: 1 + rows * hidden].view(rows, hidden)
    assert x.data_ptr() % 16 == 2 and r.data_ptr() % 16 == 2
    x_in, r_in = x.clone(), r.clone()
    before_x, before_r = x_buf.clone(), r_buf.clone()
    custom_fused_add_rms_norm(x, r, weight, EPSILON)
    check(x_in, r_in, weight, EPSILON, x, r, "2048x3584 misaligned")
    # Elements outside the views are untouched.
    for buf, before in ((x_buf, before_x), (r_buf, before_r)):
        assert torch.equal(buf[:1], before[:1]) and torch.equal(buf[1 + rows * hidden:], before[1 + rows * hidden:])


@torch.inference_mode()
def test_row_sharded_262144x8192_workload_properties() -> None:
    """The full row-sharded workload on one GPU: every residual element bit-exact against the
    elementwise fp32 reference, every output element within tolerance of a chunked fp32
    reference, and sampled rows (CTA block boundaries included) checked against the oracle."""
    rows, hidden, eps = 262144, 8192, 1e-5
    generator = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(rows, hidden, device="cuda", dtype=torch.bfloat16, generator=generator)
    r = torch.randn(rows, hidden, device="cuda", dtype=torch.bfloat16, generator=generator)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    x_ref, r_ref = x.clone(), r.clone()
    custom_fused_add_rms_norm(x, r, w, eps)
    chunk = 16384
    for s in range(0, rows, chunk):
        v = x_ref[s: s + chunk].float() + r_ref[s: s + chunk].float()
        assert torch.equal(r[s: s + chunk], v.to(torch.bfloat16)), f"residual rows {s}+"
        ref = (v * torch.rsqrt(v.square().mean(-1, keepdim=True) + eps) * w.float()).to(torch.bfloat16)
        torch.testing.assert_close(x[s: s + chunk], ref, rtol=1e-2, atol=1e-2)
    boundaries = [rows * k // 148 for k in range(149)]
    picks = sorted({min(max(b + d, 0), rows - 1) for b in boundaries[::16] for d in (-1, 0)})
    picks += torch.randint(0, rows, (32,), device="cuda", generator=generator).tolist()
    sample = torch.tensor(sorted(set(picks)), device="cuda")
    expected_out, expected_r = oracle_bits(x_ref[sample], r_ref[sample], w, eps)
    assert_bits_equal(r[sample], expected_r, "sampled residual")
    assert_close_to_oracle(x[sample], expected_out, "sampled output")


# ---- boundary: C ABI, streams, graphs, empty input, errors ------------------------------------


@torch.inference_mode()
def test_c_abi_entry_point_matches_torch_op() -> None:
    torch.manual_seed(3)
    x = torch.randn(300, 3584, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(3584, device="cuda", dtype=torch.bfloat16) * 0.1 + 1
    x1, r1, x2, r2 = x.clone(), r.clone(), x.clone(), r.clone()
    custom_fused_add_rms_norm(x1, r1, w, EPSILON)
    capi.fused_add_rms_norm_tensors(x2, r2, w, EPSILON)
    torch.cuda.synchronize()
    assert torch.equal(x1, x2) and torch.equal(r1, r2)
    check(x, r, w, EPSILON, x2, r2, "C ABI")


@torch.inference_mode()
def test_runs_on_the_current_stream_and_captures_in_a_graph() -> None:
    torch.manual_seed(4)
    x = torch.randn(2048, 3584, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(3584, device="cuda", dtype=torch.bfloat16) * 0.1 + 1
    x_in, r_in = x.clone(), r.clone()
    stream = torch.cuda.Stream()
    xs, rs = x.clone(), r.clone()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        custom_fused_add_rms_norm(xs, rs, w, EPSILON)
    torch.cuda.current_stream().wait_stream(stream)
    check(x_in, r_in, w, EPSILON, xs, rs, "side stream")

    xg, rg = x.clone(), r.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        custom_fused_add_rms_norm(xg, rg, w, EPSILON)
    xg.copy_(x_in)
    rg.copy_(r_in)
    graph.replay()
    torch.cuda.synchronize()
    check(x_in, r_in, w, EPSILON, xg, rg, "graph replay")
    del graph


@torch.inference_mode()
def test_back_to_back_calls_chain_correctly() -> None:
    """Consecutive dependent calls (each launched with programmatic stream serialisation) see
    the previous call's results: ten layers of a residual stream launched without host syncs
    end in the same state as ten layers each checked against the oracle."""
    torch.manual_seed(5)
    x = torch.randn(512, 4096, device="cuda", dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.randn(4096, device="cuda", dtype=torch.bfloat16) * 0.1 + 1
    xg, rg = x.clone(), r.clone()
    for _ in range(10):
        custom_fused_add_rms_norm(xg, rg, w, EPSILON)
    xk, rk = x.clone(), r.clone()
    for layer in range(10):
        x_prev, r_prev = xk.clone(), rk.clone()
        custom_fused_add_rms_norm(xk, rk, w, EPSILON)
        check(x_prev, r_prev, w, EPSILON, xk, rk, f"layer {layer}")
    assert torch.equal(xk, xg) and torch.equal(rk, rg)


@pytest.mark.parametrize("rows, hidden", [(32768, 8192), (2048, 3584), (4096, 1024)])
@torch.inference_mode()
def test_chained_launches_after_copies_and_in_graphs(rows: int, hidden: int) -> None:
    """Launch patterns of real callers: after host-to-device copies into the same buffers, and
    as a chain of in-place calls replayed from a CUDA graph. Every call must complete (the
    device fault word stays 0) and the chain must equal the same calls made one at a time."""
    capi.clear_device_fault_flags(torch.cuda.current_device())
    torch.manual_seed(6)
    x_h = torch.randn(rows, hidden, dtype=torch.bfloat16).pin_memory()
    r_h = torch.randn(rows, hidden, dtype=torch.bfloat16).pin_memory()
    w = (torch.randn(hidden, device="cuda") * 0.1 + 1).to(torch.bfloat16)
    x = torch.empty(rows, hidden, device="cuda", dtype=torch.bfloat16)
    r = torch.empty_like(x)
    for _ in range(3):
        x.copy_(x_h, non_blocking=True)
        r.copy_(r_h, non_blocking=True)
        custom_fused_add_rms_norm(x, r, w, EPSILON)
    torch.cuda.synchronize()
    if rows * hidden <= 8 * 2**20:
        check(x_h, r_h, w, EPSILON, x, r, "after copies")

    x_ref, r_ref = x.clone(), r.clone()
    for _ in range(8):
        custom_fused_add_rms_norm(x_ref, r_ref, w, EPSILON)
        torch.cuda.synchronize()
    xg, rg = x.clone(), r.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(8):
            custom_fused_add_rms_norm(xg, rg, w, EPSILON)
    xg.copy_(x)
    rg.copy_(r)
    graph.replay()
    torch.cuda.synchronize()
    del graph
    assert torch.equal(xg, x_ref) and torch.equal(rg, r_ref)
    assert capi.device_fault_flags(torch.cuda.current_device()) == 0


@torch.inference_mode()
def test_empty_and_error_cases() -> None:
    w = torch.ones(3584, device="cuda", dtype=torch.bfloat16)
    empty = torch.empty(0, 3584, device="cuda", dtype=torch.bfloat16)
    custom_fused_add_rms_norm(empty, empty.clone(), w, EPSILON)  # no-op, no launch error
    x = torch.randn(4, 3584, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must use bfloat16"):
        custom_fused_add_rms_norm(x.float(), x.clone(), w, EPSILON)
    with pytest.raises(RuntimeError, match="x must be contiguous"):
        custom_fused_add_rms_norm(x.t(), x.t().clone(), w, EPSILON)
    with pytest.raises(RuntimeError, match="identical shapes"):
        custom_fused_add_rms_norm(x, x[:2].clone(), w, EPSILON)
    with pytest.raises(RuntimeError, match="weight must match the final tensor dimension"):
        custom_fused_add_rms_norm(x, x.clone(), w[:100].contiguous(), EPSILON)
    with pytest.raises(RuntimeError, match="epsilon must be positive"):
        custom_fused_add_rms_norm(x, x.clone(), w, 0.0)
    with pytest.raises(RuntimeError, match="weight must be one-dimensional"):
        custom_fused_add_rms_norm(x, x.clone(), w.view(1, -1), EPSILON)


def test_no_kernel_gave_up_on_a_wait() -> None:
    torch.cuda.synchronize()
    assert capi.device_fault_flags(torch.cuda.current_device()) == 0
