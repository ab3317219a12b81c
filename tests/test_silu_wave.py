"""GPU parity of the one-wave SiLU kernel (one 16-byte pack a thread, 1024-thread CTAs, two an SM;
planned when the launch's 16-byte packs number more than the SMs x 1024 and at most the SMs x 2048)
against the oracle: aligned and 16-byte-offset tensors with canary guards, widths whose rows end
inside a warp, a last CTA only partly filled, a single long row, edge values, both op names, and
launches queued back to back and replayed from a CUDA graph."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from oracle import oracle
from parity import Guarded, assert_close_to_oracle, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()


def _sms() -> int:
    return torch.cuda.get_device_properties(0).multi_processor_count


def _wave_shape(rows: int, inter: int) -> bool:
    packs = rows * (inter // 8)
    return inter % 8 == 0 and _sms() * 1024 < packs <= _sms() * 2048


# rows, intermediate, output offset, input offset (elements); every shape one wave at 148 SMs.
CASES = [
    (128, 18944, 0, 0),      # the [128, 37888] workload: 303,104 packs, exactly one wave
    (128, 18944, 8, 8),      # 16-byte but not 32-byte aligned
    (128, 18944, 8, 0),
    (127, 18952, 0, 0),      # 2369 packs a row: rows end inside a warp (line prefetch there)
    (97, 18944, 0, 0),       # 229,696 packs: the last CTA partly filled
    (160, 14336, 0, 0),
    (300, 4096, 0, 0),       # 153,600 packs: just above half a wave
    (76, 16000, 0, 0),
    (151, 16000, 0, 0),
    (1, 2400000, 0, 0),      # one row of 300,000 packs
]


@pytest.mark.parametrize("rows, inter, out_off, in_off", CASES)
@torch.inference_mode()
def test_wave_kernel_against_oracle(rows: int, inter: int, out_off: int, in_off: int) -> None:
    assert _wave_shape(rows, inter), (rows, inter, _sms())
    generator = torch.Generator(device="cuda").manual_seed(rows * 13 + inter + out_off)
    x = (torch.randn(rows, 2 * inter, device="cuda", generator=generator) * 2).to(torch.bfloat16)
    gi, go = Guarded(x.shape, in_off), Guarded((rows, inter), out_off)
    xin = gi.load(oracle.tensor_bits(x))
    assert capi.silu_and_mul_plan(go.tensor.data_ptr(), xin.data_ptr(), rows, inter) == "silu_wave_kernel"
    torch.ops.inference_performance_lab.silu_and_mul(go.tensor, xin)
    want = oracle.c_silu_and_mul(oracle.tensor_bits(x))
    assert_close_to_oracle(go.tensor, want, f"rows={rows} I={inter} offsets={out_off},{in_off}")
    assert torch.equal(xin, x), "input must not be modified"
    gi.assert_guards_intact()
    go.assert_guards_intact()
    # The packed op name runs the same kernel on the same (16-byte aligned) tensors.
    out2 = torch.empty(rows, inter, device="cuda", dtype=torch.bfloat16)
    torch.ops.inference_performance_lab.silu_and_mul_packed(out2, x)
    assert torch.equal(out2, go.tensor)


@torch.inference_mode()
def test_wave_kernel_edge_values() -> None:
    """Infinities, NaN, gates far below -87 (silu underflows to 0) and large magnitudes scattered
    over a one-wave launch, including the first and last pack of rows and of the launch."""
    rows, inter = 128, 18944
    generator = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(rows, 2 * inter, device="cuda", generator=generator) * 2).to(torch.bfloat16)
    specials = torch.tensor([float("inf"), float("-inf"), float("nan"), -100.0, -88.0, 88.0, 3e38, -3e38, 0.0,
                             -0.0, 1e-30, -1e-30], dtype=torch.bfloat16, device="cuda")
    for row in (0, 63, 127):
        for col in (0, 7, 8, inter - 8, inter - 1):
            for half in (0, inter):
                x[row, half + col] = specials[(row + col + half) % specials.numel()]
    out = torch.empty(rows, inter, device="cuda", dtype=torch.bfloat16)
    assert capi.silu_and_mul_plan(out.data_ptr(), x.data_ptr(), rows, inter) == "silu_wave_kernel"
    torch.ops.inference_performance_lab.silu_and_mul(out, x)
    want = oracle.c_silu_and_mul(oracle.tensor_bits(x))
    # NaN exactly where the oracle has NaN (NaN inputs, gate = -inf, inf x 0), the rest within
    # tolerance.
    want_nan = np.isnan(oracle.bf16_bits_to_f32(want))
    assert want_nan.any()
    assert np.array_equal(np.isnan(oracle.bf16_bits_to_f32(oracle.tensor_bits(out))), want_nan)
    mask = torch.from_numpy(want_nan).to(out.device)
    want = want.copy()
    want[want_nan] = 0
    assert_close_to_oracle(out.masked_fill(mask, 0.0), want, "edge values")


@torch.inference_mode()
def test_wave_kernel_queued_and_in_a_graph() -> None:
    """Four launches over four input/output pairs: one at a time with a synchronize between them,
    queued back to back (each launch's CTAs prefetch while the previous drains) and replayed from
    a CUDA graph, all the same bits; the first pair also matches the oracle."""
    rows, inter = 128, 18944
    generator = torch.Generator(device="cuda").manual_seed(5)
    xs = [(torch.randn(rows, 2 * inter, device="cuda", generator=generator) * 2).to(torch.bfloat16)
          for _ in range(4)]
    solo = []
    for x in xs:
        out = torch.empty(rows, inter, device="cuda", dtype=torch.bfloat16)
        torch.ops.inference_performance_lab.silu_and_mul(out, x)
        torch.cuda.synchronize()
        solo.append(out)
    assert_close_to_oracle(solo[0], oracle.c_silu_and_mul(oracle.tensor_bits(xs[0])), "first launch")
    queued = [torch.full((rows, inter), 7.0, device="cuda", dtype=torch.bfloat16) for _ in xs]
    for x, out in zip(xs, queued):
        torch.ops.inference_performance_lab.silu_and_mul(out, x)
    torch.cuda.synchronize()
    for a, b in zip(solo, queued):
        assert torch.equal(a, b)
    outs = [torch.empty(rows, inter, device="cuda", dtype=torch.bfloat16) for _ in xs]
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for x, out in zip(xs, outs):
                torch.ops.inference_performance_lab.silu_and_mul(out, x)
    for out in outs:
        out.fill_(7.0)
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(solo, outs):
        assert torch.equal(a, b)
    del graph


@pytest.mark.parametrize("rows, inter, kernel", [(64, 18944, "silu_vector_kernel<32>"),
                                                 (129, 18944, "silu_vector_kernel<32>"),
                                                 (300, 1000, "silu_vector_kernel<16>")])
@torch.inference_mode()
def test_shapes_beside_the_wave_keep_their_kernels(rows: int, inter: int, kernel: str) -> None:
    """Half a wave or less, and more than one wave, stay on the unrolled vector kernel."""
    x = torch.randn(rows, 2 * inter, device="cuda").to(torch.bfloat16)
    out = torch.empty(rows, inter, device="cuda", dtype=torch.bfloat16)
    assert capi.silu_and_mul_plan(out.data_ptr(), x.data_ptr(), rows, inter) == kernel
    torch.ops.inference_performance_lab.silu_and_mul(out, x)
    assert_close_to_oracle(out, oracle.c_silu_and_mul(oracle.tensor_bits(x)), f"{rows}x{inter}")
