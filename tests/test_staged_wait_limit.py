"""A bounded wait of the staged kernel that runs out: the kernel returns, records the fault, and
leaves the CUDA context usable.

Runs the test-only build of the library (``build.py --tests`` ->
``_native/test/libipl_b200_waittest.so``): the same sources with every wait limited to 1 ms and
with CTA 0 of the staged kernel never issuing the copy of its row 0 - a barrier phase that nothing
completes, so the consumers waiting for it give up. Nothing is left in flight for that stage, no
GPU fault is involved, and every other CTA runs normally. The shapes cover the staged kernel's
three schedules: one row per CTA with all 16 consumer warps on it (their group barrier), several
rows per CTA each in its own stage (the abort crossing groups), and a streaming ring of two stages
(the producer's own wait on a stage that is never released, then its drain).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from inference_performance_lab.kernels import capi
from inference_performance_lab.kernels.extension import NATIVE_DIR
from oracle import oracle

from parity import assert_bits_equal, assert_close_to_oracle, require_cuda

pytestmark = pytest.mark.gpu

WAIT_TEST_LIBRARY = NATIVE_DIR / "test" / "libipl_b200_waittest.so"
FAULT_FULL_BARRIER_TIMEOUT = 1 << 0   # a consumer gave up waiting for its row
FAULT_EMPTY_BARRIER_TIMEOUT = 1 << 1  # the producer gave up waiting for a stage to be released
FAULT_COPY_DRAIN_TIMEOUT = 1 << 2     # a copy the producer issued had not landed at its exit


def _library() -> ctypes.CDLL:
    if not WAIT_TEST_LIBRARY.exists():
        pytest.fail(f"{WAIT_TEST_LIBRARY} is missing: run inference-performance-lab_b200/build.py --tests")
    lib = ctypes.CDLL(str(WAIT_TEST_LIBRARY))
    for name, (restype, argtypes) in capi.SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def _flags(lib: ctypes.CDLL) -> int:
    flags = ctypes.c_uint32(0)
    assert lib.ipl_device_fault_flags(0, ctypes.byref(flags)) == 0, lib.ipl_last_error()
    return flags.value


def _inputs(rows: int, hidden: int, seed: int):
    generator = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, device="cuda", generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, device="cuda", generator=generator) * 0.1 + 1).to(torch.bfloat16)
    return x, r, w


@pytest.mark.parametrize(
    ("rows", "hidden", "expected_bits"),
    [
        # Every row has a stage of its own: only consumers wait, so a consumer gives up first.
        (64, 1001, FAULT_FULL_BARRIER_TIMEOUT),
        (1000, 1001, FAULT_FULL_BARRIER_TIMEOUT),
        # Two stages: the producer, waiting for the never-filled stage to be released, and the
        # consumers of that row, waiting for it to fill, start their waits microseconds apart;
        # whichever gives up first records its bit and the others leave on the abort flag.
        (600, 16001, FAULT_FULL_BARRIER_TIMEOUT | FAULT_EMPTY_BARRIER_TIMEOUT),
    ],
    ids=["row-per-cta", "rows-in-own-stages", "streaming-ring"],
)
def test_staged_wait_runs_out_and_the_kernel_returns(rows: int, hidden: int, expected_bits: int) -> None:
    require_cuda()
    torch.cuda.set_device(0)
    lib = _library()
    x, r, w = _inputs(rows, hidden, seed=rows + hidden)
    plan = lib.ipl_fused_add_rms_norm_plan(x.data_ptr(), r.data_ptr(), w.data_ptr(), rows, hidden).decode()
    assert plan.startswith("rmsnorm_staged_kernel<"), plan
    x_in, r_in, w_bits = oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w)
    want_out, want_res = oracle.c_fused_add_rms_norm(x_in, r_in, w_bits, 1e-6)

    assert lib.ipl_clear_device_fault_flags(0) == 0
    status = lib.ipl_fused_add_rms_norm_bf16(x.data_ptr(), r.data_ptr(), w.data_ptr(), rows, hidden, 1e-6,
                                            torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.ipl_last_error()
    torch.cuda.synchronize()  # the kernel returned and the context is intact

    flags = _flags(lib)
    assert flags & expected_bits, f"fault word {flags:#x}"
    assert not flags & ~expected_bits, f"fault word {flags:#x}"  # in particular no copy was left in flight
    # CTA b owns rows [rows * b // grid, rows * (b + 1) // grid), so CTA 0 rows [0, rows // grid);
    # its row 0 was never copied, so nothing wrote it.
    grid = min(rows, torch.cuda.get_device_properties(0).multi_processor_count)
    first_other = rows // grid
    assert_bits_equal(x[0], x_in[0], "x row 0 (never staged)")
    assert_bits_equal(r[0], r_in[0], "residual row 0 (never staged)")
    # Every other CTA's rows are complete and exact.
    assert_bits_equal(r[first_other:], want_res[first_other:], "residual of the other CTAs' rows")
    assert_close_to_oracle(x[first_other:], want_out[first_other:], "output of the other CTAs' rows")

    assert lib.ipl_clear_device_fault_flags(0) == 0
    assert _flags(lib) == 0


def test_context_stays_usable_after_a_wait_ran_out() -> None:
    """After a staged launch gave up on a wait, a launch of another kernel from the same library
    on the same stream runs to completion, exact, with the fault word left at zero."""
    require_cuda()
    torch.cuda.set_device(0)
    lib = _library()
    x, r, w = _inputs(64, 1001, seed=1)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.ipl_fused_add_rms_norm_plan(x.data_ptr(), r.data_ptr(), w.data_ptr(), 64, 1001).decode() \
        .startswith("rmsnorm_staged_kernel<")
    assert lib.ipl_fused_add_rms_norm_bf16(x.data_ptr(), r.data_ptr(), w.data_ptr(), 64, 1001, 1e-6, stream) == 0
    torch.cuda.synchronize()
    assert _flags(lib) & FAULT_FULL_BARRIER_TIMEOUT
    assert lib.ipl_clear_device_fault_flags(0) == 0

    x, r, w = _inputs(2048, 3584, seed=2)
    assert lib.ipl_fused_add_rms_norm_plan(x.data_ptr(), r.data_ptr(), w.data_ptr(), 2048, 3584).decode() \
        == "rmsnorm_stash_v8_kernel"
    want_out, want_res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r),
                                                     oracle.tensor_bits(w), 1e-6)
    assert lib.ipl_fused_add_rms_norm_bf16(x.data_ptr(), r.data_ptr(), w.data_ptr(), 2048, 3584, 1e-6, stream) == 0
    torch.cuda.synchronize()
    assert _flags(lib) == 0
    assert_bits_equal(r, want_res, "residual")
    assert_close_to_oracle(x, want_out, "output")
    # The product library's own fault word was never touched by any of this.
    assert capi.device_fault_flags(0) == 0
    assert np.array_equal(oracle.tensor_bits(r), want_res)
