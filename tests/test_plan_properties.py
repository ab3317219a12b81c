"""Kernel selection over random shapes and pointer offsets (CPU, no device): whatever the planner
picks, the named kernel's preconditions hold - the vector kernels (the cluster kernel included)
only see 16-byte aligned rows within their width limits, the shifted kernel only the phase it is
instantiated for, the staged kernel x and residual (or out) at the same offset and no fp8 output,
and "none" means no rows."""

from __future__ import annotations

import re

from hypothesis import given, settings
from hypothesis import strategies as st

from inference_performance_lab.kernels import capi

BASE = 0x7F0000000000  # never dereferenced; 256-byte aligned

offsets = st.integers(min_value=0, max_value=7)  # bf16 elements off a 16-byte boundary
widths = st.one_of(st.integers(min_value=1, max_value=40000),
                   st.sampled_from([256, 1024, 1032, 2048, 3584, 4096, 6144, 8192, 12288, 16384, 16392, 20480,
                                    32768, 32776, 65536, 131072, 131080]))
rows_st = st.one_of(st.integers(min_value=0, max_value=300000), st.sampled_from([1, 256, 257, 444, 445, 1184, 4096]))


def check(name: str, rows: int, hidden: int, x_off: int, o_off: int, w_off: int, mode: str, out8_off: int = 0) -> None:
    assert name not in ("invalid", ""), name
    if rows == 0:
        assert name == "none"
        return
    assert name != "none"
    aligned = x_off == 0 and o_off == 0 and hidden % 8 == 0 and (mode != "fp8" or out8_off % 8 == 0)
    kernel = name.split("<")[0]
    if kernel in ("rmsnorm_warp_kernel", "rmsnorm_cta_kernel", "rmsnorm_stash_kernel"):
        assert aligned, name
        limit = {"rmsnorm_warp_kernel": 1024, "rmsnorm_cta_kernel": 16384, "rmsnorm_stash_kernel": 32768}[kernel]
        assert hidden <= limit, name
        if kernel == "rmsnorm_cta_kernel" and rows > 256:
            assert hidden <= 4096, name  # above 256 rows only one chunk a thread, one wave
    elif kernel == "rmsnorm_shifted_v8_kernel":
        phase = int(re.match(r"rmsnorm_shifted_v8_kernel<(\d)", name).group(1))
        assert mode == "fused" and x_off == o_off == phase and w_off == 0 and hidden % 16 == 0, name
        assert 1536 <= hidden <= 4080 and 256 < rows <= 4096, name
    elif kernel == "rmsnorm_shifted_kernel":
        phase = int(re.match(r"rmsnorm_shifted_kernel<(\d)", name).group(1))
        assert mode != "fp8" and x_off == o_off == phase and hidden % 8 == 0 and rows > 256, name
        assert hidden <= (12288 if mode == "fused" else 4096), name
    elif kernel == "rmsnorm_stash_v8_kernel":
        # 256-bit accesses: rows 32 bytes aligned, H % 16 == 0, a 16-byte aligned weight and fp8 output.
        assert mode != "plain" and x_off == 0 and o_off == 0 and w_off == 0 and hidden % 16 == 0, name
        assert 1536 <= hidden <= 5120 and 256 < rows <= 4096 and (mode != "fp8" or out8_off == 0), name
    elif kernel == "rmsnorm_cluster_kernel":
        assert aligned and 6144 <= hidden <= 131072, name
        if hidden <= 32768:
            assert rows <= 256, name  # few long rows only
    elif kernel == "rmsnorm_staged_kernel":
        assert mode != "fp8" and x_off == o_off, name
    else:
        assert kernel == "rmsnorm_rowwise_kernel", name


@settings(max_examples=400, deadline=None)
@given(rows=rows_st, hidden=widths, x_off=offsets, r_off=offsets, w_off=offsets)
def test_fused_plans_respect_kernel_preconditions(rows, hidden, x_off, r_off, w_off) -> None:
    name = capi.fused_add_rms_norm_plan(BASE + 2 * x_off, BASE + (1 << 34) + 2 * r_off,
                                        BASE + (1 << 35) + 2 * w_off, rows, hidden)
    check(name, rows, hidden, x_off, r_off, w_off, "fused")


@settings(max_examples=400, deadline=None)
@given(rows=rows_st, hidden=widths, x_off=offsets, o_off=offsets, w_off=offsets)
def test_plain_plans_respect_kernel_preconditions(rows, hidden, x_off, o_off, w_off) -> None:
    name = capi.rms_norm_plan(BASE + (1 << 34) + 2 * o_off, BASE + 2 * x_off, BASE + (1 << 35) + 2 * w_off,
                              rows, hidden)
    check(name, rows, hidden, x_off, o_off, w_off, "plain")


@settings(max_examples=400, deadline=None)
@given(rows=rows_st, hidden=widths, x_off=offsets, r_off=offsets, out8_off=st.integers(min_value=0, max_value=15))
def test_fp8_plans_respect_kernel_preconditions(rows, hidden, x_off, r_off, out8_off) -> None:
    name = capi.fused_add_rms_norm_static_fp8_quant_plan(BASE + (1 << 36) + out8_off, BASE + 2 * x_off,
                                                         BASE + (1 << 34) + 2 * r_off, BASE + (1 << 35), rows, hidden)
    # The fp8 op's vector kernels need x and residual 16-byte aligned and an 8-byte aligned output.
    check(name, rows, hidden, x_off, r_off, 0, "fp8", out8_off)


@settings(max_examples=400, deadline=None)
@given(rows=st.integers(min_value=0, max_value=20000), inter=st.integers(min_value=0, max_value=60000),
       out_off=st.integers(min_value=0, max_value=31), in_off=st.integers(min_value=0, max_value=31))
def test_silu_plans_take_the_widest_vector_their_alignment_allows(rows, inter, out_off, in_off) -> None:
    name = capi.silu_and_mul_plan(BASE + 2 * out_off, BASE + (1 << 34) + 2 * in_off, rows, inter)
    if rows * inter == 0:
        assert name == "none"
        return
    offset_bytes = (2 * out_off) | (2 * in_off)
    packs16 = rows * (inter // 8)
    if inter % 8 == 0 and offset_bytes % 16 == 0 and 148 * 1024 < packs16 <= 148 * 2048:
        assert name == "silu_wave_kernel", name  # one 16-byte pack a thread, one wave of 148 x 2048 threads
    elif inter % 16 == 0 and offset_bytes % 32 == 0:
        assert name == "silu_vector_kernel<32>", name  # 32-byte packs: gate, up and out rows all aligned
    elif inter % 8 == 0 and offset_bytes % 16 == 0:
        assert name == "silu_vector_kernel<16>", name
    else:
        assert name == "silu_scalar_kernel", name
