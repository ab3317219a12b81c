"""The C-ABI library without a GPU: it loads, exports every declared symbol, validates arguments
before touching the device, and its kernel selection (a pure function of pointers and sizes)
picks the intended path for each shape and alignment of the parity and bench cases."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from inference_performance_lab.kernels import capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "ipl_b200.h"

# Fake, never-dereferenced device addresses: 256-byte aligned base plus an element offset.
BASE = 0x7F0000000000


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*IPL_API\s+[\w\s*]*?\b(ipl_\w+)\s*\(", text, re.M)))


def test_header_declares_the_path_entry_points() -> None:
    names = declared_functions()
    for required in (
        "ipl_fused_add_rms_norm_bf16",
        "ipl_silu_and_mul_bf16",
        "ipl_silu_and_mul_packed_bf16",
        "ipl_last_error",
    ):
        assert required in names


def test_library_exports_every_declared_symbol() -> None:
    lib = capi.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(capi.SIGNATURES)


C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "ipl_b200.h"

int main(void) {
    const uintptr_t base = (uintptr_t)0x7F0000000000ull; /* never dereferenced */
    void* x = (void*)base;
    void* r = (void*)(base + ((uintptr_t)1 << 34));
    const void* w = (const void*)(base + ((uintptr_t)1 << 35));
    if (ipl_abi_version() != 1) return 1;
    /* Plans are pure functions of pointers and sizes: no device needed. */
    printf("%s\n", ipl_fused_add_rms_norm_plan(x, r, w, 2048, 3584));
    printf("%s\n", ipl_silu_and_mul_plan(x, r, 128, 18944));
    /* Argument errors return before any device access. */
    ipl_status s = ipl_fused_add_rms_norm_bf16(x, r, w, 4, 3584, 0.0, NULL);
    printf("%s: %s\n", ipl_status_string(s), ipl_last_error());
    s = ipl_silu_and_mul_packed_bf16(x, r, 4, 18, NULL);
    printf("%s: %s\n", ipl_status_string(s), ipl_last_error());
    return 0;
}
"""


def test_c_caller_builds_links_and_runs(tmp_path: Path) -> None:
    """A plain C99 program includes the header and links the library, as a non-torch caller."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = Path(capi.library()._name)
    source = tmp_path / "caller.c"
    source.write_text(C_CALLER)
    exe = tmp_path / "caller"
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(HEADER.parent), str(source),
                    "-L", str(lib.parent), "-l:" + lib.name, "-Wl,-rpath," + str(lib.parent), "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()
    assert out[0] == "rmsnorm_stash_v8_kernel"
    assert out[1] == "silu_wave_kernel"
    assert out[2] == "IPL_ERROR_INVALID_VALUE: epsilon must be positive"
    assert out[3].startswith("IPL_ERROR_MISALIGNED: ") and "divisible by 8" in out[3]


def test_abi_version_and_status_strings() -> None:
    lib = capi.library()
    assert lib.ipl_abi_version() == 1
    assert lib.ipl_status_string(capi.IPL_ERROR_MISALIGNED) == b"IPL_ERROR_MISALIGNED"
    assert lib.ipl_status_string(99) == b"IPL_UNKNOWN_STATUS"


@pytest.mark.parametrize(
    "args, status, message",
    [
        ((BASE, BASE + 4096, BASE + 8192, 4, 3584, 0.0), capi.IPL_ERROR_INVALID_VALUE, "epsilon must be positive"),
        ((BASE, BASE + 4096, BASE + 8192, 4, 3584, -1.0), capi.IPL_ERROR_INVALID_VALUE, "epsilon must be positive"),
        ((BASE, BASE + 4096, BASE + 8192, 4, 0, 1e-6), capi.IPL_ERROR_INVALID_VALUE, "non-empty final dimension"),
        ((BASE, BASE + 4096, BASE + 8192, -1, 16, 1e-6), capi.IPL_ERROR_INVALID_VALUE, "non-negative"),
        ((0, BASE + 4096, BASE + 8192, 4, 16, 1e-6), capi.IPL_ERROR_INVALID_VALUE, "non-null"),
        ((BASE, BASE, BASE + 8192, 4, 16, 1e-6), capi.IPL_ERROR_INVALID_VALUE, "must not alias"),
        ((BASE + 1, BASE + 4096, BASE + 8192, 4, 16, 1e-6), capi.IPL_ERROR_INVALID_VALUE, "2-byte aligned"),
        ((BASE, BASE + 4096, BASE + 8192, 4, 2**31, 1e-6), capi.IPL_ERROR_TOO_LARGE, "hidden dimension is too large"),
        ((BASE, BASE + 4096, BASE + 8192, 2**31, 16, 1e-6), capi.IPL_ERROR_TOO_LARGE, "number of rows is too large"),
    ],
)
def test_rms_argument_errors(args, status, message) -> None:
    with pytest.raises(capi.IplError, match=message) as info:
        capi.fused_add_rms_norm(*args)
    assert info.value.status == status


@pytest.mark.parametrize(
    "args, message",
    [
        ((BASE, BASE + 4096, BASE + 8192, 4, 3584, 0.0), "epsilon must be positive"),
        ((0, BASE + 4096, BASE + 8192, 4, 3584, 1e-6), "output, input and weight must be non-null"),
        ((BASE, BASE + 4096, BASE + 8192, 4, 0, 1e-6), "non-empty final dimension"),
        ((BASE + 1, BASE + 4096, BASE + 8192, 4, 16, 1e-6), "2-byte aligned"),
    ],
)
def test_plain_rms_argument_errors(args, message) -> None:
    with pytest.raises(capi.IplError, match=message):
        capi.rms_norm(*args)


def test_plain_rms_in_place_is_accepted_by_the_plan() -> None:
    # output == input is allowed (vLLM calls it out of place, callers may reuse the buffer).
    # Each stash thread reads its chunks into registers before it writes them, so in place is safe.
    assert capi.rms_norm_plan(BASE, BASE, BASE + 8192, 2048, 3584) == "rmsnorm_stash_kernel<4, plain>"
    assert capi.rms_norm_plan(BASE + 2, BASE, BASE + 8192, 8, 3584) == "rmsnorm_rowwise_kernel<cached, plain>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 64, 8192) == "rmsnorm_cta_kernel<2, plain>"
    # Rows of 8192+ elements, 4096+ of them: eight chunks a thread.
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 4095, 8192) == "rmsnorm_stash_kernel<4, plain>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 8192, 8192) == "rmsnorm_stash_kernel<8, plain>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 4096, 12288) == "rmsnorm_stash_kernel<8, plain>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 32768, 4096) == "rmsnorm_stash_kernel<4, plain>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 32768, 2048) == "rmsnorm_stash_kernel<4, plain>"
    # x and out one element off 16 bytes alike: the shifted kernel up to H = 4096, then the staged ring.
    assert capi.rms_norm_plan(BASE + 2, BASE + (1 << 34) + 2, BASE + 8192, 2048, 3584) == (
        "rmsnorm_shifted_kernel<1, plain>"
    )
    assert capi.rms_norm_plan(BASE + 2, BASE + (1 << 34) + 2, BASE + 8192, 2048, 8192).startswith(
        "rmsnorm_staged_kernel"
    )
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 4096, 16384) == "rmsnorm_stash_kernel<8, plain>"


def test_fp8_quant_arguments_and_plans() -> None:
    with pytest.raises(capi.IplError, match="output and scale must be non-null"):
        capi.fused_add_rms_norm_static_fp8_quant(BASE, BASE + 4096, BASE + 8192, BASE + 12288, 0, 4, 16, 1e-6)
    with pytest.raises(capi.IplError, match="epsilon must be positive"):
        capi.fused_add_rms_norm_static_fp8_quant(BASE, BASE + 4096, BASE + 8192, BASE + 12288, BASE, 4, 16, 0.0)
    plan = capi.fused_add_rms_norm_static_fp8_quant_plan
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 2048, 3584) == "rmsnorm_stash_v8_kernel<fp8>"
    assert plan(BASE + 8, BASE + 4096, BASE + (1 << 34), BASE + 12288, 2048, 3584) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12290, 2048, 3584) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 262144, 8192) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 600, 16384) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 600, 18432) == "rmsnorm_stash_kernel<8, fp8, capped>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 600, 32768) == "rmsnorm_stash_kernel<8, fp8>"
    # Longer aligned rows: the cluster kernel, eight CTAs a row, up to H = 131072.
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 600, 32776) == "rmsnorm_cluster_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 8, 32768) == "rmsnorm_cluster_kernel<4, fp8>"
    # The fp8 output has no staged plan: rows it cannot vectorise go to the row kernel.
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 600, 131080).startswith("rmsnorm_rowwise_kernel")
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 100000, 1024) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 100000, 896) == "rmsnorm_warp_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 2048, 1024) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 7, 3584) == "rmsnorm_cta_kernel<1, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 9000, 4096) == "rmsnorm_stash_kernel<4, fp8>"
    # The fp8 op's one-chunk CTA holds 64 registers: 2 CTAs of 448 threads an SM at H = 3584 (where
    # the 256-bit stash kernel does not apply: here a weight off 16 bytes).
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12290, 296, 3584) == "rmsnorm_cta_kernel<1, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12290, 297, 3584) == "rmsnorm_stash_kernel<4, fp8>"
    assert plan(BASE, BASE + 4096, BASE + (1 << 34), BASE + 12288, 296, 3584) == "rmsnorm_stash_v8_kernel<fp8>"
    # fp8 vector stores need 16-byte aligned rows and an 8-byte aligned output.
    assert plan(BASE + 4, BASE + 4098, BASE + (1 << 34) + 2, BASE + 12288, 2048, 3584).startswith(
        "rmsnorm_rowwise_kernel"
    )
    assert plan(BASE + 1, BASE + 4096, BASE + (1 << 34), BASE + 12288, 2048, 3584).startswith(
        "rmsnorm_rowwise_kernel"
    )


def test_rms_empty_batch_is_a_no_op() -> None:
    # rows == 0 returns before any device query.
    capi.fused_add_rms_norm(0, 0, 0, 0, 3584, 1e-6)


@pytest.mark.parametrize(
    "fn, args, status, message",
    [
        (capi.silu_and_mul_packed, (BASE, BASE + 4096, 4, 18), capi.IPL_ERROR_MISALIGNED,
         "the output width must be divisible by 8"),
        (capi.silu_and_mul_packed, (BASE + 2, BASE + 4096, 4, 16), capi.IPL_ERROR_MISALIGNED,
         "input and output must be 16-byte aligned"),
        (capi.silu_and_mul_packed, (BASE, BASE + 4098, 4, 16), capi.IPL_ERROR_MISALIGNED,
         "input and output must be 16-byte aligned"),
        (capi.silu_and_mul, (0, BASE, 4, 16), capi.IPL_ERROR_INVALID_VALUE, "non-null"),
        (capi.silu_and_mul, (BASE, BASE + 4096, -1, 16), capi.IPL_ERROR_INVALID_VALUE, "non-negative"),
        (capi.silu_and_mul, (BASE + 1, BASE + 4096, 1, 16), capi.IPL_ERROR_INVALID_VALUE, "2-byte aligned"),
        (capi.silu_and_mul, (BASE, BASE + 4096, 2**40, 2**40), capi.IPL_ERROR_TOO_LARGE, "too large"),
    ],
)
def test_silu_argument_errors(fn, args, status, message) -> None:
    with pytest.raises(capi.IplError, match=message) as info:
        fn(*args)
    assert info.value.status == status


def test_silu_empty_is_a_no_op() -> None:
    capi.silu_and_mul(0, 0, 0, 18944)
    capi.silu_and_mul_packed(0, 0, 128, 0)


def rms_plan(x_off: int, r_off: int, w_off: int, rows: int, hidden: int) -> str:
    # Offsets in bf16 elements from 256-byte aligned bases.
    return capi.fused_add_rms_norm_plan(
        BASE + 2 * x_off, BASE + (1 << 34) + 2 * r_off, BASE + (1 << 35) + 2 * w_off, rows, hidden
    )


def test_rms_plan_selection() -> None:
    # 2048 x 3584 aligned (the bench workload): a 224-thread CTA per row, one 32-byte pair of chunks
    # a thread; with a weight off 16 bytes, 128 threads of four 16-byte chunks.
    assert rms_plan(0, 0, 0, 2048, 3584) == "rmsnorm_stash_v8_kernel"
    assert rms_plan(0, 0, 1, 2048, 3584) == "rmsnorm_stash_kernel<4>"
    # x and residual both off 16 bytes alike, more than 256 rows: the shifted kernel, one instance
    # per phase, up to H = 12288; fewer rows or longer ones: the staged kernel. 257-4096 rows of
    # 1536-4080 elements (H % 16 == 0) with a 16-byte aligned weight, rows in the first half of a
    # 32-byte block: its 256-bit variant.
    for off in range(1, 8):
        assert rms_plan(off, off, 0, 2048, 3584) == f"rmsnorm_shifted_v8_kernel<{off}>"
        assert rms_plan(off, off, 1, 2048, 3584) == f"rmsnorm_shifted_kernel<{off}>"
        assert rms_plan(off + 8, off + 8, 0, 2048, 3584) == f"rmsnorm_shifted_kernel<{off}>"  # second half
    assert rms_plan(1, 1, 0, 4097, 3584) == "rmsnorm_shifted_kernel<1>"
    assert rms_plan(1, 1, 0, 2048, 4096) == "rmsnorm_shifted_kernel<1>"
    assert rms_plan(1, 1, 0, 2048, 4080) == "rmsnorm_shifted_v8_kernel<1>"
    assert capi.rms_norm_plan(BASE + 2, BASE + (1 << 34) + 2, BASE + 8192, 2048, 3584) == "rmsnorm_shifted_kernel<1, plain>"
    assert rms_plan(3, 3, 1, 300, 12288) == "rmsnorm_shifted_kernel<3>"
    assert rms_plan(1, 1, 0, 256, 3584).startswith("rmsnorm_staged_kernel")
    assert rms_plan(1, 1, 0, 2048, 12296).startswith("rmsnorm_staged_kernel")
    assert rms_plan(1, 1, 0, 2048, 1024).startswith("rmsnorm_staged_kernel")
    assert capi.fused_add_rms_norm_static_fp8_quant_plan(BASE + 2, BASE + 2, BASE + (1 << 34) + 2, BASE + 8192,
                                                          2048, 3584).startswith("rmsnorm_rowwise_kernel")
    # Only one of them misaligned (the reference's misaligned tests): the general row kernel.
    assert rms_plan(1, 0, 0, 8, 3584) == "rmsnorm_rowwise_kernel<cached>"
    assert rms_plan(0, 1, 0, 8, 3584) == "rmsnorm_rowwise_kernel<cached>"
    # Up to 256 aligned rows (decode batches): a CTA per row, the row in registers; a misaligned
    # weight is loaded element by element.
    assert rms_plan(0, 0, 1, 8, 3584) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 1, 3584) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 256, 8192) == "rmsnorm_cta_kernel<2>"
    assert rms_plan(0, 0, 0, 100, 16384) == "rmsnorm_cta_kernel<4>"
    assert rms_plan(0, 0, 0, 5, 2048) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 64, 2056) == "rmsnorm_cta_kernel<1>"
    # One chunk a thread (H <= 4096): the CTA per row also while every row's CTA is resident at once
    # - 148 SMs x 3 CTAs of 448 threads at H = 3584, x 6 of 256 at 2048, x 8 of 192 at 1536 - where
    # the 256-bit stash kernel does not apply (here: a weight off 16 bytes; below H = 1536).
    for rows in (257, 148 * 2, 148 * 3):
        assert rms_plan(0, 0, 1, rows, 3584) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 1, 148 * 3, 4096) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 1, 148 * 6, 2048) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 1, 148 * 8, 1536) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 148 * 8, 1032) == "rmsnorm_cta_kernel<1>"  # at most 8 CTAs an SM counted
    assert rms_plan(0, 0, 0, 148 * 8 + 1, 1032) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 1, 257, 5120) == "rmsnorm_stash_kernel<4>"
    # 257-4096 aligned rows of 1536-5120 elements (H % 16 == 0, 16-byte aligned weight): the
    # 256-bit stash kernel, the cta kernel's one-wave launches included.
    for rows in (257, 148 * 3, 148 * 3 + 1, 2048, 4096):
        for hidden in (1536, 2048, 2560, 3584, 4096, 5120):
            assert rms_plan(0, 0, 0, rows, hidden) == "rmsnorm_stash_v8_kernel"
    assert rms_plan(0, 0, 0, 2048, 5136) == "rmsnorm_stash_kernel<4>"  # wider
    assert rms_plan(0, 0, 0, 2048, 1528) == "rmsnorm_stash_kernel<4>"  # narrower
    assert rms_plan(0, 0, 0, 2048, 3592) == "rmsnorm_stash_kernel<4>"  # H % 16 != 0
    assert capi.fused_add_rms_norm_plan(BASE + 16, BASE + (1 << 34) + 16, BASE + (1 << 35), 2048, 3584) == \
        "rmsnorm_stash_kernel<4>"  # rows 16 bytes off 32
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 2048, 3584) == "rmsnorm_stash_kernel<4, plain>"
    # More rows, up to 12288 elements each: a small CTA for every row (128 threads of four chunks
    # at H = 3584), the row-sharded workload's 2^28-element shards included.
    for rows in (4097, 148 * 28, 32768):
        assert rms_plan(0, 0, 0, rows, 3584) == "rmsnorm_stash_kernel<4>"
    for rows in (148 * 3 + 1, 148 * 6, 148 * 14, 148 * 16):
        assert rms_plan(0, 0, 1, rows, 3584) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 148 * 28, 4096) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 1, 148 * 6 + 1, 2048) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 1, 148 * 8 + 1, 1536) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 16384, 8192) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 20000, 12288) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 262144, 8192) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 100000, 12288) == "rmsnorm_stash_kernel<4>"
    # Up to 16384 elements (512 threads of four chunks); longer rows: the staged kernel.
    assert rms_plan(0, 0, 0, 32768, 16384) == "rmsnorm_stash_kernel<4>"
    assert rms_plan(0, 0, 0, 300, 13312) == "rmsnorm_stash_kernel<4>"
    # 16384 < H <= 32768: eight chunks a thread; add+RMSNorm and the fp8 op at 96 registers (two CTAs
    # an SM) up to 320 threads (H = 20480) for more than 256 rows, at 128 registers otherwise.
    assert rms_plan(0, 0, 0, 1000, 16392) == "rmsnorm_stash_kernel<8, capped>"
    assert rms_plan(0, 0, 0, 8192, 18432) == "rmsnorm_stash_kernel<8, capped>"
    assert rms_plan(0, 0, 0, 257, 20480) == "rmsnorm_stash_kernel<8, capped>"
    assert rms_plan(0, 0, 0, 257, 18432) == "rmsnorm_stash_kernel<8, capped>"
    assert rms_plan(0, 0, 0, 8192, 20488) == "rmsnorm_stash_kernel<8>"
    assert rms_plan(0, 0, 0, 8192, 32768) == "rmsnorm_stash_kernel<8>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 8192, 18432) == "rmsnorm_stash_kernel<8, plain>"
    # Longer aligned rows: the cluster kernel (test_cluster_plan_selection); rows off 16 bytes too
    # long for the CTA kernels: the staged ring while two stages fit, else the two-pass row kernel.
    assert rms_plan(0, 0, 0, 1000, 32776) == "rmsnorm_cluster_kernel<4>"
    assert rms_plan(0, 0, 0, 1000, 131080) == "rmsnorm_rowwise_kernel<two-pass>"
    assert rms_plan(1, 1, 0, 1000, 16392).startswith("rmsnorm_staged_kernel")
    # Short aligned rows: a CTA per row while the CTAs are resident at once; beyond that a warp per
    # row (eight rows a CTA) for rows that move under 7 KiB, the stash kernel for longer ones.
    assert rms_plan(0, 0, 3, 5, 1000) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 5, 256) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 148 * 8, 128) == "rmsnorm_cta_kernel<1>"
    assert rms_plan(0, 0, 0, 148 * 8 + 1, 128) == "rmsnorm_warp_kernel<1>"
    assert rms_plan(0, 0, 0, 148 * 64, 512) == "rmsnorm_warp_kernel<2>"
    assert rms_plan(0, 0, 0, 2000, 768) == "rmsnorm_warp_kernel<4>"  # 6 KiB a row
    assert rms_plan(0, 0, 0, 2000, 896) == "rmsnorm_stash_kernel<4>"  # 7 KiB
    assert rms_plan(0, 0, 0, 148 * 64, 1024) == "rmsnorm_stash_kernel<4>"
    assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, 100000, 1024) == "rmsnorm_warp_kernel<4, plain>"
    assert rms_plan(1, 1, 0, 5, 1024).startswith("rmsnorm_staged_kernel")
    # Widths that are not a multiple of 8 stay on the staged kernel when x and residual share
    # their offset.
    assert rms_plan(0, 0, 0, 64, 1001).startswith("rmsnorm_staged_kernel")
    assert rms_plan(0, 0, 0, 64, 2052).startswith("rmsnorm_staged_kernel")
    assert rms_plan(0, 0, 0, 100000, 3580).startswith("rmsnorm_staged_kernel")
    # Widths under one 16-byte chunk, many rows: the planner's occupancy arithmetic is skipped.
    for hidden in range(1, 8):
        for rows in (300, 1000, 100000):
            assert rms_plan(0, 0, 0, rows, hidden).startswith(("rmsnorm_staged_kernel", "rmsnorm_rowwise_kernel"))
            assert capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, rows, hidden) != "invalid"
    # Rows too long for two stages fall back to the two-pass row kernel (aligned ones of H % 8 == 0
    # to the cluster kernel).
    assert rms_plan(0, 0, 0, 64, 40002) == "rmsnorm_rowwise_kernel<two-pass>"
    assert rms_plan(1, 0, 0, 64, 40000) == "rmsnorm_rowwise_kernel<two-pass>"
    assert rms_plan(0, 0, 0, 64, 40000) == "rmsnorm_cluster_kernel<4>"
    assert rms_plan(0, 0, 0, 0, 3584) == "none"
    assert rms_plan(0, 0, 0, 4, 0) == "invalid"


def silu_plan(out_off: int, in_off: int, rows: int, inter: int) -> str:
    return capi.silu_and_mul_plan(BASE + 2 * out_off, BASE + (1 << 34) + 2 * in_off, rows, inter)


def test_cluster_plan_selection() -> None:
    """Rows split over a thread-block cluster: aligned rows longer than 32768 elements always, few
    long rows where one CTA a row leaves SMs idle; the kernel name carries the chunks a thread
    (the most that leave each CTA 128+ threads)."""
    plain = lambda rows, hidden: capi.rms_norm_plan(BASE, BASE + (1 << 34), BASE + 8192, rows, hidden)
    # H > 32768: eight CTAs a row at any row count (512 threads of four chunks at H = 131072).
    for rows in (1, 64, 2048, 262144):
        assert rms_plan(0, 0, 0, rows, 65536) == "rmsnorm_cluster_kernel<4>"
        assert plain(rows, 131072) == "rmsnorm_cluster_kernel<4, plain>"
    # 16384 < H <= 32768: up to 256 rows (RMSNorm 128), then the stash kernel.
    assert rms_plan(0, 0, 0, 256, 32768) == "rmsnorm_cluster_kernel<4>"
    assert rms_plan(0, 0, 0, 257, 32768) == "rmsnorm_stash_kernel<8>"
    assert plain(128, 32768) == "rmsnorm_cluster_kernel<4, plain>"
    assert plain(129, 32768) == "rmsnorm_stash_kernel<8, plain>"
    # 8192 <= H <= 16384: up to 32 rows; 6144 <= H < 8192: up to 16; shorter rows never.
    assert rms_plan(0, 0, 0, 1, 8192) == "rmsnorm_cluster_kernel<1>"  # 8 CTAs of 128 threads
    assert rms_plan(0, 0, 0, 32, 8192) == "rmsnorm_cluster_kernel<2>"  # 4 CTAs of 128 threads
    assert rms_plan(0, 0, 0, 33, 8192) == "rmsnorm_cta_kernel<2>"
    assert rms_plan(0, 0, 0, 16, 6144) == "rmsnorm_cluster_kernel<1>"
    assert rms_plan(0, 0, 0, 17, 6144) == "rmsnorm_cta_kernel<2>"
    assert rms_plan(0, 0, 0, 1, 6136) == "rmsnorm_cta_kernel<2>"
    assert rms_plan(0, 0, 0, 1, 4096) == "rmsnorm_cta_kernel<1>"
    # H >= 12288, more rows than SMs up to 256 (where one CTA a row needs a second wave).
    assert rms_plan(0, 0, 0, 148, 12288) == "rmsnorm_cta_kernel<4>"
    assert rms_plan(0, 0, 0, 149, 12288) == "rmsnorm_cluster_kernel<2>"
    assert rms_plan(0, 0, 0, 256, 16384) == "rmsnorm_cluster_kernel<4>"
    assert rms_plan(0, 0, 0, 257, 16384) == "rmsnorm_stash_kernel<4>"
    # Misaligned rows, widths not a multiple of 8 and misaligned fp8 outputs stay off it; a
    # misaligned weight does not.
    assert not rms_plan(1, 1, 0, 8, 65536).startswith("rmsnorm_cluster")
    assert not rms_plan(0, 0, 0, 8, 65540).startswith("rmsnorm_cluster")
    assert rms_plan(0, 0, 1, 8, 65536) == "rmsnorm_cluster_kernel<4>"
    assert not capi.fused_add_rms_norm_static_fp8_quant_plan(BASE, BASE + 4096, BASE + (1 << 34) + 2, BASE + 12288,
                                                             8, 65536).startswith("rmsnorm_cluster")


def test_silu_plan_selection() -> None:
    # 128 x 2368 = 303,104 16-byte packs: one wave of 148 SMs x 2048 threads, one pack a thread.
    assert silu_plan(0, 0, 128, 18944) == "silu_wave_kernel"
    assert silu_plan(8, 0, 128, 18944) == "silu_wave_kernel"
    assert silu_plan(0, 0, 127, 18952) == "silu_wave_kernel"
    assert silu_plan(0, 0, 128, 18952) == "silu_vector_kernel<16>"  # 303,232 packs: above one wave
    # At most half a wave, or more than one: one 32-byte pack a thread where aligned, else 16.
    assert silu_plan(0, 0, 64, 18944) == "silu_vector_kernel<32>"
    assert silu_plan(0, 0, 65, 18944) == "silu_wave_kernel"
    assert silu_plan(0, 0, 129, 18944) == "silu_vector_kernel<32>"
    assert silu_plan(8, 0, 2048, 18944) == "silu_vector_kernel<16>"
    assert silu_plan(0, 0, 2048, 18952) == "silu_vector_kernel<16>"
    assert silu_plan(4, 0, 128, 18944) == "silu_scalar_kernel"  # 8 bytes off: no 16-byte packs
    assert silu_plan(0, 0, 3, 1001) == "silu_scalar_kernel"
    assert silu_plan(1, 0, 128, 18944) == "silu_scalar_kernel"
    assert silu_plan(0, 0, 0, 18944) == "none"
