"""The compiled kernels' register budgets, from the ptxas report the build writes beside the library.

The planner counts how many CTAs of the CTA-per-row kernel an SM holds at once from the registers
its one-chunk instances are held to (40 for the bf16 ops, 64 for the fp8 op), the stash kernel's
eight rows per SM rest on its 64-register bound, and its capped instance for rows of up to 20480
elements on two CTAs an SM at 96 registers; the cluster kernel's 2 CTAs of 512 threads an SM on its
64-register bound. A compiler that broke any of them, or began
to spill, would change the measured crossovers silently; this test reads the report instead.
"""

from __future__ import annotations

import re
from pathlib import Path

import pytest

REPORT = (Path(__file__).resolve().parents[1] / "inference-performance-lab_b200" / "inference_performance_lab"
          / "_native" / "libipl_b200.ptxas.txt")


def kernel_resources() -> dict[str, tuple[int, int]]:
    """{mangled kernel name: (registers, spill store bytes)} from the ptxas report."""
    if not REPORT.exists():
        pytest.skip("library not built here (no ptxas report)")
    resources: dict[str, tuple[int, int]] = {}
    name, spills = None, 0
    for line in REPORT.read_text().splitlines():
        m = re.search(r"Compiling entry function '(\w+)'", line)
        if m:
            name, spills = m.group(1), 0
            continue
        m = re.search(r"(\d+) bytes spill stores", line)
        if m and name:
            spills = int(m.group(1))
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and name:
            resources[name] = (int(m.group(1)), spills)
            name = None
    return resources


def test_cta_row_kernel_one_chunk_registers() -> None:
    res = kernel_resources()
    for mode, cap in ((0, 40), (1, 40), (2, 64)):
        regs, spills = res[f"_ZN3ipl18rmsnorm_cta_kernelILi1ELi{mode}EEEvNS_13WarpRowParamsE"]
        assert regs <= cap and spills == 0, (mode, regs, spills)


def test_stash_kernel_registers() -> None:
    res = kernel_resources()
    # <4, mode> and <8, plain> at 64 (eight rows an SM at four chunks); <8> of add+RMSNorm and the
    # fp8 op at 128 (one CTA an SM), their capped instances at 96 (two CTAs of 320 threads).
    caps = {f"_ZN3ipl20rmsnorm_stash_kernelILi{u}ELi{m}ELb{c}EEEvNS_13WarpRowParamsE": cap
            for u, m, c, cap in ((4, 0, 0, 64), (4, 1, 0, 64), (4, 2, 0, 64), (8, 1, 0, 64),
                                 (8, 0, 0, 128), (8, 2, 0, 128), (8, 0, 1, 96), (8, 2, 1, 96))}
    names = [n for n in res if n.startswith("_ZN3ipl20rmsnorm_stash_kernel")]
    assert sorted(names) == sorted(caps)
    for n, cap in caps.items():
        regs, spills = res[n]
        assert regs <= cap and spills == 0, (n, regs, spills)


def test_shifted_kernel_registers() -> None:
    res = kernel_resources()
    names = [n for n in res if n.startswith("_ZN3ipl22rmsnorm_shifted_kernel")]
    assert len(names) == 14  # seven phases, add+RMSNorm and RMSNorm
    for n in names:
        regs, spills = res[n]
        assert regs <= 64 and spills == 0, (n, regs, spills)


def test_stash_v8_kernel_registers() -> None:
    """The 256-bit stash kernel's two instances (add+RMSNorm, fp8 output) within 64 registers."""
    res = kernel_resources()
    names = [n for n in res if n.startswith("_ZN3ipl23rmsnorm_stash_v8_kernel")]
    assert len(names) == 2, names
    for n in names:
        regs, spills = res[n]
        assert regs <= 64 and spills == 0, (n, regs, spills)


def test_shifted_v8_kernel_registers() -> None:
    """The 256-bit shifted kernel's seven phase instances within 64 registers (four CTAs an SM)."""
    res = kernel_resources()
    names = [n for n in res if n.startswith("_ZN3ipl25rmsnorm_shifted_v8_kernel")]
    assert len(names) == 7, names
    for n in names:
        regs, spills = res[n]
        assert regs <= 64 and spills == 0, (n, regs, spills)


def test_cluster_kernel_registers() -> None:
    """Nine instances (1, 2 and 4 chunks a thread; three modes), each within the 64 registers that
    let two CTAs of 512 threads, or four of 256, share an SM."""
    res = kernel_resources()
    names = [n for n in res if n.startswith("_ZN3ipl22rmsnorm_cluster_kernel")]
    assert len(names) == 9, names
    for n in names:
        regs, spills = res[n]
        assert regs <= 64 and spills == 0, (n, regs, spills)


def test_silu_wave_kernel_registers() -> None:
    """The one-wave SiLU kernel within the 32 registers that let two CTAs of 1024 threads share an
    SM (2 x 1024 x 32 = 65,536)."""
    res = kernel_resources()
    names = [n for n in res if n.startswith("_ZN3ipl16silu_wave_kernel")]
    assert len(names) == 1, names
    regs, spills = res[names[0]]
    assert regs <= 32 and spills == 0, (names[0], regs, spills)


def test_no_kernel_spills() -> None:
    res = kernel_resources()
    spilling = {n: s for n, (_, s) in res.items() if s}
    assert not spilling, spilling
