"""Build step for the native libraries (in-tree, sm_100a only).

Produces, under ``inference_performance_lab/_native/``:

* ``libipl_b200.so`` - every CUDA kernel and the C ABI of ``include/ipl_b200.h`` (nvcc, static
  cudart, no torch dependency);
* ``inference_performance_lab_cuda.so`` - the stable-LibTorch-ABI op registration
  (``csrc/torch_ops.cpp``, g++), linked against ``libipl_b200.so`` through ``$ORIGIN``.

Run ``python inference-performance-lab_b200/build.py`` (or call :func:`build`). Rebuilds only what
is older than its sources or was built with different flags.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_ROOT.parent
CSRC = PACKAGE_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
NATIVE = PACKAGE_ROOT / "inference_performance_lab" / "_native"

LIB_NAME = "libipl_b200.so"
TORCH_OPS_NAME = "inference_performance_lab_cuda.so"
# Test-only variant of LIB_NAME (never loaded by the package): see build_wait_test().
WAIT_TEST_NAME = "test/libipl_b200_waittest.so"
WAIT_TEST_DEFINES = ["-DIPL_WAIT_LIMIT_NS=1000000ull", "-DIPL_TEST_STAGED_SKIP_ROW=0"]

# Stable ABI target: torch 2.10 (the oldest version that has every call the shim uses).
TORCH_TARGET_VERSION = "0x020a000000000000"

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xptxas=-v",
    "-Xcompiler=-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _host_cxx() -> str:
    """The system C++ compiler, whose libstdc++ is the shared one torch itself uses.

    The shim throws C++ exceptions (std::runtime_error from STD_TORCH_CHECK) into torch's
    dispatcher, so it must share torch's libstdc++.so.6. A compiler that links its own static
    libstdc++ (as the one named by $CXX in some images does) embeds and exports a second copy,
    and building an exception message through it crashes inside the host process.
    """
    for candidate in ("/usr/bin/g++", shutil.which("g++")):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("g++ not found")


def _stamp(sources: list[Path], flags: list[str]) -> str:
    """Hash of the flags (repo paths made relative, so a moved checkout still matches) and sources."""
    digest = hashlib.sha256()
    for flag in flags:
        digest.update(flag.replace(str(REPO_ROOT), "<repo>").encode())
    for source in sources:
        digest.update(source.read_bytes())
    return digest.hexdigest()


def _up_to_date(output: Path, stamp: str) -> bool:
    stamp_file = output.with_suffix(output.suffix + ".stamp")
    return output.exists() and stamp_file.exists() and stamp_file.read_text() == stamp


def _write_stamp(output: Path, stamp: str) -> None:
    output.with_suffix(output.suffix + ".stamp").write_text(stamp)


def _run(command: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(command), flush=True)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            f"build command failed ({result.returncode}): {' '.join(command)}\n"
            f"{result.stdout}\n{result.stderr}"
        )
    return result.stdout + result.stderr


def build_native(verbose: bool = False) -> Path:
    """Compile the CUDA kernels + C ABI into libipl_b200.so."""
    NATIVE.mkdir(parents=True, exist_ok=True)
    output = NATIVE / LIB_NAME
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "ipl_b200.h"]
    flags = [*NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}"]
    stamp = _stamp(sources, flags)
    if _up_to_date(output, stamp):
        return output
    command = [
        _nvcc(),
        *flags,
        "-shared",
        "-o",
        str(output),
        str(CSRC / "ipl_b200.cu"),
    ]
    log = _run(command, verbose)
    (NATIVE / "libipl_b200.ptxas.txt").write_text(log)
    _write_stamp(output, stamp)
    return output


def build_wait_test(verbose: bool = False) -> Path:
    """The same kernels and C ABI built for a test of the staged kernel's bounded waits: every wait
    gives up after 1 ms instead of 2 s, and CTA 0 of the staged kernel never issues its row 0, so
    the consumers waiting for that row run out of time. A test loads it (ctypes) to check that the
    kernel then returns, records the fault bit and leaves the context usable."""
    output = NATIVE / WAIT_TEST_NAME
    output.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "ipl_b200.h"]
    flags = [*NVCC_FLAGS, *WAIT_TEST_DEFINES, f"-I{INCLUDE}", f"-I{CSRC}"]
    stamp = _stamp(sources, flags)
    if _up_to_date(output, stamp):
        return output
    _run([_nvcc(), *flags, "-shared", "-o", str(output), str(CSRC / "ipl_b200.cu")], verbose)
    _write_stamp(output, stamp)
    return output


def build_torch_ops(verbose: bool = False) -> Path:
    """Compile the stable-ABI op registration, linked against libipl_b200.so."""
    import torch

    torch_root = Path(torch.__file__).resolve().parent
    output = NATIVE / TORCH_OPS_NAME
    sources = [CSRC / "torch_ops.cpp", INCLUDE / "ipl_b200.h"]
    flags = [
        "-O3",
        "-std=c++17",
        "-fPIC",
        f"-DTORCH_TARGET_VERSION={TORCH_TARGET_VERSION}",
        f"-I{torch_root / 'include'}",
        f"-I{INCLUDE}",
    ]
    stamp = _stamp(sources + [NATIVE / LIB_NAME], flags)
    if _up_to_date(output, stamp):
        return output
    command = [
        _host_cxx(),
        *flags,
        "-shared",
        "-o",
        str(output),
        str(CSRC / "torch_ops.cpp"),
        f"-L{NATIVE}",
        "-lipl_b200",
        f"-L{torch_root / 'lib'}",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-lc10",
        "-Wl,-rpath,$ORIGIN",
        f"-Wl,-rpath,{torch_root / 'lib'}",
    ]
    _run(command, verbose)
    _write_stamp(output, stamp)
    return output


def build(verbose: bool = False, tests: bool = False) -> None:
    """Build both libraries (and, with ``tests``, the test-only wait-limit variant); concurrent
    callers (e.g. several ranks) serialise on a lock file."""
    import fcntl

    NATIVE.mkdir(parents=True, exist_ok=True)
    with open(NATIVE / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            build_native(verbose)
            build_torch_ops(verbose)
            if tests:
                build_wait_test(verbose)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv, tests="--tests" in sys.argv)
