"""Builds the reference's own CUDA kernels for sm_100a, as a same-box comparison arm.

TEST INFRASTRUCTURE ONLY (like the rest of ``oracle/``): the product never loads this library.
It is the reference's custom-op library compiled from its sources where they lie
(``csrc/fused_add_rms_norm_kernel.cu``, ``csrc/silu_and_mul_kernel.cu``, ``csrc/torch_ops.cpp`` of
sreeganeshji/inference-performance-lab), with two build-level changes and no edit of any source:

* ``oracle/ref_overlay/`` is put on the include path before torch's headers. Its
  ``torch/csrc/stable/accelerator.h`` includes torch's own header and supplies
  ``getCurrentStream(i).nativeHandle()``, the one stable-ABI accessor the reference's wrappers use
  (fused_add_rms_norm_kernel.cu:305, silu_and_mul_kernel.cu:121,174) that torch 2.11 lacks;
* the op namespace token ``inference_performance_lab`` is defined to
  ``inference_performance_lab_ref`` when compiling ``torch_ops.cpp``, so the reference's ops register
  as ``torch.ops.inference_performance_lab_ref.*`` beside this repository's
  ``torch.ops.inference_performance_lab.*`` in one process.

Output: ``oracle/_ref/libref_kernels.so`` (git-ignored; it travels with the working tree to a GPU
machine, where the reference's sources are not needed). Kernels compile with
``-gencode arch=compute_100a,code=sm_100a`` and the flags of the reference's own loader
(src/inference_performance_lab/kernels/extension.py:18-35: ``-O3``, ``-std=c++17``).

    python oracle/build_ref_kernels.py --reference <path to the reference checkout>
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
OUT_DIR = ORACLE_DIR / "_ref"
LIBRARY = OUT_DIR / "libref_kernels.so"
OVERLAY = ORACLE_DIR / "ref_overlay"
SOURCES = ("csrc/fused_add_rms_norm_kernel.cu", "csrc/silu_and_mul_kernel.cu", "csrc/torch_ops.cpp")
TORCH_TARGET_VERSION = "0x020a000000000000"


def _run(command: list[str]) -> None:
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"command failed ({result.returncode}): {' '.join(command)}\n{result.stdout}\n{result.stderr}")


def build(reference: Path) -> Path:
    """Compiles the three reference sources into oracle/_ref/libref_kernels.so."""
    import torch

    reference = reference.resolve()
    missing = [s for s in SOURCES if not (reference / s).is_file()]
    if missing:
        raise FileNotFoundError(f"reference sources not found under {reference}: {missing}")
    inputs = [reference / s for s in SOURCES] + list(OVERLAY.rglob("*.h")) + [Path(__file__)]
    if LIBRARY.exists() and LIBRARY.stat().st_mtime > max(p.stat().st_mtime for p in inputs):
        return LIBRARY
    torch_root = Path(torch.__file__).resolve().parent
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    nvcc = cuda_home / "bin" / "nvcc"
    cxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else shutil.which("g++")
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    includes = [f"-I{OVERLAY}", f"-I{torch_root / 'include'}", f"-I{cuda_home / 'include'}"]
    defines = [f"-DTORCH_TARGET_VERSION={TORCH_TARGET_VERSION}"]
    objects = []
    for source in SOURCES[:2]:
        obj = OUT_DIR / (Path(source).stem + ".o")
        _run([str(nvcc), "-gencode=arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
              "-Xcompiler=-fPIC", *defines, *includes, "-c", str(reference / source), "-o", str(obj)])
        objects.append(obj)
    ops_obj = OUT_DIR / "torch_ops.o"
    _run([cxx, "-O3", "-std=c++17", "-fPIC", *defines, "-Dinference_performance_lab=inference_performance_lab_ref",
          *includes, "-c", str(reference / SOURCES[2]), "-o", str(ops_obj)])
    objects.append(ops_obj)
    _run([cxx, "-shared", "-o", str(LIBRARY), *map(str, objects), f"-L{cuda_home / 'lib64'}", "-lcudart",
          f"-L{torch_root / 'lib'}", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10",
          f"-Wl,-rpath,{torch_root / 'lib'}", f"-Wl,-rpath,{cuda_home / 'lib64'}"])
    for obj in objects:
        obj.unlink()
    return LIBRARY


def load() -> bool:
    """Loads the built library into torch (registers torch.ops.inference_performance_lab_ref.*).
    False when it has not been built."""
    import torch

    if not LIBRARY.exists():
        return False
    torch.ops.load_library(str(LIBRARY))
    return True


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", type=Path, required=True, help="root of the reference checkout")
    args = parser.parse_args()
    print(build(args.reference))
    sys.exit(0)
