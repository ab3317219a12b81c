"""Op loader and Python wrappers.

Mirrors ``src/inference_performance_lab/kernels/extension.py`` of the reference (load_extension at
:12-35, wrappers at :38-71): same function names, arguments, in-place behaviour and errors. The
difference is the loader: instead of JIT-compiling with ``torch.utils.cpp_extension.load`` into a
cache directory, it loads the in-tree library built by ``build.py`` (building it first if it is
missing or stale and nvcc is present). There is no fallback: if the native library cannot be
loaded, every op raises.
"""

from __future__ import annotations

import importlib.util
from functools import cache
from pathlib import Path

import torch

PACKAGE_DIR = Path(__file__).resolve().parents[1]
NATIVE_DIR = PACKAGE_DIR / "_native"
TORCH_OPS_LIBRARY = NATIVE_DIR / "inference_performance_lab_cuda.so"
C_ABI_LIBRARY = NATIVE_DIR / "libipl_b200.so"


def _build_module():
    spec = importlib.util.spec_from_file_location(
        "_ipl_build", PACKAGE_DIR.parent / "build.py"
    )
    module = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    spec.loader.exec_module(module)
    return module


def ensure_built(*, verbose: bool = False) -> None:
    """Build the native libraries in-tree if they are missing or older than their sources."""
    try:
        builder = _build_module()
    except FileNotFoundError:
        builder = None
    if builder is not None:
        import shutil

        if shutil.which("nvcc") or Path("/usr/local/cuda/bin/nvcc").exists():
            builder.build(verbose=verbose)
    if not TORCH_OPS_LIBRARY.exists() or not C_ABI_LIBRARY.exists():
        raise RuntimeError(
            f"native library missing: {TORCH_OPS_LIBRARY} (run inference-performance-lab_b200/build.py)"
        )


@cache
def load_extension(*, verbose: bool = False) -> None:
    """Load the op library and register ``torch.ops.inference_performance_lab.*``."""
    ensure_built(verbose=verbose)
    torch.ops.load_library(str(TORCH_OPS_LIBRARY))


def fused_add_rms_norm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, epsilon: float
) -> None:
    """In place: ``residual := x + residual``; ``x := rmsnorm(x + residual) * weight``."""
    load_extension()

    torch.ops.inference_performance_lab.fused_add_rms_norm(x, residual, weight, epsilon)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, epsilon: float) -> torch.Tensor:
    """``rmsnorm(x) * weight`` into a new tensor (no residual; not in the reference library)."""
    load_extension()

    output = torch.empty_like(x)
    torch.ops.inference_performance_lab.rms_norm(output, x, weight, epsilon)

    return output


def fused_add_rms_norm_static_fp8_quant(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor, epsilon: float
) -> torch.Tensor:
    """``residual := x + residual`` in place; returns ``e4m3(rmsnorm(x + residual) * weight / scale)``
    (x is not modified; not in the reference library)."""
    load_extension()

    output = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    torch.ops.inference_performance_lab.fused_add_rms_norm_static_fp8_quant(
        output, x, residual, weight, scale, epsilon
    )

    return output


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """``silu(x[..., :I]) * x[..., I:]`` into a new ``[..., I]`` tensor (any width/alignment)."""
    load_extension()

    if x.ndim == 0 or x.shape[-1] % 2 != 0:
        raise ValueError("the final tensor dimension must be even")

    output_shape = x.shape[:-1] + (x.shape[-1] // 2,)
    output = torch.empty(output_shape, dtype=x.dtype, device=x.device)

    torch.ops.inference_performance_lab.silu_and_mul(output, x)

    return output


def silu_and_mul_packed(x: torch.Tensor) -> torch.Tensor:
    """Same result; keeps the reference's packed contract (I % 8 == 0, 16-byte aligned)."""
    load_extension()

    if x.ndim == 0 or x.shape[-1] % 2 != 0:
        raise ValueError("the final tensor dimension must be even")

    output_shape = x.shape[:-1] + (x.shape[-1] // 2,)
    output = torch.empty(output_shape, dtype=x.dtype, device=x.device)

    torch.ops.inference_performance_lab.silu_and_mul_packed(output, x)

    return output
