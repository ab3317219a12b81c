"""CPU oracle for the fused add+RMSNorm and SiLU-and-mul path.

TEST INFRASTRUCTURE ONLY. Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` (and ``bench.py --impl reference``) as the checker / the timed CPU path. The
product (``inference_performance_lab``) never imports it and has no CPU fallback.

Two restatements of the reference's fp32 oracle,
``src/inference_performance_lab/kernels/reference.py`` (sreeganeshji/inference-performance-lab):

* ``c_*`` - plain C (``ipl_oracle.c``), on raw bf16 bit patterns held in numpy ``uint16`` arrays;
* ``torch_*`` - the same torch fp32 operations as the reference (reference.py:18-23, :32-35),
  restated; this is the reference's own CPU path, timed by ``bench.py`` as the CPU baseline.

Both are pinned against golden vectors made by running the reference's ``reference.py`` itself
(``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``).
"""

from __future__ import annotations

import ctypes
import subprocess
from functools import cache
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIBRARY = ORACLE_DIR / "_build" / "libipl_oracle.so"

_U16P = ctypes.POINTER(ctypes.c_uint16)


def build() -> Path:
    """Compile ipl_oracle.c (make) if the shared object is missing or stale."""
    source = ORACLE_DIR / "ipl_oracle.c"
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < source.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIBRARY


@cache
def _lib() -> ctypes.CDLL:
    lib = ctypes.CDLL(str(build()))
    lib.oracle_fused_add_rms_norm_bf16.restype = ctypes.c_int
    lib.oracle_fused_add_rms_norm_bf16.argtypes = [
        _U16P, _U16P, _U16P, ctypes.c_int64, ctypes.c_int64, ctypes.c_double, _U16P, _U16P,
    ]
    lib.oracle_rms_norm_bf16.restype = ctypes.c_int
    lib.oracle_rms_norm_bf16.argtypes = [_U16P, _U16P, ctypes.c_int64, ctypes.c_int64, ctypes.c_double, _U16P]
    lib.oracle_silu_and_mul_bf16.restype = None
    lib.oracle_silu_and_mul_bf16.argtypes = [_U16P, ctypes.c_int64, ctypes.c_int64, _U16P]
    lib.oracle_fused_add_rms_norm_static_fp8_quant.restype = ctypes.c_int
    lib.oracle_fused_add_rms_norm_static_fp8_quant.argtypes = [
        _U16P, _U16P, _U16P, ctypes.c_int64, ctypes.c_int64, ctypes.c_double, ctypes.c_float,
        ctypes.POINTER(ctypes.c_uint8), _U16P,
    ]
    lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
    lib.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
    lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
    lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
    return lib


def _u16(array: np.ndarray) -> np.ndarray:
    array = np.ascontiguousarray(array)
    if array.dtype != np.uint16:
        raise TypeError("bf16 data is passed as uint16 bit patterns")
    return array


def _ptr(array: np.ndarray):
    return array.ctypes.data_as(_U16P)


def c_fused_add_rms_norm(
    x: np.ndarray, residual: np.ndarray, weight: np.ndarray, epsilon: float
) -> tuple[np.ndarray, np.ndarray]:
    """(output, residual_out) as uint16 bf16 bit patterns, shapes of ``x``."""
    x, residual, weight = _u16(x), _u16(residual), _u16(weight)
    if x.shape != residual.shape:
        raise ValueError("x and residual must have identical shapes")
    if weight.ndim != 1 or x.ndim == 0 or weight.shape[0] != x.shape[-1]:
        raise ValueError("weight must match the final tensor dimension")
    hidden = x.shape[-1]
    rows = x.size // hidden if hidden else 0
    out = np.empty_like(x)
    res = np.empty_like(x)
    if rows and hidden:
        status = _lib().oracle_fused_add_rms_norm_bf16(
            _ptr(x), _ptr(residual), _ptr(weight), rows, hidden, epsilon, _ptr(out), _ptr(res)
        )
        if status != 0:
            raise MemoryError("oracle scratch allocation failed")
    return out, res


def c_fused_add_rms_norm_static_fp8_quant(
    x: np.ndarray, residual: np.ndarray, weight: np.ndarray, scale: float, epsilon: float
) -> tuple[np.ndarray, np.ndarray]:
    """(e4m3 output as uint8, residual_out as uint16 bf16 bits)."""
    x, residual, weight = _u16(x), _u16(residual), _u16(weight)
    if x.shape != residual.shape:
        raise ValueError("x and residual must have identical shapes")
    hidden = x.shape[-1]
    rows = x.size // hidden if hidden else 0
    out = np.empty(x.shape, dtype=np.uint8)
    res = np.empty_like(x)
    if rows and hidden:
        status = _lib().oracle_fused_add_rms_norm_static_fp8_quant(
            _ptr(x), _ptr(residual), _ptr(weight), rows, hidden, epsilon, scale,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), _ptr(res),
        )
        if status != 0:
            raise MemoryError("oracle scratch allocation failed")
    return out, res


def c_f32_to_e4m3(values: np.ndarray) -> np.ndarray:
    lib = _lib()
    return np.array([lib.oracle_f32_to_e4m3(float(v)) for v in np.asarray(values, dtype=np.float32).ravel()],
                    dtype=np.uint8)


def c_rms_norm(x: np.ndarray, weight: np.ndarray, epsilon: float) -> np.ndarray:
    """Plain RMSNorm (no residual) as uint16 bf16 bit patterns."""
    x, weight = _u16(x), _u16(weight)
    if weight.ndim != 1 or x.ndim == 0 or weight.shape[0] != x.shape[-1]:
        raise ValueError("weight must match the final tensor dimension")
    hidden = x.shape[-1]
    rows = x.size // hidden if hidden else 0
    out = np.empty_like(x)
    if rows and hidden:
        _lib().oracle_rms_norm_bf16(_ptr(x), _ptr(weight), rows, hidden, epsilon, _ptr(out))
    return out


def c_silu_and_mul(x: np.ndarray) -> np.ndarray:
    x = _u16(x)
    if x.ndim == 0 or x.shape[-1] % 2 != 0:
        raise ValueError("the final tensor dimension must be even")
    inter = x.shape[-1] // 2
    out = np.empty(x.shape[:-1] + (inter,), dtype=np.uint16)
    rows = out.size // inter if inter else 0
    if rows and inter:
        _lib().oracle_silu_and_mul_bf16(_ptr(x), rows, inter, _ptr(out))
    return out


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN -> 0x7FC0), vectorised in numpy."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounded = ((u + (np.uint32(0x7FFF) + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    rounded[nan] = 0x7FC0
    return rounded


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------------------------
# torch restatement (the reference's CPU path)


def torch_fused_add_rms_norm(x, residual, weight, epsilon: float):
    """reference.py:7-23 restated: returns (output, residual_out) in x's dtype."""
    import torch

    if x.shape != residual.shape:
        raise ValueError("x and residual must have identical shapes")
    if weight.ndim != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError("weight must match the final tensor dimension")
    summed = x.float() + residual.float()
    inverse_rms = torch.rsqrt(summed.square().mean(dim=-1, keepdim=True) + epsilon)
    return (summed * inverse_rms * weight.float()).to(x.dtype), summed.to(residual.dtype)


def torch_rms_norm(x, weight, epsilon: float):
    """Plain RMSNorm in the reference oracle's fp32 arithmetic (reference.py:19-23, no residual)."""
    import torch

    if weight.ndim != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError("weight must match the final tensor dimension")
    v = x.float()
    inverse_rms = torch.rsqrt(v.square().mean(dim=-1, keepdim=True) + epsilon)
    return (v * inverse_rms * weight.float()).to(x.dtype)


def torch_fused_add_rms_norm_static_fp8_quant(x, residual, weight, scale: float, epsilon: float):
    """reference.py:18-21 in fp32, then e4m3 of product / scale saturated to +-448 (torch's own
    float8_e4m3fn conversion, which rounds to nearest even)."""
    import torch

    summed = x.float() + residual.float()
    inverse_rms = torch.rsqrt(summed.square().mean(dim=-1, keepdim=True) + epsilon)
    normed = summed * inverse_rms * weight.float()
    quantised = (normed * (1.0 / torch.tensor(scale, dtype=torch.float32))).clamp(-448.0, 448.0)
    return quantised.to(torch.float8_e4m3fn), summed.to(residual.dtype)


def torch_silu_and_mul(x):
    """reference.py:26-35 restated."""
    import torch.nn.functional as F

    if x.ndim == 0 or x.shape[-1] % 2 != 0:
        raise ValueError("the final tensor dimension must be even")
    gate, up = x.float().chunk(2, dim=-1)
    return (F.silu(gate) * up).to(x.dtype)


def tensor_bits(tensor) -> np.ndarray:
    """bf16 torch tensor (any device) -> uint16 numpy bit patterns."""
    import torch

    return tensor.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def bits_tensor(bits: np.ndarray, device="cpu"):
    """uint16 numpy bit patterns -> bf16 torch tensor on ``device``."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)
