"""ctypes binding of the C ABI (``include/ipl_b200.h``, ``_native/libipl_b200.so``).

This is the binding a non-torch caller uses: raw device pointers, sizes and a ``cudaStream_t``.
Each wrapper raises ``RuntimeError`` with the library's message when the call fails, the same
error surface as the torch ops (which raise through STD_TORCH_CHECK).
"""

from __future__ import annotations

import ctypes
from functools import cache

from inference_performance_lab.kernels.extension import C_ABI_LIBRARY, ensure_built

IPL_SUCCESS = 0
IPL_ERROR_INVALID_VALUE = 1
IPL_ERROR_MISALIGNED = 2
IPL_ERROR_TOO_LARGE = 3
IPL_ERROR_CUDA = 4

# name -> (restype, argtypes): every symbol include/ipl_b200.h declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ipl_fused_add_rms_norm_bf16": (
        ctypes.c_int,
        [
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_int64,
            ctypes.c_int64,
            ctypes.c_double,
            ctypes.c_void_p,
        ],
    ),
    "ipl_rms_norm_bf16": (
        ctypes.c_int,
        [
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_int64,
            ctypes.c_int64,
            ctypes.c_double,
            ctypes.c_void_p,
        ],
    ),
    "ipl_fused_add_rms_norm_static_fp8_quant": (
        ctypes.c_int,
        [
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_void_p,
            ctypes.c_int64,
            ctypes.c_int64,
            ctypes.c_double,
            ctypes.c_void_p,
        ],
    ),
    "ipl_silu_and_mul_bf16": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p],
    ),
    "ipl_silu_and_mul_packed_bf16": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p],
    ),
    "ipl_last_error": (ctypes.c_char_p, []),
    "ipl_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ipl_abi_version": (ctypes.c_int, []),
    "ipl_device_fault_flags": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
    "ipl_clear_device_fault_flags": (ctypes.c_int, [ctypes.c_int]),
    "ipl_fused_add_rms_norm_plan": (
        ctypes.c_char_p,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64],
    ),
    "ipl_rms_norm_plan": (
        ctypes.c_char_p,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64],
    ),
    "ipl_fused_add_rms_norm_static_fp8_quant_plan": (
        ctypes.c_char_p,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64],
    ),
    "ipl_silu_and_mul_plan": (
        ctypes.c_char_p,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64],
    ),
}


class IplError(RuntimeError):
    """A nonzero ipl_status; ``status`` holds the code."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(message)
        self.status = status


@cache
def library() -> ctypes.CDLL:
    """Load libipl_b200.so once and attach the prototypes."""
    ensure_built()
    lib = ctypes.CDLL(str(C_ABI_LIBRARY))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def _check(status: int) -> None:
    if status != IPL_SUCCESS:
        raise IplError(status, library().ipl_last_error().decode())


def fused_add_rms_norm(
    x_ptr: int,
    residual_ptr: int,
    weight_ptr: int,
    rows: int,
    hidden_size: int,
    epsilon: float,
    stream: int = 0,
) -> None:
    _check(
        library().ipl_fused_add_rms_norm_bf16(
            x_ptr, residual_ptr, weight_ptr, rows, hidden_size, epsilon, stream
        )
    )


def rms_norm(
    output_ptr: int,
    input_ptr: int,
    weight_ptr: int,
    rows: int,
    hidden_size: int,
    epsilon: float,
    stream: int = 0,
) -> None:
    _check(
        library().ipl_rms_norm_bf16(output_ptr, input_ptr, weight_ptr, rows, hidden_size, epsilon, stream)
    )


def fused_add_rms_norm_static_fp8_quant(
    output_ptr: int,
    input_ptr: int,
    residual_ptr: int,
    weight_ptr: int,
    scale_ptr: int,
    rows: int,
    hidden_size: int,
    epsilon: float,
    stream: int = 0,
) -> None:
    _check(
        library().ipl_fused_add_rms_norm_static_fp8_quant(
            output_ptr, input_ptr, residual_ptr, weight_ptr, scale_ptr, rows, hidden_size, epsilon, stream
        )
    )


def silu_and_mul(
    output_ptr: int, input_ptr: int, rows: int, intermediate_size: int, stream: int = 0
) -> None:
    _check(library().ipl_silu_and_mul_bf16(output_ptr, input_ptr, rows, intermediate_size, stream))


def silu_and_mul_packed(
    output_ptr: int, input_ptr: int, rows: int, intermediate_size: int, stream: int = 0
) -> None:
    _check(
        library().ipl_silu_and_mul_packed_bf16(
            output_ptr, input_ptr, rows, intermediate_size, stream
        )
    )


def device_fault_flags(device: int) -> int:
    flags = ctypes.c_uint32(0)
    _check(library().ipl_device_fault_flags(device, ctypes.byref(flags)))
    return flags.value


def clear_device_fault_flags(device: int) -> None:
    _check(library().ipl_clear_device_fault_flags(device))


def fused_add_rms_norm_plan(
    x_ptr: int, residual_ptr: int, weight_ptr: int, rows: int, hidden_size: int
) -> str:
    return library().ipl_fused_add_rms_norm_plan(
        x_ptr, residual_ptr, weight_ptr, rows, hidden_size
    ).decode()


def rms_norm_plan(output_ptr: int, input_ptr: int, weight_ptr: int, rows: int, hidden_size: int) -> str:
    return library().ipl_rms_norm_plan(output_ptr, input_ptr, weight_ptr, rows, hidden_size).decode()


def fused_add_rms_norm_static_fp8_quant_plan(
    output_ptr: int, input_ptr: int, residual_ptr: int, weight_ptr: int, rows: int, hidden_size: int
) -> str:
    return library().ipl_fused_add_rms_norm_static_fp8_quant_plan(
        output_ptr, input_ptr, residual_ptr, weight_ptr, rows, hidden_size
    ).decode()


def silu_and_mul_plan(output_ptr: int, input_ptr: int, rows: int, intermediate_size: int) -> str:
    return library().ipl_silu_and_mul_plan(output_ptr, input_ptr, rows, intermediate_size).decode()


# Tensor-level conveniences (torch tensors on the current CUDA device, current stream).


def _stream_handle() -> int:
    import torch

    return torch.cuda.current_stream().cuda_stream


def fused_add_rms_norm_tensors(x, residual, weight, epsilon: float) -> None:
    hidden = x.shape[-1]
    rows = x.numel() // hidden if hidden else 0
    fused_add_rms_norm(
        x.data_ptr(), residual.data_ptr(), weight.data_ptr(), rows, hidden, epsilon, _stream_handle()
    )


def rms_norm_tensors(output, input_, weight, epsilon: float) -> None:
    hidden = input_.shape[-1]
    rows = input_.numel() // hidden if hidden else 0
    rms_norm(
        output.data_ptr(), input_.data_ptr(), weight.data_ptr(), rows, hidden, epsilon, _stream_handle()
    )


def silu_and_mul_tensors(output, input_, packed: bool = False) -> None:
    inter = input_.shape[-1] // 2
    rows = output.numel() // inter if inter else 0
    fn = silu_and_mul_packed if packed else silu_and_mul
    fn(output.data_ptr(), input_.data_ptr(), rows, inter, _stream_handle())
