"""vLLM general plugin: the ``inference_lab`` provider of ``vllm.ir.ops.fused_add_rms_norm`` and
``vllm.ir.ops.rms_norm``.

Same entry point, provider name and registration as the reference
(src/inference_performance_lab/kernels/vllm_plugin.py:11,43-69; entry point
``vllm.general_plugins: inference_performance_lab = ...vllm_plugin:register``, pyproject.toml:39-40).
The argument filter is wider: the reference accepted only 2-D inputs with hidden size 3584
(:15-40, the one shape its specialised kernel handled); the B200 kernels take any hidden size and
alignment, so any contiguous bf16 input on one CUDA device with a weight and no
``variance_size`` is accepted. The plain ``rms_norm`` provider (not in the reference; the norm
before the first and after the last decoder layer) follows the same rules.
"""

from __future__ import annotations

import torch
from torch import Tensor

from inference_performance_lab.kernels.extension import (
    fused_add_rms_norm as custom_fused_add_rms_norm,
)
from inference_performance_lab.kernels.extension import load_extension
from inference_performance_lab.kernels.extension import rms_norm as custom_rms_norm

PROVIDER = "inference_lab"


def _share_memory(a: Tensor, b: Tensor) -> bool:
    """Whether a and b start at the same address. vLLM's Inductor lowering pass chooses the
    provider on fake tensors, which carry no data (their data_ptr() reads 0 for every tensor):
    there they are two distinct arguments of the IR op, so they do not alias."""
    from torch._subclasses.fake_tensor import is_fake

    if is_fake(a) or is_fake(b):
        return False
    return a.data_ptr() == b.data_ptr()


def supports_fused_add_rms_norm(
    x: Tensor,
    x_residual: Tensor,
    weight: Tensor | None,
    epsilon: float,
    variance_size: int | None = None,
) -> bool:
    del epsilon

    return (
        variance_size is None
        and weight is not None
        and x.device.type == "cuda"
        and x_residual.device == x.device
        and weight.device == x.device
        and x.dtype == torch.bfloat16
        and x_residual.dtype == x.dtype
        and weight.dtype == x.dtype
        and x.ndim >= 1
        and x.shape == x_residual.shape
        and x.shape[-1] > 0
        and weight.shape == (x.shape[-1],)
        and x.is_contiguous()
        and x_residual.is_contiguous()
        and weight.is_contiguous()
        and not _share_memory(x, x_residual)
    )


def supports_rms_norm(
    x: Tensor, weight: Tensor | None, epsilon: float, variance_size: int | None = None
) -> bool:
    del epsilon

    return (
        variance_size is None
        and weight is not None
        and x.device.type == "cuda"
        and weight.device == x.device
        and x.dtype == torch.bfloat16
        and weight.dtype == x.dtype
        and x.ndim >= 1
        and x.shape[-1] > 0
        and weight.shape == (x.shape[-1],)
        and x.is_contiguous()
        and weight.is_contiguous()
    )


def register() -> None:
    from vllm import ir

    load_extension()
    _register_rms_norm(ir.ops.rms_norm)

    op = ir.ops.fused_add_rms_norm
    if PROVIDER in op.impls:
        return

    @op.register_impl(
        PROVIDER,
        supported=torch.cuda.is_available(),
        supports_args=supports_fused_add_rms_norm,
        inplace=True,
    )
    def inference_lab_fused_add_rms_norm(
        x: Tensor,
        x_residual: Tensor,
        weight: Tensor | None,
        epsilon: float,
        variance_size: int | None = None,
    ) -> tuple[Tensor, Tensor]:
        assert weight is not None
        assert variance_size is None

        custom_fused_add_rms_norm(x, x_residual, weight, epsilon)
        return x, x_residual


def _register_rms_norm(op) -> None:
    if PROVIDER in op.impls:
        return

    @op.register_impl(PROVIDER, supported=torch.cuda.is_available(), supports_args=supports_rms_norm)
    def inference_lab_rms_norm(
        x: Tensor, weight: Tensor | None, epsilon: float, variance_size: int | None = None
    ) -> Tensor:
        assert weight is not None
        assert variance_size is None

        return custom_rms_norm(x, weight, epsilon)


def supports_silu_and_mul(x: Tensor) -> bool:
    return (
        x.device.type == "cuda"
        and x.dtype == torch.bfloat16
        and x.ndim >= 1
        and x.shape[-1] % 2 == 0
        and x.is_contiguous()
    )


def register_silu_and_mul() -> None:
    """Replace vLLM's SiluAndMul custom op with one that runs these kernels.

    vLLM 0.22 has no IR op for SiLU-and-mul, so the replacement goes through its out-of-tree
    custom-op registry: every ``SiluAndMul`` a model builds afterwards is this subclass, whose
    CUDA path calls ``torch.ops.inference_performance_lab.silu_and_mul`` for contiguous bf16
    inputs and vLLM's own kernel otherwise. It is a separate entry point (not called by
    :func:`register`) because, unlike the IR providers, it takes effect without a priority list.
    """
    from vllm.model_executor.custom_op import op_registry_oot
    from vllm.model_executor.layers.activation import SiluAndMul

    if "SiluAndMul" in op_registry_oot:
        return

    load_extension()

    @SiluAndMul.register_oot(name="SiluAndMul")
    class InferenceLabSiluAndMul(SiluAndMul):
        def forward_cuda(self, x: Tensor) -> Tensor:
            if not supports_silu_and_mul(x):
                return super().forward_cuda(x)
            output = torch.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=x.dtype, device=x.device)
            torch.ops.inference_performance_lab.silu_and_mul(output, x)
            return output

    # The registry keys the replacement by the class it replaces ("SiluAndMul"), and registering
    # renames it to that key; vLLM's switch for the op under compilation is its op name,
    # `custom_ops: ["+silu_and_mul"]`, so give the replacement that name back: the same switch that
    # turns vLLM's own SiLU kernel on (it is off by default under torch.compile, where Inductor
    # fuses the native SiLU) turns this one on.
    InferenceLabSiluAndMul.name = SiluAndMul.name
