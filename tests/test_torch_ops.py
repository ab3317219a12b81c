"""The stable-ABI op library without a GPU: it loads, registers the reference's exact schemas, and
has no CPU kernel (no silent fallback): CPU tensors are rejected by the dispatcher."""

from __future__ import annotations

import pytest
import torch

from inference_performance_lab.kernels import extension

# csrc/torch_ops.cpp:13-15 of the reference.
REFERENCE_SCHEMAS = {
    "fused_add_rms_norm": "inference_performance_lab::fused_add_rms_norm(Tensor(a!) x, "
    "Tensor(b!) residual, Tensor weight, float epsilon) -> ()",
    "silu_and_mul": "inference_performance_lab::silu_and_mul(Tensor(a!) output, Tensor input) -> ()",
    "silu_and_mul_packed": "inference_performance_lab::silu_and_mul_packed(Tensor(a!) output, "
    "Tensor input) -> ()",
}


def test_schemas_match_the_reference() -> None:
    extension.load_extension()
    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(torch.ops.inference_performance_lab, name).default._schema) == schema


def test_no_cpu_fallback() -> None:
    extension.load_extension()
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError, match="CPU"):
        torch.ops.inference_performance_lab.fused_add_rms_norm(
            x, x.clone(), torch.ones(8, dtype=torch.bfloat16), 1e-6
        )
    with pytest.raises(NotImplementedError, match="CPU"):
        torch.ops.inference_performance_lab.silu_and_mul(x[:, :4].contiguous(), x)


def test_python_wrappers_reject_odd_width() -> None:
    with pytest.raises(ValueError, match="final tensor dimension must be even"):
        extension.silu_and_mul(torch.zeros(2, 7, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="final tensor dimension must be even"):
        extension.silu_and_mul_packed(torch.zeros(2, 7, dtype=torch.bfloat16))


def test_vllm_provider_registers_and_filters_arguments() -> None:
    pytest.importorskip("vllm.ir")
    from vllm import ir

    from inference_performance_lab.kernels import vllm_plugin

    vllm_plugin.register()
    vllm_plugin.register()  # idempotent
    assert vllm_plugin.PROVIDER in ir.ops.fused_add_rms_norm.impls

    x = torch.zeros(4, 3584, dtype=torch.bfloat16)
    w = torch.ones(3584, dtype=torch.bfloat16)
    # CPU tensors are never routed to the CUDA provider.
    assert not vllm_plugin.supports_fused_add_rms_norm(x, x.clone(), w, 1e-6)


def test_shim_shares_torchs_libstdcxx() -> None:
    """The op library throws C++ exceptions into torch's dispatcher, so it must use the shared
    libstdc++ that torch uses and export no copy of its own (a statically linked libstdc++
    crashed while formatting the first error message)."""
    import shutil
    import subprocess

    extension.ensure_built()
    if shutil.which("nm") is None:
        pytest.skip("binutils nm unavailable")
    exported = subprocess.run(
        ["nm", "-D", "--defined-only", str(extension.TORCH_OPS_LIBRARY)],
        capture_output=True, text=True, check=True,
    ).stdout.split()
    # Inline template instantiations (weak symbols) are normal; the library's own copy of the
    # stream / locale machinery is not.
    bundled = [s for s in exported if any(k in s for k in ("codecvt", "ios_base", "locale", "_ZNSo"))]
    assert not bundled, bundled[:5]
    assert len(exported) < 100
    needed = subprocess.run(
        ["readelf", "-d", str(extension.TORCH_OPS_LIBRARY)], capture_output=True, text=True, check=True
    ).stdout
    assert "libstdc++.so.6" in needed


def test_vllm_rms_norm_provider_registers() -> None:
    pytest.importorskip("vllm.ir")
    from vllm import ir

    from inference_performance_lab.kernels import vllm_plugin

    vllm_plugin.register()
    assert vllm_plugin.PROVIDER in ir.ops.rms_norm.impls
    x = torch.zeros(4, 3584, dtype=torch.bfloat16)
    assert not vllm_plugin.supports_rms_norm(x, torch.ones(3584, dtype=torch.bfloat16), 1e-6)
