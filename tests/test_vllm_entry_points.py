"""The installable package and its vLLM plugin entry points.

``inference-performance-lab_b200/pyproject.toml`` declares the reference's plugin entry point
(``vllm.general_plugins: inference_performance_lab``, reference pyproject.toml:39-40) and a second
one for SiLU-and-mul. The test installs the package (with its built native libraries) into a
temporary directory, offline, and in a fresh process with ``VLLM_PLUGINS`` set lets vLLM's own
plugin loader find and run both entry points, as ``vllm serve`` does in every engine and worker
process: the ``inference_lab`` providers of vLLM's IR ops and the out-of-tree ``SiluAndMul`` must be
registered, loaded from the installed copy.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.vllm

PACKAGE_DIR = Path(__file__).resolve().parents[1] / "inference-performance-lab_b200"

PROBE = r"""
import json
from vllm.plugins import load_general_plugins
load_general_plugins()
from vllm import ir
from vllm.model_executor.custom_op import op_registry_oot
import inference_performance_lab, torch
print(json.dumps({
    "package": inference_performance_lab.__file__,
    "fused_add_rms_norm": sorted(ir.ops.fused_add_rms_norm.impls),
    "rms_norm": sorted(ir.ops.rms_norm.impls),
    "oot": sorted(op_registry_oot),
    "oot_op_name": op_registry_oot["SiluAndMul"].name,
    "schema": str(torch.ops.inference_performance_lab.fused_add_rms_norm.default._schema),
}))
"""


def test_vllm_loads_the_providers_through_the_entry_points(tmp_path: Path) -> None:
    pytest.importorskip("vllm.plugins")
    from inference_performance_lab.kernels.extension import ensure_built

    ensure_built()
    source = tmp_path / "src"
    source.mkdir()
    shutil.copy(PACKAGE_DIR / "pyproject.toml", source / "pyproject.toml")
    shutil.copytree(PACKAGE_DIR / "inference_performance_lab", source / "inference_performance_lab",
                    ignore=shutil.ignore_patterns("__pycache__", "test", "*.stamp", "*.txt", ".build.lock"))
    site = tmp_path / "site"
    install = subprocess.run(
        [sys.executable, "-m", "pip", "install", "--no-index", "--no-deps", "--no-build-isolation", "--quiet",
         "--target", str(site), str(source)],
        capture_output=True, text=True, timeout=300,
    )
    assert install.returncode == 0, install.stderr[-2000:]
    entry_points = next(site.glob("*.dist-info")).joinpath("entry_points.txt").read_text()
    assert "[vllm.general_plugins]" in entry_points
    assert "inference_performance_lab = inference_performance_lab.kernels.vllm_plugin:register" in entry_points
    assert (site / "inference_performance_lab" / "_native" / "libipl_b200.so").exists()

    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    env.update(PYTHONPATH=str(site), VLLM_PLUGINS="inference_performance_lab,inference_performance_lab_silu")
    probe = subprocess.run([sys.executable, "-c", PROBE], cwd=tmp_path, env=env, capture_output=True, text=True,
                           timeout=300)
    assert probe.returncode == 0, probe.stderr[-3000:]
    found = json.loads(probe.stdout.strip().splitlines()[-1])
    assert Path(found["package"]).is_relative_to(site)
    assert "inference_lab" in found["fused_add_rms_norm"] and "inference_lab" in found["rms_norm"]
    assert "SiluAndMul" in found["oot"]
    assert found["oot_op_name"] == "silu_and_mul"  # vLLM's custom-op switch for SiLU-and-mul applies
    assert found["schema"].startswith("inference_performance_lab::fused_add_rms_norm(Tensor(a!) x")


def test_provider_accepts_the_fake_tensors_of_inductor_lowering() -> None:
    """Under vLLM's default compilation the IR lowering pass picks the provider by calling
    supports_args on fake tensors (vllm/compilation/passes/ir/lowering_pass.py: dispatch(*fake_args))
    and then traces the provider's function on them. Fake tensors carry no data pointer, so the
    aliasing check must not reject them, and the op calls must trace; on real tensors the check
    still rejects x and residual sharing memory."""
    pytest.importorskip("vllm.ir")
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    from inference_performance_lab.kernels import extension, vllm_plugin

    extension.load_extension()
    with FakeTensorMode(allow_non_fake_inputs=True):
        x = torch.empty(16, 3584, dtype=torch.bfloat16, device="cuda")
        r = torch.empty(16, 3584, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(3584, dtype=torch.bfloat16, device="cuda")
        assert vllm_plugin.supports_fused_add_rms_norm(x, r, w, 1e-6)
        assert vllm_plugin.supports_rms_norm(x, w, 1e-6)
        torch.ops.inference_performance_lab.fused_add_rms_norm(x, r, w, 1e-6)
        torch.ops.inference_performance_lab.rms_norm(torch.empty_like(x), x, w, 1e-6)
    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    assert vllm_plugin._share_memory(a, a) and not vllm_plugin._share_memory(a, a.clone())
