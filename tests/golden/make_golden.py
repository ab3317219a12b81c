"""Generate the golden vectors in this directory by running the reference's own oracle.

Imports ``src/inference_performance_lab/kernels/reference.py`` of sreeganeshji/inference-performance-lab
(pure PyTorch, fp32 arithmetic) from a checkout of the reference, evaluates it on CPU on seeded
inputs and stores inputs and outputs as raw bf16 bit patterns (uint16) in ``golden.npz``.
The checkout is only needed to regenerate; the tests read the committed ``golden.npz``.

    python tests/golden/make_golden.py --reference /path/to/inference-performance-lab

Cases follow the reference's input recipes: x = randn, residual = randn_like(x),
weight = randn(H) * 0.1 + 1.0 in bf16 (tests/test_fused_add_rms_norm.py:20-24), SiLU input
randn(T, 2I) (tests/test_silu_and_mul.py:19-21), seed 0, drawn on CPU. ``rms_config0`` is the
reference's CPU configuration ([8, 3584], eps 1e-6) and ``silu_width18944`` a two-row slice of the
SiLU configuration's shape with its N(0, 2) inputs.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    path = root / "src" / "inference_performance_lab" / "kernels" / "reference.py"
    spec = importlib.util.spec_from_file_location("reference_oracle", path)
    module = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    spec.loader.exec_module(module)
    return module


def bits(tensor: torch.Tensor) -> np.ndarray:
    return tensor.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def rms_inputs(rows: int, hidden: int, seed: int, scale: float = 1.0):
    torch.manual_seed(seed)
    x = (torch.randn(rows, hidden) * scale).to(torch.bfloat16)
    residual = (torch.randn(rows, hidden) * scale).to(torch.bfloat16)
    weight = (torch.randn(hidden).to(torch.bfloat16) * 0.1 + 1.0).to(torch.bfloat16)
    return x, residual, weight


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True, help="root of the reference checkout")
    args = parser.parse_args()
    ref = load_reference(args.reference)

    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    rms_cases = [
        # name, rows, hidden, eps, seed, scale
        ("rms_config0", 8, 3584, 1e-6, 0, 1.0),
        ("rms_h8192", 4, 8192, 1e-5, 0, 1.0),
        ("rms_odd_width", 5, 1001, 1e-6, 1, 1.0),
        ("rms_tiny", 3, 7, 1e-6, 2, 1.0),
        ("rms_one_element", 2, 1, 1e-6, 3, 1.0),
        ("rms_large_magnitude", 2, 3584, 1e-6, 4, 300.0),
        ("rms_small_magnitude", 2, 3584, 1e-6, 5, 1e-4),
    ]
    for name, rows, hidden, eps, seed, scale in rms_cases:
        x, residual, weight = rms_inputs(rows, hidden, seed, scale)
        # reference.py takes its inputs in the recipe's layout; it does not mutate them.
        if name == "rms_config0":
            # The exact recipe of the reference's test (randn in bf16 directly).
            torch.manual_seed(0)
            x = torch.randn(rows, hidden, dtype=torch.bfloat16)
            residual = torch.randn_like(x)
            weight = torch.randn(hidden, dtype=torch.bfloat16) * 0.1 + 1.0
        out, res = ref.fused_add_rms_norm_reference(x, residual, weight, eps)
        arrays[f"{name}.x"] = bits(x)
        arrays[f"{name}.residual"] = bits(residual)
        arrays[f"{name}.weight"] = bits(weight)
        arrays[f"{name}.out"] = bits(out)
        arrays[f"{name}.residual_out"] = bits(res)
        meta[name] = {"op": "fused_add_rms_norm", "rows": rows, "hidden": hidden, "epsilon": eps}

    # Plain RMSNorm: the reference oracle's arithmetic with a zero residual (x + 0 is x for every
    # nonzero x; the inputs hold no zeros, so the sign of zero never matters).
    plain_cases = [
        ("rms_plain_3584", 8, 3584, 1e-6, 10),
        ("rms_plain_odd_width", 5, 1001, 1e-6, 11),
        ("rms_plain_8192", 2, 8192, 1e-5, 12),
    ]
    for name, rows, hidden, eps, seed in plain_cases:
        x, _, weight = rms_inputs(rows, hidden, seed)
        assert bool((x != 0).all())
        out, _ = ref.fused_add_rms_norm_reference(x, torch.zeros_like(x), weight, eps)
        arrays[f"{name}.x"] = bits(x)
        arrays[f"{name}.weight"] = bits(weight)
        arrays[f"{name}.out"] = bits(out)
        meta[name] = {"op": "rms_norm", "rows": rows, "hidden": hidden, "epsilon": eps}

    silu_cases = [
        # name, rows, intermediate, seed, std
        ("silu_width18944", 2, 18944, 0, 2.0),
        ("silu_reference_recipe", 4, 18944, 0, 1.0),
        ("silu_odd_width", 3, 1001, 1, 1.0),
        ("silu_tiny", 2, 3, 2, 1.0),
    ]
    for name, rows, inter, seed, std in silu_cases:
        torch.manual_seed(seed)
        if std == 1.0:
            x = torch.randn((rows, 2 * inter), dtype=torch.bfloat16)
        else:
            x = (torch.randn(rows, 2 * inter) * std).to(torch.bfloat16)
        out = ref.silu_and_mul_reference(x)
        arrays[f"{name}.input"] = bits(x)
        arrays[f"{name}.out"] = bits(out)
        meta[name] = {"op": "silu_and_mul", "rows": rows, "intermediate": inter}

    # Extreme gate values: saturation on both sides, signed zeros, infinities.
    gate = torch.tensor(
        [0.0, -0.0, 1.0, -1.0, 20.0, -20.0, 88.0, -88.0, 89.0, -89.0, 100.0, -100.0,
         1e4, -1e4, 3e38, -3e38, float("inf"), 1e-30, -1e-30, 0.5, -0.5, 5.0, -5.0, 10.0],
        dtype=torch.float32,
    ).to(torch.bfloat16)
    up = torch.linspace(-3.0, 3.0, gate.numel()).to(torch.bfloat16)
    x = torch.cat([gate, up]).reshape(1, -1)
    out = ref.silu_and_mul_reference(x)
    arrays["silu_extremes.input"] = bits(x)
    arrays["silu_extremes.out"] = bits(out)
    meta["silu_extremes"] = {"op": "silu_and_mul", "rows": 1, "intermediate": gate.numel()}

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(
        json.dumps(
            {"torch": torch.__version__, "generator": "tests/golden/make_golden.py", "cases": meta},
            indent=1,
        )
        + "\n"
    )
    print(f"wrote {len(meta)} cases")


if __name__ == "__main__":
    main()
