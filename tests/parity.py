"""Shared helpers of the GPU parity tests: guarded allocations and comparisons with the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle

# Output tolerance of the reference's tests (tests/test_fused_add_rms_norm.py:33,
# tests/test_silu_and_mul.py:29): rtol = atol = 1e-2. It is tighter than the 1.6e-2 rtol of
# the project target, so meeting it meets both.
RTOL = 1e-2
ATOL = 1e-2

GUARD = 4096  # elements of canary on each side of a guarded tensor
CANARY = 0x7BAD  # a finite bf16 bit pattern never produced by the tests' data paths at that spot


def require_cuda() -> None:
    """Fail (not skip) without a GPU, and register the ops for tests that call torch.ops directly."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from inference_performance_lab.kernels.extension import load_extension

    load_extension()


class Guarded:
    """A contiguous bf16 tensor at a chosen element offset inside a canary-filled buffer."""

    def __init__(self, shape, offset: int, device: str = "cuda") -> None:
        numel = int(np.prod(shape)) if len(shape) else 1
        self.offset = offset
        self.numel = numel
        self.storage = torch.empty(GUARD + offset + numel + GUARD, dtype=torch.int16, device=device)
        self.storage.fill_(CANARY)
        view = self.storage[GUARD + offset: GUARD + offset + numel]
        self.tensor = view.view(torch.bfloat16).view(shape)

    def load(self, bits: np.ndarray) -> torch.Tensor:
        self.tensor.view(torch.int16).view(-1).copy_(
            torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).reshape(-1))
        )
        return self.tensor

    def assert_guards_intact(self) -> None:
        head = self.storage[: GUARD + self.offset]
        tail = self.storage[GUARD + self.offset + self.numel:]
        assert bool((head == CANARY).all()), "write before the tensor"
        assert bool((tail == CANARY).all()), "write past the tensor"


def bf16_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two arrays of bf16 bit patterns (monotone integer map)."""
    def ordered(bits: np.ndarray) -> np.ndarray:
        i = bits.astype(np.int32)
        return np.where(i & 0x8000, 0x8000 - i, i)

    return np.abs(ordered(a) - ordered(b))


def assert_bits_equal(actual: torch.Tensor, expected_bits: np.ndarray, what: str) -> None:
    got = oracle.tensor_bits(actual)
    if not np.array_equal(got, expected_bits):
        bad = np.flatnonzero(got.reshape(-1) != expected_bits.reshape(-1))
        raise AssertionError(
            f"{what}: {bad.size} of {got.size} elements differ (first at {bad[:5].tolist()})"
        )


def assert_close_to_oracle(actual: torch.Tensor, expected_bits: np.ndarray, what: str,
                           max_ulp: int = 1) -> None:
    """Within the reference tests' tolerance, and at most ``max_ulp`` bf16 ulps from the oracle."""
    got = oracle.tensor_bits(actual)
    expected = oracle.bf16_bits_to_f32(expected_bits)
    torch.testing.assert_close(
        torch.from_numpy(oracle.bf16_bits_to_f32(got)), torch.from_numpy(expected),
        rtol=RTOL, atol=ATOL, msg=lambda m: f"{what}: {m}",
    )
    distance = bf16_ulp_distance(got.reshape(-1), expected_bits.reshape(-1))
    assert int(distance.max(initial=0)) <= max_ulp, f"{what}: {int(distance.max())} ulps from the oracle"
