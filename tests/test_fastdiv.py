"""The multiply-shift division used by the SiLU vector kernel to map a pack index to its row
(Granlund & Montgomery, PLDI 1994: q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
m = floor(2^32 (2^l - d) / d) + 1), checked exhaustively at the edges and on random operands.
The same formula is computed on the host by make_fast_div32 (csrc/silu_and_mul.cuh)."""

from __future__ import annotations

import random


def make(d: int) -> tuple[int, int]:
    shift = 0
    while (1 << shift) < d:
        shift += 1
    return ((1 << 32) * ((1 << shift) - d)) // d + 1, shift


def fast_div(n: int, multiplier: int, shift: int) -> int:
    return (((n * multiplier) >> 32) + n) >> shift


def test_fast_division_is_exact() -> None:
    rng = random.Random(0)
    divisors = [1, 2, 3, 7, 8, 1184, 2368, 448, 65535, 65536, 2**31 - 1, 2**31, 2**31 + 1, 2**32 - 1]
    divisors += [rng.randrange(1, 2**32) for _ in range(500)]
    for d in divisors:
        multiplier, shift = make(d)
        assert multiplier < 2**32
        for n in [0, 1, d - 1, d, d + 1, 2**32 - 1, (2**32 - 1) // d * d] + [rng.randrange(2**32) for _ in range(50)]:
            if 0 <= n < 2**32:
                assert fast_div(n, multiplier, shift) == n // d, (d, n)
