"""Row sharding of a large add+RMSNorm batch across the GPUs of one node.

Rows are independent (the reduction of a row never leaves the row), so a batch of R rows runs on
N GPUs as N contiguous row blocks with no collective: rank k owns rows
[R*k // N, R*(k+1) // N) and launches the single-GPU kernel on its own block, on its own device
and stream, with its own copy of the weight. Block sizes differ by at most one row.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class RowShard:
    rank: int
    world_size: int
    start: int
    stop: int

    @property
    def rows(self) -> int:
        return self.stop - self.start


def row_shard(rows: int, world_size: int, rank: int) -> RowShard:
    """Contiguous block of ``rows`` owned by ``rank`` of ``world_size``."""
    if rows < 0:
        raise ValueError("rows must be non-negative")
    if world_size < 1:
        raise ValueError("world_size must be positive")
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} is outside [0, {world_size})")
    return RowShard(rank, world_size, rows * rank // world_size, rows * (rank + 1) // world_size)


def shard_seed(seed: int, rank: int) -> int:
    """Seed of rank ``rank``'s synthetic shard (each rank generates its rows on its own device)."""
    return seed + rank
