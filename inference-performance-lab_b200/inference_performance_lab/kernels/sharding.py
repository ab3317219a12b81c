"""Row sharding of a large add+RMSNorm batch across the GPUs of one node.

Rows are independent (the reduction of a row never leaves the row), so a batch of R rows runs on
N GPUs as N contiguous row blocks with no collective: block k holds rows
[R*k // N, R*(k+1) // N), runs the single-GPU kernel on its own device and stream with its own
copy of the weight, and block sizes differ by at most one row.

Two ways to use it:

* one process per GPU (torchrun): each rank takes ``row_shard(rows, world_size, rank)`` and calls
  the op on its block (``bench.py``'s ``sharded`` record);
* one process for several GPUs: ``RowShardedBatch`` splits a batch over a list of devices, keeps
  each block, a weight replica and a stream per device, and enqueues the op on every device from
  the one host thread - the launches are asynchronous, so all devices run at once - then gathers
  the blocks back in row order.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence


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


@dataclass
class _Block:
    shard: RowShard
    device: "object"  # torch.device
    stream: "object"  # torch.cuda.Stream
    x: "object"
    residual: "object"
    weight: "object"


class RowShardedBatch:
    """A bf16 [rows, hidden] add+RMSNorm batch split by rows over several CUDA devices.

    ``x`` and ``residual`` ([rows, hidden], bf16) and ``weight`` ([hidden], bf16) may live on the
    host (pinned memory copies without blocking the host) or on any device. Block k of
    ``row_shard(rows, len(devices), k)`` is copied to ``devices[k]`` on that block's own stream,
    with its own replica of the weight; a device may appear more than once (its blocks then run
    on separate streams of that device). Nothing crosses between devices after that: no
    collective, no peer access.

    ``fused_add_rms_norm(epsilon)`` enqueues the op on every block's stream and returns at once;
    ``synchronize()`` waits for all of them; ``gather()`` copies the blocks back to the host in row
    order. The blocks are ordinary tensors (``blocks``) for callers that keep working on device.
    """

    def __init__(self, x, residual, weight, devices: Sequence) -> None:
        import torch

        if len(devices) == 0:
            raise ValueError("at least one device is needed")
        if x.ndim != 2 or x.shape != residual.shape:
            raise ValueError("x and residual must be [rows, hidden] with identical shapes")
        if weight.ndim != 1 or weight.shape[0] != x.shape[1]:
            raise ValueError("weight must match the final tensor dimension")
        if {x.dtype, residual.dtype, weight.dtype} != {torch.bfloat16}:
            raise ValueError("x, residual and weight must use bfloat16")
        self.rows, self.hidden = int(x.shape[0]), int(x.shape[1])
        self._blocks: list[_Block] = []
        for k, dev in enumerate(devices):
            device = torch.device("cuda", dev) if isinstance(dev, int) else torch.device(dev)
            if device.type != "cuda":
                raise ValueError(f"device {dev!r} is not a CUDA device")
            shard = row_shard(self.rows, len(devices), k)
            stream = torch.cuda.Stream(device=device)
            with torch.cuda.device(device), torch.cuda.stream(stream):
                block = _Block(
                    shard, device, stream,
                    x[shard.start:shard.stop].to(device, non_blocking=True).contiguous(),
                    residual[shard.start:shard.stop].to(device, non_blocking=True).contiguous(),
                    weight.to(device, non_blocking=True).contiguous(),
                )
            self._blocks.append(block)

    @property
    def blocks(self) -> list:
        """(shard, x block, residual block) per block, in row order."""
        return [(b.shard, b.x, b.residual) for b in self._blocks]

    def fused_add_rms_norm(self, epsilon: float) -> None:
        """Enqueue the op on every block's device and stream (asynchronous: all blocks run at once)."""
        import torch

        from inference_performance_lab.kernels.extension import load_extension

        load_extension()
        for b in self._blocks:
            if b.shard.rows == 0:
                continue
            with torch.cuda.device(b.device), torch.cuda.stream(b.stream):
                torch.ops.inference_performance_lab.fused_add_rms_norm(b.x, b.residual, b.weight, epsilon)

    def synchronize(self) -> None:
        for b in self._blocks:
            b.stream.synchronize()

    def gather(self):
        """(x, residual) on the host, [rows, hidden], pinned; copied on each block's stream."""
        import torch

        x = torch.empty(self.rows, self.hidden, dtype=torch.bfloat16, pin_memory=True)
        residual = torch.empty(self.rows, self.hidden, dtype=torch.bfloat16, pin_memory=True)
        for b in self._blocks:
            with torch.cuda.device(b.device), torch.cuda.stream(b.stream):
                x[b.shard.start:b.shard.stop].copy_(b.x, non_blocking=True)
                residual[b.shard.start:b.shard.stop].copy_(b.residual, non_blocking=True)
        self.synchronize()
        return x, residual
