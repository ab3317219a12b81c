"""Row sharding across ranks (host logic), including a world_size-2 gloo run.

Each rank normalises its own contiguous block of rows (here with the CPU oracle standing in for a
GPU); the gathered blocks must equal the whole batch normalised at once: rows are independent,
so sharding needs no collective on the data path.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inference_performance_lab.kernels.sharding import row_shard, shard_seed


@pytest.mark.parametrize("rows", [0, 1, 7, 2048, 262144])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_tile_the_rows(rows: int, world: int) -> None:
    shards = [row_shard(rows, world, rank) for rank in range(world)]
    assert shards[0].start == 0 and shards[-1].stop == rows
    for left, right in zip(shards, shards[1:]):
        assert left.stop == right.start
    sizes = [s.rows for s in shards]
    assert max(sizes) - min(sizes) <= 1


def test_row_shard_rejects_bad_arguments() -> None:
    with pytest.raises(ValueError):
        row_shard(10, 0, 0)
    with pytest.raises(ValueError):
        row_shard(10, 2, 2)
    with pytest.raises(ValueError):
        row_shard(-1, 2, 0)
    assert shard_seed(0, 3) == 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, rows: int, hidden: int, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle

        generator = torch.Generator().manual_seed(0)
        x = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        r = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
        w = (torch.randn(hidden, generator=generator) * 0.1 + 1).to(torch.bfloat16)
        shard = row_shard(rows, world, rank)
        out, res = oracle.c_fused_add_rms_norm(
            oracle.tensor_bits(x[shard.start:shard.stop]),
            oracle.tensor_bits(r[shard.start:shard.stop]),
            oracle.tensor_bits(w),
            1e-5,
        )
        # Timing aggregation as bench.py does it: max over ranks.
        elapsed = torch.tensor([float(rank + 1)])
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        gathered = [None] * world
        dist.all_gather_object(gathered, (shard.start, shard.stop, out, res))
        if rank == 0:
            queue.put((elapsed.item(), gathered))
    finally:
        dist.destroy_process_group()


def test_gloo_two_rank_sharding_matches_whole_batch() -> None:
    rows, hidden, world = 37, 257, 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rank, world, port, rows, hidden, queue)) for rank in range(world)]
    for p in procs:
        p.start()
    elapsed, gathered = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert elapsed == float(world)

    from oracle import oracle

    generator = torch.Generator().manual_seed(0)
    x = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
    r = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16)
    w = (torch.randn(hidden, generator=generator) * 0.1 + 1).to(torch.bfloat16)
    out, res = oracle.c_fused_add_rms_norm(
        oracle.tensor_bits(x), oracle.tensor_bits(r), oracle.tensor_bits(w), 1e-5
    )
    covered = 0
    for start, stop, shard_out, shard_res in gathered:
        np.testing.assert_array_equal(shard_out, out[start:stop])
        np.testing.assert_array_equal(shard_res, res[start:stop])
        covered += stop - start
    assert covered == rows


def _failing_rank_worker(rank: int, world: int, port: int, queue) -> None:
    import sys
    import time
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench

    d = bench.Dist(timeout_s=5.0)
    d.barrier()  # step 1 completes on both ranks
    if rank == 1:
        raise RuntimeError("rank 1 fails between steps")
    start = time.monotonic()
    try:
        d.barrier()
        queue.put(("no error", time.monotonic() - start))
    except Exception as error:  # noqa: BLE001 - any error ends the wait, which is the point
        queue.put((type(error).__name__, time.monotonic() - start))
    queue.close()
    queue.join_thread()  # the item is in the pipe before the process ends
    os._exit(3)  # leave without waiting on the failed peer


def test_failed_rank_ends_the_others_barrier() -> None:
    """bench.py's process group: a rank that raises between steps makes the surviving rank's next
    barrier end with an error within the group timeout, not hang (gloo, world size 2, CPU)."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_worker, args=(rank, 2, port, queue)) for rank in range(2)]
    for p in procs:
        p.start()
    outcome, waited = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert outcome != "no error"
    assert waited < 30.0
    assert procs[1].exitcode not in (0, None) and procs[0].exitcode == 3


def _control_plane_worker(rank: int, world: int, port: int, queue) -> None:
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench

    d = bench.Dist(timeout_s=30.0)
    try:
        d.barrier()
        elapsed = d.max(1.5 * (rank + 1))
        verdict = d.all(rank != 1)
        per_rank = d.gather({"rank": rank, "us": 10.0 + rank})
        if rank == 0:
            queue.put((d.pg.get_backend(), elapsed, verdict, per_rank))
    finally:
        d.close()


def test_bench_control_plane_is_gloo_on_the_host() -> None:
    """bench.py's timing control plane (barrier, max over ranks, the parity verdict, per-rank
    records) runs on a gloo group of host tensors: no NCCL and no device collective."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_control_plane_worker, args=(rank, 2, port, queue)) for rank in range(2)]
    for p in procs:
        p.start()
    backend, elapsed, verdict, per_rank = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert backend == "gloo"
    assert elapsed == 3.0
    assert verdict is False  # one rank's failed check fails the run
    assert [r["rank"] for r in per_rank] == [0, 1] and per_rank[1]["us"] == 11.0


def test_row_sharded_batch_rejects_bad_arguments() -> None:
    from inference_performance_lab.kernels.sharding import RowShardedBatch

    x = torch.zeros(8, 16, dtype=torch.bfloat16)
    w = torch.zeros(16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="at least one device"):
        RowShardedBatch(x, x.clone(), w, [])
    with pytest.raises(ValueError, match="identical shapes"):
        RowShardedBatch(x, torch.zeros(8, 8, dtype=torch.bfloat16), w, ["cuda:0"])
    with pytest.raises(ValueError, match="final tensor dimension"):
        RowShardedBatch(x, x.clone(), torch.zeros(8, dtype=torch.bfloat16), ["cuda:0"])
    with pytest.raises(ValueError, match="bfloat16"):
        RowShardedBatch(x.float(), x.float(), w, ["cuda:0"])
    with pytest.raises(ValueError, match="not a CUDA device"):
        RowShardedBatch(x, x.clone(), w, ["cpu"])
