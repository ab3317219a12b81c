"""Row sharding on GPUs: every block of rows runs through the CUDA kernel on its own device and is
checked against the oracle, with no peer memory and no collective on the data path.

* One process per GPU: two ranks (spawned), a gloo group for the verdicts only. The batch is a
  [4099, 8192] slice of the row-sharded workload's recipe (eps 1e-5, each rank's rows generated on
  its own device from seed + rank, the same weight on every device): an odd row count, so the two
  blocks differ by one row. Each rank checks its first and last row and a spread sample against
  the C oracle - residual bit for bit, output within rtol = atol = 1e-2 and one bf16 ulp - and the
  gathered blocks must tile the batch. Needs two GPUs; skipped on fewer.
* One process for several devices (``RowShardedBatch``): a [4099, 8192] host batch split into
  blocks, one stream and weight replica per block, enqueued from one thread and gathered back;
  every row is checked. Three blocks on one GPU's separate streams always run; two GPUs when
  present.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROWS, HIDDEN, EPS, WORLD = 4099, 8192, 1e-5, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, queue) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for path in (str(root / "inference-performance-lab_b200"), str(root), str(root / "tests")):
        sys.path.insert(0, path)
    import numpy as np
    import torch.distributed as dist

    from inference_performance_lab.kernels import capi, extension
    from inference_performance_lab.kernels.sharding import row_shard, shard_seed
    from oracle import oracle
    from parity import bf16_ulp_distance

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        torch.cuda.set_device(rank)
        extension.load_extension()
        shard = row_shard(ROWS, WORLD, rank)
        device = torch.device("cuda", rank)
        generator = torch.Generator(device=device).manual_seed(shard_seed(0, rank))
        x = torch.randn(shard.rows, HIDDEN, device=device, generator=generator).to(torch.bfloat16)
        r = torch.randn(shard.rows, HIDDEN, device=device, generator=generator).to(torch.bfloat16)
        w_gen = torch.Generator().manual_seed(0)
        w = (torch.randn(HIDDEN, generator=w_gen) * 0.1 + 1).to(torch.bfloat16).to(device)
        index = sorted({0, shard.rows - 1, *range(0, shard.rows, max(1, shard.rows // 64))})
        idx = torch.tensor(index, device=device)
        x_in, r_in = x.index_select(0, idx), r.index_select(0, idx)
        kernel = capi.fused_add_rms_norm_plan(x.data_ptr(), r.data_ptr(), w.data_ptr(), shard.rows, HIDDEN)
        torch.ops.inference_performance_lab.fused_add_rms_norm(x, r, w, EPS)
        torch.cuda.synchronize()
        want_out, want_res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x_in), oracle.tensor_bits(r_in),
                                                         oracle.tensor_bits(w), EPS)
        got_out = oracle.tensor_bits(x.index_select(0, idx))
        got_res = oracle.tensor_bits(r.index_select(0, idx))
        g, e = oracle.bf16_bits_to_f32(got_out), oracle.bf16_bits_to_f32(want_out)
        ok = (np.array_equal(got_res, want_res)
              and bool(np.all(np.abs(g - e) <= 1e-2 + 1e-2 * np.abs(e)))
              and int(bf16_ulp_distance(got_out.reshape(-1), want_out.reshape(-1)).max()) <= 1)
        record = {"rank": rank, "device": torch.cuda.current_device(), "start": shard.start, "stop": shard.stop,
                  "rows_checked": len(index), "kernel": kernel, "ok": bool(ok),
                  "fault": capi.device_fault_flags(rank)}
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, record)
        if rank == 0:
            queue.put(gathered)
    finally:
        dist.destroy_process_group()


def test_each_rank_runs_its_shard_on_its_own_gpu() -> None:
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs, found {torch.cuda.device_count()}")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(rank, port, queue)) for rank in range(WORLD)]
    for p in procs:
        p.start()
    gathered = queue.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [g["device"] for g in gathered] == list(range(WORLD))
    assert gathered[0]["start"] == 0 and gathered[-1]["stop"] == ROWS
    assert all(a["stop"] == b["start"] for a, b in zip(gathered, gathered[1:]))
    for g in gathered:
        assert g["ok"], g
        assert g["fault"] == 0 and g["rows_checked"] >= 64 and g["kernel"].startswith("rmsnorm_stash_kernel")


def _check_batch(devices) -> None:
    from inference_performance_lab.kernels.sharding import RowShardedBatch
    from oracle import oracle

    from parity import assert_bits_equal, assert_close_to_oracle

    rows, hidden = 4099, 8192
    generator = torch.Generator().manual_seed(11)
    x = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16).pin_memory()
    r = torch.randn(rows, hidden, generator=generator).to(torch.bfloat16).pin_memory()
    w = (torch.randn(hidden, generator=generator) * 0.1 + 1).to(torch.bfloat16)
    want_out, want_res = oracle.c_fused_add_rms_norm(oracle.tensor_bits(x), oracle.tensor_bits(r),
                                                     oracle.tensor_bits(w), EPS)
    batch = RowShardedBatch(x, r, w, devices)
    shards = [shard for shard, _, _ in batch.blocks]
    assert shards[0].start == 0 and shards[-1].stop == rows
    assert [b.device.index for b in batch._blocks] == [torch.device("cuda", d).index for d in devices]
    batch.fused_add_rms_norm(EPS)
    got_x, got_r = batch.gather()
    assert_bits_equal(got_r, want_res, f"residual over {devices}")
    assert_close_to_oracle(got_x, want_out, f"output over {devices}")


def test_row_sharded_batch_blocks_on_separate_streams_of_one_gpu() -> None:
    """Three row blocks of one host batch on GPU 0, each on its own stream with its own weight
    replica, enqueued from one thread; gathered in row order, every row matches the oracle."""
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    _check_batch([0, 0, 0])


def test_row_sharded_batch_over_two_gpus() -> None:
    """The same batch split over two GPUs from one process: each device runs its block on its own
    stream, nothing crosses between devices, and the gathered rows match the oracle."""
    if torch.cuda.device_count() < 2:
        pytest.skip(f"needs 2 GPUs, found {torch.cuda.device_count()}")
    _check_batch([0, 1])
