"""Batch-sharding host logic on CPU ranks (gloo, world_size 2).

Each rank convolves its own images; the oracle stands in for the GPU kernel
here (test only), so this checks the split, the slicing and the verification
gather, not the kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import sharding


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (5, 2), (3, 4), (7, 3)])
def test_shard_range_partitions_the_batch(n, world):
    ranges = [sharding.shard_range(n, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shape_tuple, result_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "..", "oracle"))
    import pyoracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = m.ConvShape(*shape_tuple)
        x, w, b = m.make_inputs(full, seed=11)
        local = sharding.shard_shape(full, rank, world)
        xl = sharding.input_slice(x, full, rank, world)
        yl = torch.from_numpy(pyoracle.conv(local, xl, w, b, threads=1))
        gathered = sharding.gather_outputs(yl, full, rank, world, dist)
        if rank == 0:
            ok = np.array_equal(gathered.numpy(), pyoracle.conv(full, x, w, b, threads=2))
            with open(result_path, "w") as f:
                f.write("ok" if ok else "mismatch")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [4, 5])
def test_sharded_outputs_gather_to_the_unsharded_result(tmp_path, n):
    shape = m.ConvShape(n, 9, 7, 32, 24, 3, 3, 1, 1, 1, 1, 1, 1)
    result = tmp_path / "result.txt"
    mp.spawn(_rank_main, args=(2, _free_port(), shape.as_tuple(), str(result)), nprocs=2,
             join=True)
    assert result.read_text() == "ok"


def _verify_rank_main(rank, world, port, plant, result_path):
    # bench.verify_sharded on CPU ranks: each rank holds its shard's output
    # (computed here by the oracle, standing in for the timed launches), rank
    # 0 gathers and checks against the oracle.  `plant` corrupts one output
    # of rank 1's timed slice, which the check must catch.
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, ".."))
    sys.path.insert(0, os.path.join(here, "..", "oracle"))
    import pyoracle

    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = m.ConvShape(6, 9, 9, 32, 24, 3, 3, 1, 1, 1, 1, 1, 1)
        x, w, b = m.make_inputs(full, seed=4)
        local = sharding.shard_shape(full, rank, world)
        xl = sharding.input_slice(x, full, rank, world)
        yl = pyoracle.conv(local, xl, w, b, threads=1)
        timed = torch.from_numpy(yl.copy())
        if plant and rank == 1:
            timed[timed.numel() // 2] += 1
        e2e = torch.from_numpy(yl.copy())
        res = bench.verify_sharded(full, x, w, b, timed, e2e, dist, rank, world,
                                   {"sm_mhz": 1000.0 + rank})
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(f"{res['timed_output']} {res['e2e_output']} "
                        f"{len(res['clocks_per_rank'])} {res['clocks_per_rank'][1]['sm_mhz']}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", [False, True])
def test_bench_sharded_verification_against_the_oracle(tmp_path, plant):
    out = tmp_path / "result"
    mp.start_processes(_verify_rank_main, args=(2, _free_port(), plant, str(out)), nprocs=2,
                       join=True, start_method="spawn")
    timed, e2e, nclocks, mhz = out.read_text().split()
    assert timed == ("False" if plant else "True")
    assert e2e == "True" and nclocks == "2" and float(mhz) == 1001.0
