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
