"""The bench's N > 1 host path on CPU: two gloo ranks (replicas only, no data-path
collective) line up at barriers, take the slowest rank's time, sum the ranks'
work, and only rank 0 runs the reference arm."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ranks = bench.Ranks(dist, "cpu")
        ranks.barrier()
        slowest = ranks.max(0.5 + rank)  # rank r took 0.5 + r seconds
        value = bench.aggregate_rate(world, 62, slowest)

        class Args:
            steps, warmup, seed, checkpoint = 1, 3, 0, "/nonexistent"

        rc = bench.run_reference(Args, rank, world) if rank != 0 else 0  # rank 0 would time the oracle
        ranks.barrier()
        out[rank] = (slowest, value, rc)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_slowest_time_and_sum_work():
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    for rank in range(world):
        slowest, value, rc = out[rank]
        assert slowest == pytest.approx(1.5)
        assert value == pytest.approx(2 * 62 / 1.5)
        assert rc == 0


def test_single_rank_is_a_no_op():
    sys.path.insert(0, ROOT)
    import bench
    r = bench.Ranks()
    r.barrier()
    assert r.max(3.25) == 3.25
    assert bench.aggregate_rate(1, 10, 2.0) == 5.0
