"""Host side of data-parallel serving (wam_b200/dp.py), on CPU: request
sharding, the max-over-ranks time reduction, whole-job throughput and the
ordered gather of results, the last two over a world-size-2 gloo process group
on 127.0.0.1 (the same calls bench.py makes over NCCL under torchrun)."""
import socket

import pytest


def test_shard_tiles_requests_in_rank_order():
    from wam_b200 import dp

    for n in (0, 1, 5, 63, 64, 65, 1000):
        for world in (1, 2, 3, 4, 8):
            blocks = [dp.shard(n, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == n
            for (s0, e0), (s1, _) in zip(blocks, blocks[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in blocks]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)
    assert dp.shard(64, 8, 3) == (24, 32)  # config 4: 64 requests over 8 GPUs


def test_shard_rejects_bad_ranks():
    from wam_b200 import dp

    with pytest.raises(ValueError):
        dp.shard(10, 2, 2)
    with pytest.raises(ValueError):
        dp.shard(10, 0, 0)
    with pytest.raises(ValueError):
        dp.shard(-1, 2, 0)


def test_request_seeds_distinct_across_ranks():
    from wam_b200 import dp

    seeds = {dp.request_seed(20261201, r, i) for r in range(8) for i in range(64)}
    assert len(seeds) == 8 * 64


def test_single_process_paths():
    from wam_b200 import dp

    assert dp.max_over_ranks(3.5) == 3.5
    assert dp.gather_in_order([1, 2, 3], 3) == [1, 2, 3]
    assert dp.job_throughput([10, 10], 2.0) == 10.0
    with pytest.raises(ValueError):
        dp.job_throughput([1], 0.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n):
    import datetime
    import os
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "wam.cpp_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from wam_b200 import dp

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        start, stop = dp.shard(n, world, rank)
        # results of this rank's requests, tagged with the request index
        local = [f"chunk-{i}" for i in range(start, stop)]
        got = dp.gather_in_order(local, n, dist)
        if rank == 0:
            assert got == [f"chunk-{i}" for i in range(n)], got
        else:
            assert got is None
        # the job time is the slowest rank's
        t = dp.max_over_ranks(1.0 + rank * 0.25, dist)
        assert t == 1.0 + (world - 1) * 0.25
        sizes = [0] * world
        for r in range(world):
            s, e = dp.shard(n, world, r)
            sizes[r] = e - s
        assert dp.job_throughput(sizes, t) == n / t
        # a rank holding the wrong number of results is an error, raised
        # before the collective (no rank is left waiting in it)
        if rank == 1:
            with pytest.raises(ValueError):
                dp.gather_in_order(local + ["extra"], n, dist)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [5, 64])
def test_gloo_world2_gather_and_max(n):
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port(), n), nprocs=2, join=True)
