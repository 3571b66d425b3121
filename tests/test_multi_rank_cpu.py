"""The N > 1 path of bench.py on CPU: gloo ranks shard configs[4]'s fixed
512-utterance job round-robin (utterance u on rank u mod N), every utterance
exactly once, and reduce the whole-job figures (max of the per-rank times, sum
of the audio, every rank's job time) with no data-path collective."""
import os
import socket

import pytest

from tests.conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int) -> None:
    import sys

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"], os.environ["WORLD_SIZE"] = str(rank), str(world)
    bench.init_ranks(world)
    try:
        # the shards partition the job: every utterance once, round-robin, batches of <= 8
        mine = bench.job_shard(world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        flat = [u for r in gathered for b in r for u in b]
        assert sorted(flat) == list(range(bench.JOB_UTTS)), "the shards do not partition the job"
        for r, shard in enumerate(gathered):
            assert all(u % world == r for b in shard for u in b) and all(1 <= len(b) <= 8 for b in shard)
        # whole-job aggregation: the slowest rank's times, the sum of the audio, all job times
        dev, e2e, audio = 1.0 + rank, 2.0 + 3 * rank, 100.0 * (rank + 1)
        got = bench.reduce_over_ranks(dev, e2e, audio)
        want = (float(world), 2.0 + 3 * (world - 1), 100.0 * world * (world + 1) / 2)
        assert got == want, (got, want)
        assert bench.gather_over_ranks(10.0 + rank) == [10.0 + r for r in range(world)]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_shard_the_job_and_reduce(world):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(world, _free_port()), nprocs=world, join=True, start_method="spawn")


def test_single_process_reduce_is_identity():
    import bench

    assert bench.reduce_over_ranks(1.5, 2.5, 30.0) == (1.5, 2.5, 30.0)
    assert bench.gather_over_ranks(4.0) == [4.0]


def test_job_is_configs4():
    """512 seeded utterances with lengths in [5, 30] s; one shard per GPU count splits
    into whole batches of 8 at N = 1, 2, 4, 8."""
    import bench

    lens = bench.job_lengths()
    assert len(lens) == 512 and lens == bench.job_lengths()
    assert all(16000 * 5 <= n <= 16000 * 30 for n in lens)
    for world in (1, 2, 4, 8):
        shards = [bench.job_shard(world, r) for r in range(world)]
        assert all(len(s) == 64 // world and all(len(b) == 8 for b in s) for s in shards)
