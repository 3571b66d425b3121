"""The N > 1 path of bench.py on CPU: two gloo ranks shard utterances (each
rank draws its own batches) and reduce the whole-job figures (max of the
per-rank times, sum of the audio) with no data-path collective."""
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
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # each rank's batches are its own: no utterance is processed twice
        mine = [tuple(bench.utterance_lengths(step, rank)) for step in range(4)]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        flat = [b for r in gathered for b in r]
        assert len(set(flat)) == len(flat), "ranks drew the same batch"
        for r in gathered:
            for batch in r:
                assert len(batch) == 8 and all(16000 * 5 <= n <= 16000 * 30 for n in batch)
        # whole-job aggregation: the slowest rank's times, the sum of the audio
        dev, e2e, audio = 1.0 + rank, 2.0 + 3 * rank, 100.0 * (rank + 1)
        got = bench.reduce_over_ranks(dev, e2e, audio, "cpu")
        want = (float(world), 2.0 + 3 * (world - 1), 100.0 * world * (world + 1) / 2)
        assert got == want, (got, want)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


def test_single_process_reduce_is_identity():
    import bench

    assert bench.reduce_over_ranks(1.5, 2.5, 30.0, "cpu") == (1.5, 2.5, 30.0)


@pytest.mark.parametrize("rank", [0, 1, 7])
def test_utterance_lengths_are_seeded(rank):
    import bench

    assert bench.utterance_lengths(3, rank) == bench.utterance_lengths(3, rank)
