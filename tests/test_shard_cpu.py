"""Replica sharding host logic on CPU: the length-balanced partition, and a world-size-2 gloo
job (two processes on 127.0.0.1) that runs each rank's share through a stand-in transcriber,
gathers the results on rank 0 in input order and reduces the time as the max over ranks."""
import os
import socket

import numpy as np
import pytest

from moonshine_b200.shard import partition_by_length


def test_partition_covers_every_item_once_and_balances():
    rng = np.random.Generator(np.random.PCG64(3))
    lengths = rng.integers(16000 * 2, 16000 * 30, size=257).tolist()
    for world in (1, 2, 3, 8):
        shares = partition_by_length(lengths, world)
        flat = sorted(i for s in shares for i in s)
        assert flat == list(range(len(lengths)))
        assert all(s == sorted(s) for s in shares)
        totals = [sum(lengths[i] for i in s) for s in shares]
        assert max(totals) - min(totals) <= max(lengths)
    assert partition_by_length([], 4) == [[], [], [], []]
    assert partition_by_length([5, 5, 5], 2) == [[0, 2], [1]]
    with pytest.raises(ValueError):
        partition_by_length([1], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path):
    import datetime
    import time
    import torch.distributed as dist
    from moonshine_b200.shard import sharded_transcription
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    items = [f"utt{i}" for i in range(11)]
    lengths = [(i * 37) % 11 + 1 for i in range(11)]

    def transcribe(batch):  # stand-in for a model call: ids derived from the item
        time.sleep(0.05 * (rank + 1))
        return [[int(s[3:]), rank] for s in batch]

    res, seconds = sharded_transcription(items, lengths, transcribe)
    if rank == 0:
        with open(out_path, "w") as f:
            f.write(repr((res, seconds)))
    dist.destroy_process_group()


def test_two_rank_gloo_job(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "res.txt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    res, seconds = eval(open(out).read())
    assert [r[0] for r in res] == list(range(11))
    lengths = [(i * 37) % 11 + 1 for i in range(11)]
    shares = partition_by_length(lengths, 2)
    for rank, share in enumerate(shares):
        assert all(res[i][1] == rank for i in share)
    assert seconds >= 0.1  # the slower rank (rank 1 sleeps 0.1 s) sets the job time
