"""Host logic of bench.py's multi-GPU mode on CPU: two gloo ranks, as
torchrun would start them (one process per rank, 127.0.0.1 rendezvous).
Replicas are independent (same weights, own prompt per rank) and the job's
time is the maximum over ranks. No device is used."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results):
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "light-rocm-runtime_b200"))
    import datetime

    import torch.distributed as dist

    import bench
    from lrrt_b200 import synthetic as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        weight_seed, prompt_seed = bench.rank_seeds(rank)
        prompt = S.prompt(prompt_seed, bench.PROMPT, bench.VOCAB)
        # Rank r "took" 1 + r seconds of device time and 10 - r end to end.
        elapsed, e2e = bench.max_over_ranks([1.0 + rank, 10.0 - rank], dist)
        gathered = [None] * world
        dist.all_gather_object(gathered, (weight_seed, prompt.tolist(),
                                          bench.stream_slice(rank, world)))
        results[rank] = (elapsed, e2e, gathered)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_max_and_keep_replicas_independent():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        processes = [ctx.Process(target=_rank_main, args=(r, world, port, results))
                     for r in range(world)]
        for p in processes:
            p.start()
        for p in processes:
            p.join(timeout=120)
        assert all(p.exitcode == 0 for p in processes), [p.exitcode for p in processes]
        results = dict(results)
    for rank in range(world):
        elapsed, e2e, gathered = results[rank]
        assert elapsed == 2.0 and e2e == 10.0  # max over ranks, on every rank
        (seed0, prompt0, streams0), (seed1, prompt1, streams1) = gathered
        assert seed0 == seed1                 # one model, replicated
        assert prompt0 != prompt1             # independent streams
        assert len(prompt0) == len(prompt1) == 32
        assert sorted(streams0 + streams1) == list(range(32))  # config 4, each stream once


def test_config4_stream_slices_cover_every_stream_once():
    """bench.py's config-4 partition: for 1, 2, 4 and 8 ranks the ranks'
    slices are disjoint, equal in size and together cover streams 0..31."""
    sys.path.insert(0, str(REPO))
    import pytest

    import bench
    for world in (1, 2, 4, 8):
        slices = [bench.stream_slice(rank, world) for rank in range(world)]
        assert all(len(s) == 32 // world for s in slices)
        assert sorted(stream for s in slices for stream in s) == list(range(32))
    for bad in ((0, 3), (2, 2), (0, 0)):
        with pytest.raises(ValueError):
            bench.stream_slice(*bad)
