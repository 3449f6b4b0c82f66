"""Data-parallel host logic on CPU: world_size-2 gloo ranks (no GPU).

Configs 1-4 shard as independent sequences with no collective on the data path; the only
cross-rank step is bench.py's whole-job reduction (max of device time, sum of tokens), and each rank
decodes its own seeded prompt.
"""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench

        ms, tok = bench.reduce_over_ranks(dist, ms=100.0 + 50.0 * rank, tokens=10 + rank)
        cfg = dict(bench.CONFIGS[2])
        p = bench.prompt_for(cfg, 151936, rank)
        out[rank] = (ms, tok, tuple(p[:8]), len(p))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_time_by_max_and_tokens_by_sum():
    port = free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    r0, r1 = out[0], out[1]
    assert r0[0] == r1[0] == 150.0  # slowest rank
    assert r0[1] == r1[1] == 21.0  # all tokens
    assert r0[3] == r1[3] == 512  # config-2 prompt length on every rank
    assert r0[2] != r1[2]  # independent sequences: each rank its own seeded prompt
