"""Multi-rank host logic of the replicated decode benchmark, as world-size-2 gloo ranks on the CPU.

Batch-1 decode does not shard: under torchrun every rank runs an independent replica with its own
prompt (config 1) or its own partition of the sequence set (config 5), and the only collectives are a
barrier and one max-all-reduce of the timings.  These tests run that host logic (`bench.py`'s
helpers) in two spawned processes over gloo, with the same calls the GPU ranks make over NCCL.
"""
import datetime
import importlib
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    try:
        bench = importlib.import_module("bench")
        dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
        assert bench.dist_setup() == (ws, rank, rank)
        # per-rank device and end-to-end times (ms): rank 1 is slower on the first, rank 0 on the second
        local = [100.0 + 10.0 * rank, 50.0 - 5.0 * rank]
        dist.barrier()
        reduced = bench.max_over_ranks(dist, local, "cpu")
        value = bench.aggregate_rate(128, 4, ws, reduced[0])
        seeds = bench.batched_sequence_seeds(rank, 256)
        prompt_seed = bench.replica_prompt_seed(0, rank)
        gathered = [None] * ws
        dist.all_gather_object(gathered, (seeds, prompt_seed))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, reduced, value, gathered, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, None, None, repr(e)))


def test_two_gloo_ranks_reduce_the_max_and_partition_the_replicas():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ws, port = 2, _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(ws):
            rank, reduced, value, gathered, err = q.get(timeout=120)
            results[rank] = (reduced, value, gathered, err)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(ws):
        assert results[r][3] is None, results[r][3]
    # every rank receives the same element-wise max (110 ms device, 50 ms end to end)
    for r in range(ws):
        assert results[r][0] == [110.0, 50.0]
    # whole-job rate: the tokens of both ranks (2 x 4 steps x 128) over the slowest rank's 110 ms
    for r in range(ws):
        assert results[r][1] == pytest.approx(2 * 4 * 128 / 0.110)
    # replicas are independent: disjoint sequence partitions, distinct batch-1 prompt seeds
    (s0, p0), (s1, p1) = results[0][2]
    assert len(s0) == len(s1) == 256
    assert not set(s0) & set(s1)
    assert s1[0] == s0[-1] + 1
    assert p0 != p1


def test_single_process_helpers_need_no_process_group():
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    assert bench.max_over_ranks(None, [3, 4.5], "cpu") == [3.0, 4.5]
    assert bench.aggregate_rate(128, 10, 1, 616.6) == pytest.approx(128 * 10 / 0.6166)
    assert bench.batched_sequence_seeds(0, 3) == [4000, 4001, 4002]
    assert bench.replica_prompt_seed(2, 0) == 2
