"""The multi-GPU bench's host logic on CPU: two `gloo` ranks.

`bench.py --gpus N` runs one process per GPU with no collective on the hot
path: each rank decodes its own requests over its own pool, the timed windows
are bracketed by barriers, the step time is the max over ranks, and rank 0
alone prints the JSON line (and, for the reference arm, alone does the work).
These tests run that logic as two CPU processes joined by gloo.
"""

import importlib.util
import multiprocessing as mp
import os
import socket
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, REPO)
    bench = _bench()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # rank r timed [1 + r, 10 - r, 5]: every rank must see the max of each
        got = bench.max_over_ranks([1.0 + rank, 10.0 - rank, 5.0], dist, "cpu")
        per_rank = bench.gather_ranks(0.5 + rank, dist, "cpu")
        seeds = bench.shard_seeds(rank)
        ref_line = bench.run_reference_arm(None, rank) if rank != 0 else "rank0"
        q.put((rank, got, seeds, ref_line, per_rank))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_max_and_shard_their_data():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    by_rank = {r: (got, seeds, ref, per) for r, got, seeds, ref, per in results}
    for r in range(world):
        assert by_rank[r][0] == [2.0, 10.0, 5.0]          # max over ranks, on every rank
        assert by_rank[r][3] == [0.5, 1.5]                # every rank's step time, rank order
    assert by_rank[0][1] != by_rank[1][1]                  # each rank its own pool and sets
    assert by_rank[1][2] is None                           # reference arm: rank 1 does no work


def test_job_throughput_counts_every_rank():
    bench = _bench()
    kv = 64 * 2048 * 656
    one = bench.job_kv_gbs(1, kv, 0.089)
    assert abs(bench.job_kv_gbs(8, kv, 0.089) - 8 * one) < 1e-6 * one
    assert bench.max_over_ranks([3.0, 4.0], None, "cpu") == [3.0, 4.0]
