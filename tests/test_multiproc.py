"""Multi-process (gloo, world_size 2, CPU) tests of the benchmark's rank
plumbing: ranks start together at a barrier, the timed region is the maximum
over ranks and throughput the sum of per-rank payloads; each rank draws its
own shard (seed = rank). No collective touches the data path."""

import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import bench  # noqa: E402  (repository root is on sys.path via conftest)
    from lmcache_b200 import workloads as wl

    r, w, local = bench.dist_setup()
    assert (r, w, local) == (rank, world, rank)
    bench.barrier(w)
    t_max = bench.max_over_ranks(10.0 + rank, w)
    total = bench.sum_over_ranks(100.0 * (rank + 1), w)
    slots = wl.make_slot_mapping(wl.SPECS["c5"], seed=rank)
    out.put((rank, t_max, total, slots[:64].tolist()))
    import torch.distributed as dist

    dist.destroy_process_group()


def test_two_rank_timing_reduction():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert all(t == 11.0 for _, t, _, _ in results)  # max over ranks
    assert all(s == 300.0 for _, _, s, _ in results)  # sum of payloads
    assert results[0][3] != results[1][3]  # independent per-rank shards
