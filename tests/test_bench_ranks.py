"""bench.py's multi-rank plumbing on CPU: two gloo ranks (one process each,
rendezvous on 127.0.0.1) take the max of their timings and meet at the
barrier, the same calls the GPU run makes over NCCL."""

import os
import socket

import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, root, out):
    import datetime
    import sys

    import torch.distributed as dist

    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        times = [3.5, 7.25]  # per-rank device milliseconds
        m = bench.reduce_max(dist, times[rank])
        bench.barrier(dist)
        out.put((rank, m, bench.reduce_max(None, times[rank])))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_max_time():
    from conftest import ROOT
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, ROOT, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, 7.25, 3.5), (1, 7.25, 7.25)]
