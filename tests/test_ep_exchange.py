"""The expert-parallel exchange protocol on two gloo ranks (CPU, no GPU).

The GPU path (engine `ep_moe`, csrc/ep.cu) sends each routed (token, rank)
slot's FFN input row to the owner of its expert (expert e on rank
e / (32 / world)), the owner runs that expert on it, the down rows come back
in the order they were sent, and the origin combines them in rank order
(kernels/resident.rs:101-117). Here the same send plan (`lfm_ep_plan` of the
engine library, host code) drives a gloo all-to-all with a stand-in expert
function, and each rank's result must equal the single-process combine bit
for bit: the plan covers every slot once, groups it by owner, owners only see
their own experts, and the returned rows land on the right slots.
"""

import os
import socket

import numpy as np
import pytest

DIM = 16


def stand_in_expert(e, x):
    return (np.float32(e + 1) * x + np.float32(0.5) * np.float32(e)).astype(np.float32)


def routing(rank, n):
    rng = np.random.default_rng(50 + rank)
    sel = np.stack([rng.permutation(32)[:4] for _ in range(n)]).astype(np.int32)
    w = rng.random((n, 4), dtype=np.float32)
    x = rng.normal(size=(n, DIM)).astype(np.float32)
    return sel, w, x


def combine(x, w, down):
    """x[t] + sum_r w[t, r] * down[t, r] in rank order, float32 (resident.rs:101-117)."""
    out = x.copy()
    for t in range(x.shape[0]):
        acc = out[t].copy()
        for r in range(4):
            acc = (acc + w[t, r] * down[t, r]).astype(np.float32)
        out[t] = acc
    return out


def worker(rank, world, port, ns, results):
    import torch
    import torch.distributed as dist

    import lfm2_b200
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = ns[rank]
        sel, w, x = routing(rank, n)
        per = 32 // world
        counts, order = lfm2_b200.ep_plan(sel, world)
        assert int(counts.sum()) == 4 * n and sorted(order.tolist()) == list(range(4 * n))
        for o, part in enumerate(np.split(order, np.cumsum(counts)[:-1])):
            assert (sel.ravel()[part] // per == o).all() and (np.diff(part) > 0).all()
        send = x[order // 4]
        tags = sel.ravel()[order]
        # counts of every rank, then the rows and their expert ids
        allc = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(counts.astype(np.int64)))
        recv_counts = [int(allc[p][rank]) for p in range(world)]
        rows = torch.empty(sum(recv_counts), DIM)
        dist.all_to_all_single(rows, torch.from_numpy(send), recv_counts, counts.tolist())
        rtags = torch.empty(sum(recv_counts), dtype=torch.int64)
        dist.all_to_all_single(rtags, torch.from_numpy(tags.astype(np.int64)), recv_counts, counts.tolist())
        rtags = rtags.numpy()
        assert (rtags // per == rank).all(), "a slot reached a rank that does not own its expert"
        out = np.stack([stand_in_expert(int(e), r) for e, r in zip(rtags, rows.numpy())]) if len(rtags) else \
            np.zeros((0, DIM), np.float32)
        back = torch.empty(4 * n, DIM)
        dist.all_to_all_single(back, torch.from_numpy(out), counts.tolist(), recv_counts)
        down = np.empty((4 * n, DIM), np.float32)
        down[order] = back.numpy()
        got = combine(x, w, down.reshape(n, 4, DIM))
        ref = combine(x, w, np.stack([[stand_in_expert(int(sel[t, r]), x[t]) for r in range(4)] for t in range(n)]))
        results[rank] = bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ns", [(7, 5), (1, 12)])
def test_two_rank_exchange_matches_single_process(ns):
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(worker, args=(2, _free_port(), ns, results), nprocs=2, join=True)
    assert dict(results) == {0: True, 1: True}


def test_plan_four_ranks_and_rejects_bad_ids():
    import lfm2_b200
    sel = np.array([[0, 8, 16, 24], [31, 30, 7, 9]], np.int32)
    counts, order = lfm2_b200.ep_plan(sel, 4)
    # owners (8 experts each): slots 0..7 -> ranks 0 1 2 3 3 3 0 1
    assert counts.tolist() == [2, 2, 1, 3]
    # destinations ascending, slots ascending within a destination
    assert order.tolist() == [0, 6, 1, 7, 2, 3, 4, 5]
    with pytest.raises(lfm2_b200.LfmError):
        lfm2_b200.ep_plan(np.array([0, 32], np.int32), 2)
