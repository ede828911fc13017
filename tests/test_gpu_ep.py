"""Expert-parallel prefill on two GPUs against the single-GPU prefill.

Two processes, one GPU each (skipped with fewer than two GPUs): each rank
prefills its own prompts once on its own (every expert local) and once
expert-parallel (lfm_ep_prefill: rank r computes experts 16r..16r+15 for the
tokens of both ranks, routed rows exchanged through NCCL), into session slots
and into the engine's own session. The routed rows, the expert GEMMs on them
and the rank-ordered combine are the same arithmetic either way, so logits
and next tokens must agree (logits within 1e-3: the plain path runs the last
layer's FFN with the decode kernels, the expert-parallel path with the prompt
GEMMs).
"""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def worker(rank, port, path, results):
    import torch
    import torch.distributed as dist

    import lfm2_b200
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    e = None
    try:
        e = lfm2_b200.GpuEngine(path, rank)
        e.set_ctx(1024)
        ids = [lfm2_b200.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        e.ep_init(ids[0], rank, 2)
        rng = np.random.default_rng(900 + rank)
        prompts = [rng.integers(0, 128000, n).astype(np.uint32) for n in ((37, 300, 5) if rank else (200, 1, 64))]
        e.batch_create(len(prompts))
        worst, same = 0.0, True
        for i, p in enumerate(prompts):
            t0 = e.batch_prefill(i, p)
            ref = e.snapshot_resident_logits()
            t1 = e.ep_prefill(p, i)
            got = e.snapshot_resident_logits()
            worst = max(worst, float(np.abs(got - ref).max()))
            same = same and t0 == t1
        e.reset_session()
        ref = e.forward(prompts[0], 0)
        t2 = e.ep_prefill(prompts[0])
        got = e.snapshot_resident_logits()
        worst = max(worst, float(np.abs(got - ref).max()))
        same = same and t2 == int(np.argmax(ref))
        e.ep_finalize()
        results[rank] = (worst, same)
    finally:
        if e is not None:
            e.close()
        dist.destroy_process_group()


def test_ep_prefill_matches_single_gpu(synth_model, cuda_lib):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(worker, args=(port, synth_model, results), nprocs=2, join=True)
    for rank in (0, 1):
        worst, same = results[rank]
        assert worst <= 1e-3 and same, (rank, worst, same)


def test_ep_group_of_one_matches_local_path(synth_model, cuda_lib):
    """A group of one GPU runs the whole exchange (plan, pack, NCCL transfers
    to itself, grouped GEMMs on the received slots, unpack, combine): the
    result must equal the plain prompt path's."""
    import lfm2_b200
    e = lfm2_b200.GpuEngine(synth_model, 0)
    try:
        e.set_ctx(512)
        e.ep_init(lfm2_b200.ep_unique_id(), 0, 1)
        rng = np.random.default_rng(77)
        errs = {}
        for n in (2, 9, 130):
            p = rng.integers(0, 128000, n).astype(np.uint32)
            e.reset_session()
            ref = e.forward(p, 0)
            t = e.ep_prefill(p)
            got = e.snapshot_resident_logits()
            errs[n] = (float(np.abs(got - ref).max()), t == int(np.argmax(ref)))
        e.ep_finalize()
        # the plain path runs the last layer's FFN with the decode kernels (f32
        # activations), the expert-parallel path with the prompt GEMMs (hi/lo)
        assert all(v[0] <= 1e-3 and v[1] for v in errs.values()), errs
    finally:
        e.close()
