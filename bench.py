#!/usr/bin/env python
"""Benchmark of the LFM2.5-8B-A1B Q6_K token loop on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: the seeded synthetic model, a 512-token seeded
prompt, then greedy batch-1 decode. A step is one decode token. `value` is
decode tok/s over all ranks with everything resident in HBM (CUDA events
around K device-chained steps); `e2e` is the same metric through the
reference-facing call `lfm_forward_token` with host buffers (8-byte token +
position upload and 4-byte argmax download every step). Prefill tok/s at a
3840-token prompt (config 3) and the Q6_K matvec microbench (config 1) are
reported beside it. Multi-GPU runs are independent replicas (one process per
GPU, no data-path collective): scaling "weak".

`--impl reference` times the reference's CPU path on this host's cores: the
reference is Rust and cannot be built here, so its C++ restatement under
oracle/ (every f32 accumulation in the reference's order) is the timed arm.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "lfm2-w9100-rust_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "decode tok/s bs1 @512 ctx; prefill tok/s @3840; % of HBM/tensor roofline"
PROMPT_LEN = 512
PREFILL_LEN = 3840
SEED = 1234
# DRAM bytes (read + write) of one decode step, taken from an ncu capture of
# the same workload (not measured by this run); keyed by decode path, with the
# profile summary that holds the capture.
TRAFFIC: dict = {"persistent-step": (1447.4e6, "profiles/k_step_decode_config2.md")}
DIM, VOCAB = 2048, 128000
N_ATTN, N_CONV, N_DENSE, N_MOE = 6, 18, 2, 22


def q6_bytes(in_dim, out_dim):
    return out_dim * (in_dim // 256) * 210


def decode_bytes_per_token(ctx_len: float) -> dict:
    """Algorithmic HBM bytes of one decode token (config 2): every dense Q6_K
    matrix once, the 4 routed experts of each MoE layer, the tied lm_head, the
    f32 routers, the fp16 K/V read up to ctx_len and the small f32 tensors."""
    attn = q6_bytes(DIM, DIM) * 2 + q6_bytes(DIM, 512) * 2
    conv = q6_bytes(DIM, 3 * DIM) + q6_bytes(DIM, DIM)
    dense = q6_bytes(DIM, 7168) * 2 + q6_bytes(7168, DIM)
    expert = q6_bytes(DIM, 1792) * 2 + q6_bytes(1792, DIM)
    lm_head = q6_bytes(DIM, VOCAB)
    q6 = N_ATTN * attn + N_CONV * conv + N_DENSE * dense + N_MOE * 4 * expert + lm_head
    router = N_MOE * DIM * 32 * 4
    kv = N_ATTN * 2 * 8 * 64 * 2 * ctx_len  # fp16 K and V read
    small = q6_bytes(DIM, 1) + (2 * 24 + 1) * DIM * 4 + N_CONV * (3 * DIM * 4 + 2 * DIM * 4 * 2)
    return {"q6": q6, "router": router, "kv": kv, "small": small, "total": q6 + router + kv + small}


def prefill_flops(n: int) -> float:
    """Algorithmic FLOPs of an n-token prefill (config 3): the Q6_K projections
    of every token (4 routed experts per MoE layer), causal attention, and the
    lm_head for the last token only."""
    mac_tok = (N_ATTN * (DIM * DIM * 2 + DIM * 512 * 2) + N_CONV * (DIM * 3 * DIM + DIM * DIM)
               + N_DENSE * 3 * DIM * 7168 + N_MOE * 4 * 3 * DIM * 1792)
    attn = N_ATTN * 4 * 32 * 64 * (n * (n + 1) / 2)
    return 2.0 * mac_tok * n + attn + 2.0 * DIM * VOCAB


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus: int):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    return ws, rank, local, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()


def reduce_max(pg, v: float) -> float:
    """Max of v over the ranks (the job's time is its slowest rank's)."""
    if pg is None:
        return v
    import torch
    dev = "cpu" if pg.get_backend() == "gloo" else "cuda"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(pg, v: float) -> float:
    if pg is None:
        return v
    import torch
    dev = "cpu" if pg.get_backend() == "gloo" else "cuda"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


def prompt(n: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, VOCAB, n).astype(np.uint32)


def model_path(rank: int, pg) -> str:
    import synth_gguf
    path = synth_gguf.default_model_path(SEED)
    if rank == 0:
        synth_gguf.ensure_gguf(path, SEED)
    barrier(pg)
    return synth_gguf.ensure_gguf(path, SEED)


def microbench(device: int) -> list:
    """Config 1: the Q6_K matvec on the decode shapes, per-launch CUDA events,
    rotating over weight copies larger than L2."""
    import ctypes

    import torch

    import lfm2_b200
    lib = lfm2_b200.lib()
    torch.cuda.set_device(device)
    s = torch.cuda.current_stream()
    out = []
    peak = measured_peaks()["hbm_gbs"]
    # (name, in, out, routed experts): routed rows run lfm_q6k_routed on a
    # 32-expert matrix with 4 selected experts, the decode's q6k_routed
    # (resident_graph.rs:446-495); their bytes count all 4 experts.
    shapes = [("lm_head 2048->128000", 2048, 128000, 0), ("lm_head 2048->65536", 2048, 65536, 0),
              ("attn/conv 2048->2048", 2048, 2048, 0), ("attn k/v 2048->512", 2048, 512, 0),
              ("conv in_proj 2048->6144", 2048, 6144, 0), ("dense gate/up 2048->7168", 2048, 7168, 0),
              ("dense down 7168->2048", 7168, 2048, 0),
              ("routed gate/up 2048->1792 x4 of 32 experts", 2048, 1792, 4),
              ("routed down 1792->2048 x4 of 32 experts", 1792, 2048, 4)]
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(s.cuda_stream)
    for name, ind, outd, routed in shapes:
        mrows = outd * 32 if routed else outd
        nbytes = lib.lfm_q6k_device_bytes(ind, mrows)
        copies = max(2 if routed else 1, int(np.ceil(512e6 / nbytes)))
        g = torch.Generator(device="cuda").manual_seed(1)
        pool = [torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda", generator=g) for _ in range(copies)]
        for w in pool:  # plausible fp16 d values: clear the top exponent bits
            w.view(-1)[-(nbytes // 105):].bitwise_and_(0x3B)
        if routed:
            # 8 disjoint groups of 4 experts, rotated with the copies: each
            # (copy, group) pair recurs only after copies*8 calls (> L2)
            ids = torch.arange(32, dtype=torch.int32, device="cuda").view(8, 4)[torch.tensor([0, 5, 2, 7, 4, 1, 6, 3])]
            ids = ids.contiguous()
            x = torch.randn(4 * ind, device="cuda")
            y = torch.empty(4 * outd, device="cuda")
            xs = ind  # one input row per slot (gate/up: the same row four times)
            cycle = copies * 8

            def call(i):
                return lib.lfm_q6k_routed(P(pool[i % copies]), ind, outd, 32, P(ids[(i // copies) % 8]), P(x), xs,
                                          P(y), st)
        else:
            x = torch.randn(ind, device="cuda")
            y = torch.empty(outd, device="cuda")
            cycle = copies

            def call(i):
                return lib.lfm_q6k_matmul(P(pool[i % copies]), ind, outd, P(x), 1, P(y), st)
        for i in range(3):
            lfm2_b200.ops_check(call(i), name)
        iters = max(20, cycle)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for i in range(iters):
            call(i)
        e1.record(s)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / iters
        k = routed or 1
        alg = k * (q6_bytes(ind, outd) + 4 * outd + 4 * ind)
        out.append({"shape": name, "us_per_call": round(us, 2), "bytes": int(alg), "gb_s": round(alg / us / 1e3, 1),
                    "frac": round(alg / us / 1e3 / peak, 4)})
        del pool
        torch.cuda.empty_cache()
    return out


def prompt_gemm_bench(device: int, n: int, reps: int = 5) -> list:
    """The prompt path's Q6_K GEMMs for an n-token prefill through the
    kernel-level C ABI, with the weight operand expanded to fp16 ahead of time
    (what the engine does at load): activation split + tensor-core GEMM per
    call, CUDA events on the launching stream. Routed rows send each token to
    4 of 32 experts (seeded, uniform); their FLOPs count the 4 n routed rows.
    Random Q6_K bytes with plausible super-block scales; the expert matrices'
    fp16 operands (235 MB) are larger than L2, the dense ones are not."""
    import ctypes

    import torch

    import lfm2_b200
    lib = lfm2_b200.lib()
    torch.cuda.set_device(device)
    s = torch.cuda.current_stream()
    st = ctypes.c_void_p(s.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    peak = measured_peaks()["bf16_tflops"]
    rng = np.random.default_rng(n)
    # routed down first: `ncu -k regex:k_tc_q6x -c 1` on this mode captures it
    shapes = [("routed down 1792->2048, grouped", 1792, 2048, 1), ("routed gate 2048->1792, grouped", 2048, 1792, 4),
              ("conv in_proj 2048->6144", 2048, 6144, 0), ("attn/conv out 2048->2048", 2048, 2048, 0),
              ("dense gate 2048->7168", 2048, 7168, 0), ("dense down 7168->2048", 7168, 2048, 0)]
    out = []
    for name, ind, outd, x_div in shapes:
        mrows = outd * 32 if x_div else outd
        nbytes = lib.lfm_q6k_device_bytes(ind, mrows)
        g = torch.Generator(device="cuda").manual_seed(2)
        w = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda", generator=g)
        w.view(-1)[-(nbytes // 105):].bitwise_and_(0x3B)  # plausible fp16 d values
        w16 = torch.empty((mrows, ind), dtype=torch.float16, device="cuda")
        lfm2_b200.ops_check(lib.lfm_q6k_expand_f16(P(w), ind, mrows, P(w16), st), "expand_f16")
        if x_div:
            ids = torch.from_numpy(np.stack([rng.permutation(32)[:4] for _ in range(n)]).astype(np.int32)).cuda()
            x = torch.randn((n if x_div == 4 else 4 * n) * ind, device="cuda")
            y = torch.empty(4 * n * outd, device="cuda")

            def call():
                return lib.lfm_q6k_prompt_grouped_x16(P(w), P(w16), ind, outd, 32, P(ids), P(x), x_div, n, P(y), st)
            flop = 2.0 * 4 * n * ind * outd
        else:
            x = torch.randn(n * ind, device="cuda")
            y = torch.empty(n * outd, device="cuda")

            def call():
                return lib.lfm_q6k_prompt_gemm_x16(P(w), P(w16), ind, outd, P(x), n, P(y), st)
            flop = 2.0 * n * ind * outd
        lfm2_b200.ops_check(call(), name)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            lfm2_b200.ops_check(call(), name)
        e1.record(s)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / reps
        tf = flop / us / 1e6
        out.append({"shape": name, "tokens": n, "us_per_call": round(us, 1), "tflops": round(tf, 1),
                    "frac_of_bf16_peak": round(tf / peak, 4)})
        del w, w16
        torch.cuda.empty_cache()
    return out


def cpu_baseline(path: str, steps: int, warmup: int, threads: int | None = None, one_core_steps: int = 3) -> dict:
    """The oracle on the host cores: 512-token prefill (untimed setup), `warmup`
    untimed and `steps` timed greedy decode steps at 512+ context on `threads`
    threads; then the first `one_core_steps` of those steps again from the
    same state on ONE thread (the reference's Engine is single-threaded,
    lfm.rs:290-694), whose logits must be bit-identical to the threaded run's;
    and config 0's 16-token prefill timed on both thread counts."""
    import oracle
    oracle.build()
    threads = threads or len(os.sched_getaffinity(0))
    os.environ["OMP_NUM_THREADS"] = str(threads)
    oracle.lib().oracle_set_threads(threads)
    o = oracle.OracleEngine(path, kv_f16=True)
    cores = oracle.lib().oracle_num_threads()
    o.set_ctx(4096)
    p = prompt(PROMPT_LEN, 7)
    t0 = time.perf_counter()
    logits = o.forward(p, 0)
    prefill_s = time.perf_counter() - t0
    pos = PROMPT_LEN
    tok = int(np.argmax(logits))
    for _ in range(warmup):
        tok = int(np.argmax(o.forward(np.array([tok], np.uint32), pos)))
        pos += 1
    o.checkpoint()
    tok0, pos0, kept = tok, pos, []
    t0 = time.perf_counter()
    for i in range(steps):
        lg = o.forward(np.array([tok], np.uint32), pos)
        if i < one_core_steps:
            kept.append(lg.copy())
        tok = int(np.argmax(lg))
        pos += 1
    dt = time.perf_counter() - t0
    # the same steps on one thread, from the same state
    o.rollback()
    oracle.lib().oracle_set_threads(1)
    tok, pos, same = tok0, pos0, True
    n1 = min(one_core_steps, steps)
    t0 = time.perf_counter()
    for i in range(n1):
        lg = o.forward(np.array([tok], np.uint32), pos)
        same = same and np.array_equal(lg.view(np.uint32), kept[i].view(np.uint32))
        tok = int(np.argmax(lg))
        pos += 1
    dt1 = time.perf_counter() - t0
    p16 = prompt(16, 0)
    t0 = time.perf_counter()
    o.forward(p16, 0)
    pf1 = time.perf_counter() - t0
    oracle.lib().oracle_set_threads(threads)
    t0 = time.perf_counter()
    o.forward(p16, 0)
    pfn = time.perf_counter() - t0
    o.close()
    return {"value": round(steps / dt, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{steps} greedy decode tokens after a {PROMPT_LEN}-token prefill (prefill "
                      f"{PROMPT_LEN / prefill_s:.1f} tok/s), synthetic model, f16 K/V, {cores} threads",
            "prefill_tok_s": round(PROMPT_LEN / prefill_s, 2), "nproc": os.cpu_count(),
            "prefill16_tok_s": round(16 / pfn, 2),
            "one_core": {"decode_tok_s": round(n1 / dt1, 4), "steps": n1, "prefill16_tok_s": round(16 / pf1, 3),
                         "bit_identical_to_threaded": bool(same),
                         "sample": f"the first {n1} of the timed decode steps again from the same state on "
                                   "1 thread; a 16-token prompt (config 0 shape) on 1 thread"}}


def workload_config(ws: int) -> dict:
    """`config` of both arms' JSON lines (the same workload)."""
    return {"workload": "config 2: 512-token seeded prompt, greedy bs1 decode", "prompt_len": PROMPT_LEN,
            "ctx": 4096, "parallelism": f"replicas x{ws}",
            "l2": "no flush needed: every step streams ~1.4 GB of weights (> 126 MB L2)"}


def run_reference(args, ws, rank, pg):
    if rank != 0:
        return
    path = model_path(0, None)
    # all the host threads this process may use (torchrun sets OMP_NUM_THREADS=1)
    cb = cpu_baseline(path, args.steps, args.warmup, threads=len(os.sched_getaffinity(0)))
    line = {"metric": METRIC, "value": cb["value"], "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / cb["value"], 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic seeded random-init Q6_K weights of the exact architecture",
            "config": workload_config(args.gpus),
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


SESSIONS, SESSION_GEN = 64, 128
PREFILL_GROUP_TOKENS = 4096


def multi_session(eng, peaks, pg, ws: int, info: dict) -> dict:
    """Config 4 on this GPU: 64 independent sessions with seeded prompt lengths
    uniform in [128, 1024] and seeded token ids, prefilled together in groups
    of about 4096 tokens (lfm_batch_prefill_many), then 128 greedy tokens for
    all of them in batched steps (one token per session per step). Device time per call (CUDA events), max over ranks;
    aggregate = all ranks' tokens / that time. The HBM roofline of a batched
    step counts every weight once (64 tokens x top-4 of 32 experts touch all
    experts) plus each session's K/V read."""
    rng = np.random.default_rng(21)
    lens = rng.integers(128, 1025, SESSIONS)
    prompts = [rng.integers(0, VOCAB, int(n)).astype(np.uint32) for n in lens]
    eng.batch_create(SESSIONS)
    sess = np.arange(SESSIONS, dtype=np.uint32)
    # prompts prefilled together in groups of about PREFILL_GROUP_TOKENS tokens
    # (one pass of the layer stack per group)
    groups, i = [], 0
    while i < SESSIONS:
        j, tot = i, 0
        while j < SESSIONS and (j == i or tot + int(lens[j]) <= PREFILL_GROUP_TOKENS):
            tot += int(lens[j])
            j += 1
        groups.append((i, j))
        i = j
    # warm-up: one prefill, one untimed pass of the same groups (the first use
    # of some code paths in a process cost up to ~10 ms of host time per call)
    # and two batched steps; the timed prefills below start the sessions afresh
    t = eng.batch_prefill(0, prompts[0][:64])
    for i, j in groups:
        eng.batch_prefill_many(sess[i:j], prompts[i:j])
    eng.batch_decode(sess[:1], [t], [64])
    eng.batch_decode(sess, np.ones(SESSIONS, np.uint32), np.zeros(SESSIONS, np.uint32))
    barrier(pg)
    pf_ms, toks = 0.0, []
    w0 = time.perf_counter()
    for i, j in groups:
        toks += list(eng.batch_prefill_many(sess[i:j], prompts[i:j]))
        pf_ms += eng.last_device_ms()
    toks = np.array(toks, np.uint32)
    pos = lens.astype(np.uint32).copy()
    dec_ms = 0.0
    steps = []
    w1 = time.perf_counter()
    for _ in range(SESSION_GEN):
        toks = eng.batch_decode(sess, toks, pos)
        dec_ms += eng.last_device_ms()
        steps.append(toks)
        pos += 1
    w2 = time.perf_counter()
    text = text_stream_rate(steps, sess)
    dec_max = reduce_max(pg, dec_ms)
    pf_max = reduce_max(pg, pf_ms)
    wall_dec = reduce_max(pg, w2 - w1)
    wall_all = reduce_max(pg, w2 - w0)
    gen = ws * SESSIONS * SESSION_GEN
    kv = sum(6 * 2 * 8 * 64 * 2 * (int(n) + SESSION_GEN / 2.0) for n in lens)  # fp16 K+V per step, mean ctx
    step_bytes = info["weight_bytes"] + kv
    step_s = dec_max / 1000.0 / SESSION_GEN
    return {"workload": "config 4: 64 sessions/GPU, prompts U[128,1024], 128 greedy tokens each, batched decode",
            "sessions_per_gpu": SESSIONS, "gen_per_session": SESSION_GEN,
            "decode_tok_s": round(gen / (dec_max / 1000.0), 1),
            "decode_ms_per_step": round(dec_max / SESSION_GEN, 3),
            "prefill_tok_s": round(ws * float(lens.sum()) / (pf_max / 1000.0), 1),
            "e2e_tok_s": round(gen / wall_all, 1), "e2e_decode_tok_s": round(gen / wall_dec, 1),
            "prefill_wall_s": round(reduce_max(pg, w1 - w0), 4), "prefill_device_s": round(pf_max / 1000.0, 4),
            "text_stream": dict(text, vs_decode=round(text["tok_s"] / (gen / (dec_max / 1000.0)), 1)),
            "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                         "achieved": round(step_bytes / step_s / 1e9, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(step_bytes / step_s / 1e9 / peaks["hbm_gbs"], 4)}}


EP_SESSIONS = 8


def ep_compare(eng, pg, ws: int, rank: int) -> dict:
    """Config 4's expert-parallel variant against replicas (N > 1 only):
    EP_SESSIONS prompts per rank (lengths U[128, 1024], seeded per rank) are
    prefilled into session slots twice: as replicas (each rank alone, every
    expert on every GPU) and expert-parallel (rank r computes experts
    r*32/N .. (r+1)*32/N - 1 for the tokens of all ranks; routed rows cross
    NVLink through NCCL point-to-point transfers). Replicas: each rank's
    summed device time, max over ranks; expert-parallel (collective calls):
    the max over ranks of each call, summed. Aggregate tok/s = all ranks'
    prompt tokens / that time. The two paths must give the same logits."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(700 + rank)
    lens = rng.integers(128, 1025, EP_SESSIONS)
    prompts = [rng.integers(0, VOCAB, int(n)).astype(np.uint32) for n in lens]
    idt = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        idt.copy_(torch.from_numpy(np.frombuffer(lfm2_b200.ep_unique_id(), dtype=np.uint8).copy()))
    pg.broadcast(idt, src=0)
    eng.ep_init(idt.cpu().numpy().tobytes(), rank, ws)
    eng.batch_create(EP_SESSIONS)
    # warm-up of both paths
    eng.batch_prefill(0, prompts[0][:128])
    eng.ep_prefill(prompts[0][:128], 0)
    rep_ms, ep_ms, worst, same = 0.0, 0.0, 0.0, True
    for i, p in enumerate(prompts):
        barrier(pg)
        t_rep = eng.batch_prefill(i, p)
        rep_ms += eng.last_device_ms()  # replicas run on their own: this rank's total
        ref = eng.snapshot_resident_logits()
        barrier(pg)
        t_ep = eng.ep_prefill(p, i)
        ep_ms += reduce_max(pg, eng.last_device_ms())
        got = eng.snapshot_resident_logits()
        worst = max(worst, float(np.abs(got - ref).max()))
        same = same and t_rep == t_ep
    rep_ms = reduce_max(pg, rep_ms)
    worst = reduce_max(pg, worst)
    same = reduce_max(pg, 0.0 if same else 1.0) == 0.0
    eng.ep_finalize()
    tok = reduce_sum(pg, float(lens.sum()))
    return {"workload": f"config 4 expert-parallel prefill: {EP_SESSIONS} prompts/rank U[128,1024]",
            "replica_tok_s": round(tok / (rep_ms / 1000.0), 1), "ep_tok_s": round(tok / (ep_ms / 1000.0), 1),
            "replica_ms": round(rep_ms, 2), "ep_ms": round(ep_ms, 2), "logits_max_abs_diff": worst,
            "next_tokens_equal": same, "kept": "ep" if ep_ms < rep_ms else "replicas"}


def text_stream_rate(steps, sess) -> dict:
    """The host text path of the batched decode (lfm_text_push: UTF-8
    assembly + the decoder's space cleanup per session, as the reference's
    StreamDecoder + DecodedText) over the tokens the batched steps produced,
    one push per step, timed on one host thread after the GPU work. Pieces of
    the synthetic vocabulary: the 16 control tokens render empty, the others
    are their own ASCII text."""
    import lfm2_b200
    pieces = [b"" if i < 16 else b" t%06d" % i for i in range(VOCAB)]
    t = lfm2_b200.TextStreams(pieces, len(sess), clean_spaces=True, replace_invalid=True)
    n = 0
    t0 = time.perf_counter()
    for toks in steps:
        t.push(sess, toks)
        n += len(toks)
    for s_ in sess:
        t.finish(int(s_))
    dt = time.perf_counter() - t0
    t.close()
    return {"tok_s": round(n / dt, 1), "threads": 1, "tokens": n,
            "path": "lfm_text_push (UTF-8 assembly + clean_spaces per session)"}


def prefill_only(local: int, n: int) -> dict:
    """One warm-up and one timed n-token prefill on GPU `local` (device time
    of the engine's prefill, CUDA events on its stream)."""
    import torch

    import lfm2_b200
    torch.cuda.set_device(local)
    eng = lfm2_b200.GpuEngine(model_path(0, None), local)
    eng.set_ctx(max(4096, n))
    p = prompt(n, 11)
    eng.reset_session()
    eng.forward(p, 0)
    eng.reset_session()
    logits = eng.forward(p, 0)
    ms = eng.last_device_ms()
    out = {"prefill_only": n, "ms": round(ms, 3), "tok_s": round(n / (ms / 1000), 1),
           "argmax": int(np.argmax(logits)), "path": eng.info().get("prefill_path", "")}
    eng.close()
    return out


def step_trace(local: int, n: int) -> dict:
    """Stage timeline of the persistent decode step (profiling entry point):
    an n-token prompt, 16 untimed decode steps, then one traced step of 8.
    Per stage type: count, span per stage (first start to last arrival), the
    median CTA's work, its staging prologue and wait for the first tile, the
    grid-barrier gap before the stage; per tile: consumer warp 0's wait and
    compute cycles. All times in microseconds."""
    import torch

    import lfm2_b200
    torch.cuda.set_device(local)
    eng = lfm2_b200.GpuEngine(model_path(0, None), local)
    eng.set_ctx(4096)
    p = prompt(n, 7)
    first = int(np.argmax(eng.forward(p, 0)))
    _, ms = eng.decode_loop(first, n, 16)
    eng.step_trace(True)
    eng.decode_loop(first, n, 8)
    tr = eng.step_trace(False)
    eng.close()
    if tr is None:
        return {"step_trace": "kernel chain decode path: no stage trace"}
    import synth_gguf
    types = ["EMBED"]
    for layer in range(24):
        types += ["QKV", "ATTN", "RESID"] if layer in synth_gguf.ATTN_LAYERS else ["CONV", "RESID"]
        types += ["SWIGLU", "DOWN28"] if layer < 2 else ["XSWIGLU", "XDOWN"]
    types.append("LMHEAD")
    tr = tr.astype(np.int64)
    ns, nc, _ = tr.shape
    if len(types) != ns:
        return {"step_trace": f"unexpected stage count {ns}"}
    t0 = tr[0, :, 0].min()
    start, staged, first_tile, done = (tr[:, :, i] - t0 for i in range(4))
    agg, prev_end = {}, 0
    for s_ in range(ns):
        a = agg.setdefault(types[s_], {"count": 0, "span": 0.0, "work": 0.0, "prologue": 0.0, "first_tile": 0.0,
                                       "gap": 0.0, "tiles": 0, "wait_cyc": 0, "compute_cyc": 0})
        a["count"] += 1
        a["span"] += (done[s_].max() - start[s_].min()) / 1e3
        a["work"] += float(np.median(done[s_] - start[s_])) / 1e3
        a["gap"] += (start[s_].min() - prev_end) / 1e3
        prev_end = done[s_].max()
        ok = tr[s_, :, 1] > 0
        if ok.any():
            a["prologue"] += float(np.median((staged[s_] - start[s_])[ok])) / 1e3
            ok2 = tr[s_, :, 2] > 0
            if ok2.any():
                a["first_tile"] += float(np.median((first_tile[s_] - staged[s_])[ok2])) / 1e3
        a["tiles"] += int(tr[s_, :, 5].sum())
        a["wait_cyc"] += int(tr[s_, :, 4].sum())
        a["compute_cyc"] += int(tr[s_, :, 6].sum())
    table = {}
    for k, a in sorted(agg.items(), key=lambda kv: -kv[1]["span"]):
        c = a["count"]
        row = {"count": c, "span_us": round(a["span"], 1), "per_stage_us": round(a["span"] / c, 2),
               "work_us": round(a["work"] / c, 2), "prologue_us": round(a["prologue"] / c, 2),
               "first_tile_us": round(a["first_tile"] / c, 2), "gap_us": round(a["gap"] / c, 2)}
        if a["tiles"]:
            row["tile_wait_cyc"] = round(a["wait_cyc"] / a["tiles"])
            row["tile_compute_cyc"] = round(a["compute_cyc"] / a["tiles"])
            row["tiles_per_cta"] = round(a["tiles"] / (c * nc), 1)
        table[k] = row
    return {"step_trace": {"prompt_len": n, "untraced_ms_per_step": round(ms / 15, 4),
                           "traced_step_us": round(float(done.max()) / 1e3, 1), "ctas": int(nc), "stages": table}}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-micro", action="store_true")
    ap.add_argument("--micro-only", action="store_true", help="only the config-1 Q6_K matvec microbench")
    ap.add_argument("--no-sessions", action="store_true", help="skip config 4 (64 independent sessions per GPU)")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel prefill comparison (N > 1)")
    ap.add_argument("--sessions-only", action="store_true", help="only config 4 on this GPU (profiling entry point)")
    ap.add_argument("--prefill-only", type=int, default=0, metavar="N",
                    help="only one warm-up and one timed N-token prefill (profiling entry point)")
    ap.add_argument("--prompt-gemm", type=int, default=0, metavar="N",
                    help="only the prompt GEMMs of an N-token prefill through the C ABI (profiling entry point)")
    ap.add_argument("--step-trace", type=int, default=0, metavar="N",
                    help="only the decode step's stage timeline after an N-token prompt (profiling entry point)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    ws, rank, local, pg = dist_setup(args.gpus)
    if args.micro_only:
        if rank == 0:
            print(json.dumps({"microbench": microbench(local)}), flush=True)
        return
    if args.prefill_only:
        if rank == 0:
            print(json.dumps(prefill_only(local, args.prefill_only)), flush=True)
        return
    if args.prompt_gemm:
        if rank == 0:
            print(json.dumps({"prompt_gemm": prompt_gemm_bench(local, args.prompt_gemm)}), flush=True)
        return
    if args.step_trace:
        if rank == 0:
            print(json.dumps(step_trace(local, args.step_trace)), flush=True)
        return
    if args.sessions_only:
        if rank == 0:
            import torch

            import lfm2_b200
            torch.cuda.set_device(local)
            eng = lfm2_b200.GpuEngine(model_path(0, None), local)
            eng.set_ctx(4096)
            print(json.dumps(multi_session(eng, measured_peaks(), None, 1, eng.info())), flush=True)
            eng.close()
        return
    if args.impl == "reference":
        run_reference(args, ws, rank, pg)
        if pg is not None:
            pg.destroy_process_group()
        return

    import torch

    import lfm2_b200
    torch.cuda.set_device(local)
    path = model_path(rank, pg)
    peaks = measured_peaks()
    eng = lfm2_b200.GpuEngine(path, local)
    eng.set_ctx(4096)
    p512 = prompt(PROMPT_LEN, 7)

    def prefill512():
        eng.reset_session()
        return int(np.argmax(eng.forward(p512, 0)))

    # warm-up (graph capture, first-touch)
    first = prefill512()
    eng.decode_loop(first, PROMPT_LEN, args.warmup)
    first = prefill512()
    c0 = eng.counters()
    barrier(pg)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        toks, dev_ms = eng.decode_loop(first, PROMPT_LEN, args.steps + 1)
    torch.cuda.synchronize()
    c1 = eng.counters()
    timed_ms = reduce_max(pg, dev_ms)
    value = ws * args.steps / (timed_ms / 1000.0)
    per_gpu = args.steps / (dev_ms / 1000.0)
    ms_per_step = timed_ms / args.steps
    launches = int(c1["kernel_launches"] - c0["kernel_launches"])
    launches = int(launches * args.steps / (args.steps + 1))

    # e2e through the reference-facing call (host buffers, per-step H2D/D2H)
    first = prefill512()
    t = first
    pos = PROMPT_LEN
    for _ in range(args.warmup):
        t = eng.forward_token(np.array([t], np.uint32), pos)
        pos += 1
    first = prefill512()
    barrier(pg)
    t, pos = first, PROMPT_LEN
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t = eng.forward_token(np.array([t], np.uint32), pos)
        pos += 1
    e2e_s = reduce_max(pg, time.perf_counter() - t0)
    e2e = {"value": round(ws * args.steps / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": 4, "call": "lfm_forward_token (api_stream decode loop)"}

    avg_ctx = PROMPT_LEN + 1 + (args.steps + 1) / 2.0
    bpt = decode_bytes_per_token(avg_ctx)
    achieved = bpt["total"] * per_gpu / 1e9
    info = eng.info()
    path_name = info["decode_path"]
    kernel = ("k_step: one persistent cooperative kernel per decode token" if path_name == "persistent-step"
              else f"decode step as a CUDA graph of {info['launches_per_decode']} kernels")
    traffic, traffic_src = TRAFFIC.get(path_name, (None, None))
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                "traffic_source": traffic_src and f"ncu capture summarised in {traffic_src}, not measured by this run",
                "kernel": kernel, "bytes_per_step": int(bpt["total"]),
                "peak_source": peaks["source"]}

    prefill = None
    if not args.no_prefill:
        p3840 = prompt(PREFILL_LEN, 11)
        eng.reset_session()
        eng.forward(p3840, 0)  # warm
        barrier(pg)
        eng.reset_session()
        eng.forward(p3840, 0)
        pms = reduce_max(pg, eng.last_device_ms())
        fl = prefill_flops(PREFILL_LEN)
        # config 3 continues with 256 greedy tokens up to the 4096-token limit
        first = int(np.argmax(eng.snapshot_resident_logits()))
        n_long = 4096 - PREFILL_LEN - 1
        _, lms = eng.decode_loop(first, PREFILL_LEN, n_long)
        lms = reduce_max(pg, lms)
        long_bpt = decode_bytes_per_token(PREFILL_LEN + n_long / 2.0)["total"]
        prefill = {"prompt_len": PREFILL_LEN, "tok_s": round(ws * PREFILL_LEN / (pms / 1000), 1),
                   "ms": round(pms, 2), "tflops": round(fl / (pms / 1000) / 1e12, 2),
                   "frac_of_bf16_peak": round(fl / (pms / 1000) / 1e12 / peaks["bf16_tflops"], 4),
                   "path": info.get("prefill_path", ""),
                   "decode_after": {"tokens": n_long, "ctx": f"{PREFILL_LEN}..4095",
                                    "tok_s": round(ws * (n_long - 1) / (lms / 1000), 1),
                                    "hbm_frac": round(long_bpt * (n_long - 1) / (lms / 1000) / 1e9 / peaks["hbm_gbs"], 4)}}
    multi = None
    if not args.no_sessions:
        multi = multi_session(eng, peaks, pg, ws, info)
    ep = None
    if ws > 1 and not args.no_ep:
        ep = ep_compare(eng, pg, ws, rank)
    micro = pgemm = None
    if rank == 0 and not args.no_micro:
        micro = microbench(local)
        pgemm = prompt_gemm_bench(local, PREFILL_LEN)
    cpu = None
    eng.close()  # release the device before the CPU leg and before interpreter teardown
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_baseline(path, 16, 2, threads=len(os.sched_getaffinity(0)))
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic seeded random-init Q6_K weights of the exact architecture",
                "config": workload_config(ws), "decode_path": path_name,
                "roofline": roofline, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk.summary(), "prefill": prefill, "multi_session": multi, "expert_parallel_prefill": ep,
                "microbench": micro, "prompt_gemm_microbench": pgemm, "cpu_baseline": cpu,
                "tokens_head": toks[:8]}
        print(json.dumps(line), flush=True)
    if pg is not None:
        barrier(pg)
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
