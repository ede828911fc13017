"""Seeded synthetic LFM2.5-8B-A1B Q6_K GGUF writer.

The reference repository ships no model weights, so parity and benchmarks run
on a random-init model with the exact tensor set, names, shapes and GGML types
that the reference loader expects:

* geometry is the reference's hard-coded one (engine/src/lfm.rs:21-29 and the
  checks in `load_hyperparams`, engine/src/lfm.rs:102-145): 24 layers, dim 2048,
  32 query heads, 8 KV heads, head_dim 64, vocab 128000, 32 experts, top-4,
  expert_ff 1792, dense n_ff 7168, 2 leading dense layers, conv L_cache 3;
* which layers are attention comes only from the per-layer
  `lfm2moe.attention.head_count_kv` array (engine/src/lfm.rs:106, 327);
* the file is GGUF v3 as validated by parser/src/gguf.rs:304-440 (arrays are
  stored as (element type, count), general.alignment = 32);
* tokenizer metadata is present because even `lfm2-greedy --cpu --tokens`
  loads the tokenizer first (engine/src/main.rs:164) and range-checks ids
  against it (tokenizer/src/vocab.rs:253-335): model "gpt2", pre "lfm2",
  128000 unique token strings and a merges string array.

Value distributions (recorded in the file under `synthetic.*` keys):
Q6_K ql/qh uniform random bytes, int8 scales uniform in [-32, 31],
d = fp16(|N(0, 2e-4)|); norm weights F32 ~ N(1, 0.02); router
`ffn_gate_inp.weight` F32 ~ N(0, 0.02); `exp_probs_b.bias` F32 ~ N(0, 0.01);
`shortconv.conv.weight` F32 ~ N(0, 0.3).

Every tensor draws from its own PCG64 stream derived from (seed, tensor index),
so the bytes depend only on the seed.
"""

from __future__ import annotations

import argparse
import os
import struct
import sys
from concurrent.futures import ThreadPoolExecutor

import numpy as np

DIM = 2048
HEADS = 32
HEAD_DIM = 64
KV_HEADS = 8
N_LAYERS = 24
VOCAB = 128000
N_EXPERT = 32
N_USED = 4
EXPERT_FF = 1792
N_FF = 7168
DENSE_LEAD = 2
CONV_L = 3
EPS = 1e-5
ROPE_THETA = 1e6
EOS_ID = 7
BOS_ID = 1
# Attention layer indices; the reference does not hard-code them (they come
# from head_count_kv), these follow the public LFM2-8B-A1B layer pattern.
ATTN_LAYERS = (2, 6, 10, 14, 18, 21)

GGML_F32 = 0
GGML_Q6_K = 14
QK_K = 256
Q6_BYTES = 210
ALIGN = 32

# GGUF metadata value types (parser/src/gguf.rs:223-265)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)


def tensor_plan(attn_layers=ATTN_LAYERS):
    """List of (name, ggml_type, ne, kind) in file order. `ne[0]` is fastest."""
    plan = [
        ("token_embd.weight", GGML_Q6_K, (DIM, VOCAB), "q6"),
        ("token_embd_norm.weight", GGML_F32, (DIM,), "norm"),
    ]
    for l in range(N_LAYERS):
        p = f"blk.{l}."
        plan.append((p + "attn_norm.weight", GGML_F32, (DIM,), "norm"))
        if l in attn_layers:
            plan += [
                (p + "attn_q.weight", GGML_Q6_K, (DIM, DIM), "q6"),
                (p + "attn_k.weight", GGML_Q6_K, (DIM, HEAD_DIM * KV_HEADS), "q6"),
                (p + "attn_v.weight", GGML_Q6_K, (DIM, HEAD_DIM * KV_HEADS), "q6"),
                (p + "attn_output.weight", GGML_Q6_K, (DIM, DIM), "q6"),
                (p + "attn_q_norm.weight", GGML_F32, (HEAD_DIM,), "norm"),
                (p + "attn_k_norm.weight", GGML_F32, (HEAD_DIM,), "norm"),
            ]
        else:
            plan += [
                (p + "shortconv.in_proj.weight", GGML_Q6_K, (DIM, 3 * DIM), "q6"),
                (p + "shortconv.out_proj.weight", GGML_Q6_K, (DIM, DIM), "q6"),
                (p + "shortconv.conv.weight", GGML_F32, (CONV_L, DIM), "conv"),
            ]
        plan.append((p + "ffn_norm.weight", GGML_F32, (DIM,), "norm"))
        if l < DENSE_LEAD:
            plan += [
                (p + "ffn_gate.weight", GGML_Q6_K, (DIM, N_FF), "q6"),
                (p + "ffn_up.weight", GGML_Q6_K, (DIM, N_FF), "q6"),
                (p + "ffn_down.weight", GGML_Q6_K, (N_FF, DIM), "q6"),
            ]
        else:
            plan += [
                (p + "ffn_gate_inp.weight", GGML_F32, (DIM, N_EXPERT), "router"),
                (p + "exp_probs_b.bias", GGML_F32, (N_EXPERT,), "bias"),
                (p + "ffn_gate_exps.weight", GGML_Q6_K, (DIM, EXPERT_FF, N_EXPERT), "q6"),
                (p + "ffn_up_exps.weight", GGML_Q6_K, (DIM, EXPERT_FF, N_EXPERT), "q6"),
                (p + "ffn_down_exps.weight", GGML_Q6_K, (EXPERT_FF, DIM, N_EXPERT), "q6"),
            ]
    return plan


def nbytes_of(gtype, ne):
    n = int(np.prod(ne))
    if gtype == GGML_F32:
        return 4 * n
    assert n % QK_K == 0
    return n // QK_K * Q6_BYTES


def random_q6k_blocks(rng: np.random.Generator, nblocks: int) -> np.ndarray:
    """`nblocks` Q6_K super-blocks (210 B each) with the synthetic distribution."""
    raw = np.frombuffer(rng.bytes(nblocks * Q6_BYTES), dtype=np.uint8).copy()
    blk = raw.reshape(nblocks, Q6_BYTES)
    blk[:, 192:208] = rng.integers(-32, 32, size=(nblocks, 16), dtype=np.int8).view(np.uint8)
    d = np.abs(rng.normal(0.0, 2e-4, size=nblocks)).astype(np.float16)
    blk[:, 208:210] = d.view(np.uint8).reshape(nblocks, 2)
    return raw


def tensor_bytes(seed: int, index: int, kind: str, gtype: int, ne) -> bytes:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))
    n = int(np.prod(ne))
    if gtype == GGML_Q6_K:
        return random_q6k_blocks(rng, n // QK_K).tobytes()
    if kind == "norm":
        v = rng.normal(1.0, 0.02, size=n)
    elif kind == "router":
        v = rng.normal(0.0, 0.02, size=n)
    elif kind == "bias":
        v = rng.normal(0.0, 0.01, size=n)
    elif kind == "conv":
        v = rng.normal(0.0, 0.3, size=n)
    else:
        raise ValueError(kind)
    return v.astype("<f4").tobytes()


class _KV:
    def __init__(self):
        self.items = []

    def _key(self, k):
        b = k.encode()
        return struct.pack("<Q", len(b)) + b

    def u32(self, k, v):
        self.items.append(self._key(k) + struct.pack("<II", T_U32, v))

    def f32(self, k, v):
        self.items.append(self._key(k) + struct.pack("<If", T_F32, v))

    def u64(self, k, v):
        self.items.append(self._key(k) + struct.pack("<IQ", T_U64, v))

    def string(self, k, v):
        b = v.encode()
        self.items.append(self._key(k) + struct.pack("<IQ", T_STR, len(b)) + b)

    def arr_u32(self, k, vals):
        self.items.append(self._key(k) + struct.pack("<IIQ", T_ARR, T_U32, len(vals))
                          + struct.pack(f"<{len(vals)}I", *vals))

    def arr_i32(self, k, vals):
        self.items.append(self._key(k) + struct.pack("<IIQ", T_ARR, T_I32, len(vals))
                          + np.asarray(vals, dtype="<i4").tobytes())

    def arr_str(self, k, vals):
        parts = [self._key(k), struct.pack("<IIQ", T_ARR, T_STR, len(vals))]
        for s in vals:
            b = s.encode()
            parts.append(struct.pack("<Q", len(b)) + b)
        self.items.append(b"".join(parts))


def metadata(seed: int, attn_layers):
    kv = _KV()
    kv.string("general.architecture", "lfm2moe")
    kv.string("general.name", "LFM2.5-8B-A1B synthetic Q6_K")
    kv.u32("general.alignment", ALIGN)
    kv.u32("lfm2moe.block_count", N_LAYERS)
    kv.u32("lfm2moe.context_length", 128000)
    kv.u32("lfm2moe.embedding_length", DIM)
    kv.u32("lfm2moe.feed_forward_length", N_FF)
    kv.u32("lfm2moe.attention.head_count", HEADS)
    kv.arr_u32("lfm2moe.attention.head_count_kv",
               [KV_HEADS if l in attn_layers else 0 for l in range(N_LAYERS)])
    kv.f32("lfm2moe.rope.freq_base", ROPE_THETA)
    kv.f32("lfm2moe.attention.layer_norm_rms_epsilon", EPS)
    kv.u32("lfm2moe.vocab_size", VOCAB)
    kv.u32("lfm2moe.shortconv.l_cache", CONV_L)
    kv.u32("lfm2moe.expert_count", N_EXPERT)
    kv.u32("lfm2moe.expert_used_count", N_USED)
    kv.u32("lfm2moe.expert_feed_forward_length", EXPERT_FF)
    kv.u32("lfm2moe.leading_dense_block_count", DENSE_LEAD)
    kv.string("tokenizer.ggml.model", "gpt2")
    kv.string("tokenizer.ggml.pre", "lfm2")
    toks = [f"<|syn_{i}|>" if i < 16 else f"t{i:06d}" for i in range(VOCAB)]
    kv.arr_str("tokenizer.ggml.tokens", toks)
    kv.arr_i32("tokenizer.ggml.token_type", [3 if i < 16 else 1 for i in range(VOCAB)])
    kv.arr_str("tokenizer.ggml.merges", ["t 0", "t 1", "t0 0"])
    kv.u32("tokenizer.ggml.bos_token_id", BOS_ID)
    kv.u32("tokenizer.ggml.eos_token_id", EOS_ID)
    kv.u64("synthetic.seed", seed)
    kv.string("synthetic.distribution",
              "q6k: ql/qh uniform bytes, scales int8 U[-32,31], d=fp16(|N(0,2e-4)|); "
              "norms N(1,0.02); router N(0,0.02); bias N(0,0.01); conv N(0,0.3)")
    return kv.items


def write_gguf(path: str, seed: int = 1234, attn_layers=ATTN_LAYERS, threads: int = 8) -> str:
    """Write the synthetic model to `path` (atomically) and return the path."""
    plan = tensor_plan(attn_layers)
    kvs = metadata(seed, attn_layers)
    header = [b"GGUF", struct.pack("<IQQ", 3, len(plan), len(kvs))] + kvs
    offset = 0
    offsets = []
    for name, gtype, ne, _ in plan:
        b = name.encode()
        header.append(struct.pack("<Q", len(b)) + b + struct.pack("<I", len(ne))
                      + struct.pack(f"<{len(ne)}Q", *ne) + struct.pack("<IQ", gtype, offset))
        offsets.append(offset)
        offset += nbytes_of(gtype, ne)
        offset = (offset + ALIGN - 1) // ALIGN * ALIGN
    head = b"".join(header)
    data_offset = (len(head) + ALIGN - 1) // ALIGN * ALIGN
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_offset - len(head)))
        pool = ThreadPoolExecutor(max_workers=threads)
        futs = [pool.submit(tensor_bytes, seed, i, kind, gtype, ne)
                for i, (name, gtype, ne, kind) in enumerate(plan)]
        pos = 0
        for i, fut in enumerate(futs):
            data = fut.result()
            futs[i] = None
            assert pos <= offsets[i]
            f.write(b"\0" * (offsets[i] - pos))
            f.write(data)
            pos = offsets[i] + len(data)
        pool.shutdown()
    os.replace(tmp, path)
    return path


def ensure_gguf(path: str, seed: int = 1234) -> str:
    """Create the synthetic model at `path` unless a file of the right size exists."""
    plan = tensor_plan()
    if os.path.exists(path):
        expect = sum(nbytes_of(g, ne) for _, g, ne, _ in plan)
        if os.path.getsize(path) > expect:
            return path
    return write_gguf(path, seed)


def default_model_path(seed: int = 1234) -> str:
    root = os.environ.get("LFM_SYNTH_DIR", "/tmp/lfm2_b200_synth")
    return os.path.join(root, f"lfm2-synth-s{seed}.gguf")


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", default=None)
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args()
    out = a.out or default_model_path(a.seed)
    import time
    t = time.time()
    write_gguf(out, a.seed)
    print(f"wrote {out} ({os.path.getsize(out) / 1e9:.3f} GB) in {time.time() - t:.1f}s", file=sys.stderr)
