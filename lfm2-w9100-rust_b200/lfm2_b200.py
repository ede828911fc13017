"""Python binding of liblfm2_b200.so (include/lfm_cuda.h) through ctypes.

`GpuEngine` mirrors the reference's `lfm2_engine::gpu_lfm::GpuEngine`
(engine/src/gpu_lfm.rs:23-245, engine/src/gpu_lfm/resident_graph.rs:90-602):
load, set_ctx, forward (full logits), forward_token (device argmax),
reset_session, snapshot/restore of the resident cache, snapshot of the last
logits. There is no CPU fallback: if the CUDA library cannot be loaded, every
call raises.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblfm2_b200.so")

VOCAB = 128000
PREFILL_CHUNK = 64  # engine/src/work_bound.rs:6


class LfmError(RuntimeError):
    pass


class Hparams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("dim", "heads", "head_dim", "n_layers", "vocab", "n_expert", "n_used", "expert_ff",
                 "n_ff", "dense_lead", "conv_l_cache", "eos")] + \
               [("eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("kv_heads", ctypes.c_uint32 * 64)]


class Counters(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("kernel_launches", "gpu_argmax", "graph_replays", "graph_captures", "prefill_tokens",
                 "expert_grouped_launches")]


_lib = None

# Every symbol declared in include/lfm_cuda.h.
EXPORTS = [
    "lfm_model_inspect", "lfm_engine_create", "lfm_engine_destroy", "lfm_engine_set_ctx", "lfm_hparams_get",
    "lfm_forward_logits", "lfm_forward_token", "lfm_generate", "lfm_decode_loop", "lfm_last_device_ms",
    "lfm_batch_create", "lfm_batch_prefill", "lfm_batch_prefill_many", "lfm_batch_decode", "lfm_batch_logits",
    "lfm_ep_unique_id", "lfm_ep_init", "lfm_ep_prefill", "lfm_ep_plan", "lfm_ep_finalize",
    "lfm_step_trace", "lfm_engine_info",
    "lfm_reset_session",
    "lfm_snapshot_cache", "lfm_restore_cache", "lfm_snapshot_logits", "lfm_counters_get",
    "lfm_device_name", "lfm_last_error", "lfm_global_error", "lfm_q6k_device_bytes",
    "lfm_q6k_upload", "lfm_q6k_dequant", "lfm_q6k_matmul", "lfm_q6k_routed", "lfm_route",
    "lfm_argmax", "lfm_argmax_noalloc", "lfm_tc_gemm_f16", "lfm_tc_gemm_f16_bmn", "lfm_attention_prefill", "lfm_selftest_wait_timeout", "lfm_q6k_prompt_gemm", "lfm_q6k_prompt_grouped",
    "lfm_q6k_expand_f16", "lfm_q6k_prompt_gemm_x16", "lfm_q6k_prompt_grouped_x16",
    "lfm_ops_error",
    "lfm_text_create", "lfm_text_destroy", "lfm_text_push", "lfm_text_finish", "lfm_text_reset", "lfm_text_error",
]


def lib() -> ctypes.CDLL:
    """Load the CUDA library (fails loudly if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LfmError(f"{LIB_PATH} is missing: run lfm2-w9100-rust_b200/build.py (no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, U32, I64, SZ = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int64, ctypes.c_size_t
    st = ctypes.c_int32
    sig = {
        "lfm_model_inspect": ([ctypes.c_char_p, ctypes.POINTER(Hparams)], st),
        "lfm_engine_create": ([ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(P)], st),
        "lfm_engine_destroy": ([P], None),
        "lfm_engine_set_ctx": ([P, U32], st),
        "lfm_hparams_get": ([P, ctypes.POINTER(Hparams)], st),
        "lfm_forward_logits": ([P, P, U32, I64, P], st),
        "lfm_forward_token": ([P, P, U32, U32, ctypes.POINTER(U32)], st),
        "lfm_generate": ([P, P, U32, U32, U32, P, ctypes.POINTER(U32)], st),
        "lfm_decode_loop": ([P, U32, U32, U32, P, ctypes.POINTER(ctypes.c_float)], st),
        "lfm_last_device_ms": ([P], ctypes.c_float),
        "lfm_batch_create": ([P, U32], st),
        "lfm_batch_prefill": ([P, U32, P, U32, ctypes.POINTER(U32)], st),
        "lfm_batch_prefill_many": ([P, P, P, P, U32, P], st),
        "lfm_batch_decode": ([P, P, P, P, U32, P], st),
        "lfm_batch_logits": ([P, U32, P], st),
        "lfm_ep_unique_id": ([P], st),
        "lfm_ep_init": ([P, P, ctypes.c_int, ctypes.c_int], st),
        "lfm_ep_prefill": ([P, U32, P, U32, ctypes.POINTER(U32)], st),
        "lfm_ep_plan": ([P, U32, U32, P, P], st),
        "lfm_ep_finalize": ([P], st),
        "lfm_step_trace": ([P, ctypes.c_int, P, SZ, ctypes.POINTER(U32), ctypes.POINTER(U32)], st),
        "lfm_engine_info": ([P], ctypes.c_char_p),
        "lfm_reset_session": ([P], st),
        "lfm_snapshot_cache": ([P, U32, P, SZ, ctypes.POINTER(SZ)], st),
        "lfm_restore_cache": ([P, U32, P, SZ], st),
        "lfm_snapshot_logits": ([P, P], st),
        "lfm_counters_get": ([P, ctypes.POINTER(Counters)], st),
        "lfm_device_name": ([P], ctypes.c_char_p),
        "lfm_last_error": ([P], ctypes.c_char_p),
        "lfm_global_error": ([], ctypes.c_char_p),
        "lfm_q6k_device_bytes": ([U32, U32], SZ),
        "lfm_q6k_upload": ([P, U32, U32, P], st),
        "lfm_q6k_dequant": ([P, U32, U32, U32, U32, P, P], st),
        "lfm_q6k_matmul": ([P, U32, U32, P, U32, P, P], st),
        "lfm_q6k_routed": ([P, U32, U32, U32, P, P, U32, P, P], st),
        "lfm_route": ([P, P, U32, U32, P, P, P], st),
        "lfm_argmax": ([P, U32, P, P], st),
        "lfm_argmax_noalloc": ([P, U32, P, P], st),
        "lfm_tc_gemm_f16": ([P, P, U32, U32, U32, P, P], st),
        "lfm_tc_gemm_f16_bmn": ([P, P, U32, U32, P, P], st),
        "lfm_attention_prefill": ([P, U32, P, P, U32, U32, U32, P, U32, P], st),
        "lfm_selftest_wait_timeout": ([ctypes.POINTER(U32), ctypes.POINTER(ctypes.c_uint64)], st),
        "lfm_q6k_prompt_gemm": ([P, U32, U32, P, U32, P, P], st),
        "lfm_q6k_prompt_grouped": ([P, U32, U32, U32, P, P, U32, U32, P, P], st),
        "lfm_q6k_expand_f16": ([P, U32, U32, P, P], st),
        "lfm_q6k_prompt_gemm_x16": ([P, P, U32, U32, P, U32, P, P], st),
        "lfm_q6k_prompt_grouped_x16": ([P, P, U32, U32, U32, P, P, U32, U32, P, P], st),
        "lfm_ops_error": ([], ctypes.c_char_p),
        "lfm_text_create": ([P, P, U32, U32, ctypes.c_int, ctypes.c_int, ctypes.POINTER(P)], st),
        "lfm_text_destroy": ([P], None),
        "lfm_text_push": ([P, P, P, U32, P, SZ, P], st),
        "lfm_text_finish": ([P, U32, P, SZ, ctypes.POINTER(SZ)], st),
        "lfm_text_reset": ([P, U32], st),
        "lfm_text_error": ([], ctypes.c_char_p),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def ep_unique_id() -> bytes:
    """A fresh NCCL id for lfm_ep_init (rank 0 creates it, every rank uses it)."""
    buf = np.zeros(128, dtype=np.uint8)
    st = lib().lfm_ep_unique_id(_p(buf))
    if st != 0:
        raise LfmError(f"lfm_ep_unique_id: {lib().lfm_global_error().decode()} (status {st})")
    return buf.tobytes()


def ep_plan(sel, world: int):
    """The expert-parallel send plan of one MoE layer (lfm_ep_plan, host only):
    (counts per destination rank, send order of the (token, rank) slots)."""
    sel = np.ascontiguousarray(sel, dtype=np.int32).ravel()
    counts = np.zeros(world, dtype=np.int32)
    order = np.zeros(max(sel.size, 1), dtype=np.int32)
    st = lib().lfm_ep_plan(_p(sel), sel.size, world, _p(counts), _p(order))
    if st != 0:
        raise LfmError(f"lfm_ep_plan: {lib().lfm_global_error().decode()} (status {st})")
    return counts, order[: sel.size]


def model_inspect(gguf_path: str) -> Hparams:
    """Validate a model file without a device (lfm_model_inspect): the GGUF
    header rules, the hyperparameters and the tensor table. Raises LfmError
    with the library's message."""
    hp = Hparams()
    st = lib().lfm_model_inspect(gguf_path.encode(), ctypes.byref(hp))
    if st != 0:
        raise LfmError(f"lfm_model_inspect: {lib().lfm_global_error().decode()} (status {st})")
    return hp


def ops_check(status: int, what: str):
    if status != 0:
        raise LfmError(f"{what}: {lib().lfm_ops_error().decode()} (status {status})")


class GpuEngine:
    """The B200 engine behind the C ABI (one per GPU per host thread)."""

    def __init__(self, gguf_path: str, device: int = 0):
        h = ctypes.c_void_p()
        st = lib().lfm_engine_create(gguf_path.encode(), device, ctypes.byref(h))
        if st != 0:
            raise LfmError(f"lfm_engine_create: {lib().lfm_global_error().decode()} (status {st})")
        self.h = h
        hp = Hparams()
        lib().lfm_hparams_get(self.h, ctypes.byref(hp))
        self.hp = hp
        self.vocab = hp.vocab
        self.eos = hp.eos

    def close(self):
        if getattr(self, "h", None):
            lib().lfm_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int, what: str):
        if st != 0:
            raise LfmError(f"{what}: {lib().lfm_last_error(self.h).decode()} (status {st})")

    @property
    def device_name(self) -> str:
        return lib().lfm_device_name(self.h).decode()

    def set_ctx(self, ctx: int):
        self._check(lib().lfm_engine_set_ctx(self.h, ctx), "set_ctx")

    def forward(self, ids, start_pos: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32)
        self._check(lib().lfm_forward_logits(self.h, _p(ids), ids.size, start_pos, _p(out)), "forward")
        return out

    def forward_token(self, ids, position: int) -> int:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        nxt = ctypes.c_uint32()
        self._check(lib().lfm_forward_token(self.h, _p(ids), ids.size, position, ctypes.byref(nxt)),
                    "forward_token")
        return int(nxt.value)

    def generate(self, prompt, n: int, eos: int):
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max(n, 1), dtype=np.uint32)
        cnt = ctypes.c_uint32()
        self._check(lib().lfm_generate(self.h, _p(prompt), prompt.size, n, eos, _p(out), ctypes.byref(cnt)),
                    "generate")
        return out[: cnt.value].tolist()

    def decode_loop(self, first_token: int, start_pos: int, steps: int):
        """Device-resident greedy decode; returns (tokens, device_ms)."""
        out = np.empty(steps, dtype=np.uint32)
        ms = ctypes.c_float()
        self._check(lib().lfm_decode_loop(self.h, first_token, start_pos, steps, _p(out), ctypes.byref(ms)),
                    "decode_loop")
        return out.tolist(), float(ms.value)

    def last_device_ms(self) -> float:
        return float(lib().lfm_last_device_ms(self.h))

    # -------- independent sessions decoded together (lfm_batch_*)
    def batch_create(self, n_sessions: int):
        self._check(lib().lfm_batch_create(self.h, n_sessions), "batch_create")

    def batch_prefill(self, session: int, ids) -> int:
        """Fresh prompt of one session; returns its greedy next token."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        t = ctypes.c_uint32()
        self._check(lib().lfm_batch_prefill(self.h, session, _p(ids), len(ids), ctypes.byref(t)), "batch_prefill")
        return int(t.value)

    def batch_prefill_many(self, sessions, prompts) -> np.ndarray:
        """Fresh prompts of several sessions in one pass; their next tokens."""
        ss = np.ascontiguousarray(sessions, dtype=np.uint32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]), dtype=np.uint32)
        lens = np.array([len(p) for p in prompts], dtype=np.uint32)
        out = np.empty(len(ss), dtype=np.uint32)
        self._check(lib().lfm_batch_prefill_many(self.h, _p(ss), _p(ids), _p(lens), len(ss), _p(out)),
                    "batch_prefill_many")
        return out

    def batch_decode(self, sessions, tokens, positions) -> np.ndarray:
        """One decode step of distinct sessions; returns their next tokens."""
        ss = np.ascontiguousarray(sessions, dtype=np.uint32)
        tt = np.ascontiguousarray(tokens, dtype=np.uint32)
        pp = np.ascontiguousarray(positions, dtype=np.uint32)
        out = np.empty(len(ss), dtype=np.uint32)
        self._check(lib().lfm_batch_decode(self.h, _p(ss), _p(tt), _p(pp), len(ss), _p(out)), "batch_decode")
        return out

    def batch_logits(self, index: int) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        self._check(lib().lfm_batch_logits(self.h, index, _p(out)), "batch_logits")
        return out

    def step_trace(self, enable: bool):
        """Switch per-stage timestamps of the persistent decode step on/off and
        return the last step's record as uint64 [stages][ctas][8] (None when
        the kernel chain runs): start, staged, first tile, done (ns stamps),
        tile wait cycles, tiles, tile compute cycles, epilogue cycles."""
        ns, nc = ctypes.c_uint32(), ctypes.c_uint32()
        self._check(lib().lfm_step_trace(self.h, 1 if enable else 0, None, 0, ctypes.byref(ns), ctypes.byref(nc)),
                    "step_trace")
        if ns.value == 0:
            return None
        out = np.zeros((ns.value, nc.value, 8), dtype=np.uint64)
        self._check(lib().lfm_step_trace(self.h, 1 if enable else 0, _p(out), out.size, None, None), "step_trace")
        return out

    def info(self) -> dict:
        """Decode path and launch facts of this engine (JSON from the library)."""
        import json
        return json.loads(lib().lfm_engine_info(self.h).decode())

    # -------- expert-parallel prompt path (lfm_ep_*), one process per GPU
    def ep_init(self, nccl_id: bytes, rank: int, world: int):
        buf = np.frombuffer(nccl_id, dtype=np.uint8).copy()
        self._check(lib().lfm_ep_init(self.h, _p(buf), rank, world), "ep_init")

    def ep_prefill(self, ids, session: int = 0xFFFFFFFF) -> int:
        """Collective: every rank of the group prefills its own prompt."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        t = ctypes.c_uint32()
        self._check(lib().lfm_ep_prefill(self.h, session, _p(ids), len(ids), ctypes.byref(t)), "ep_prefill")
        return int(t.value)

    def ep_finalize(self):
        self._check(lib().lfm_ep_finalize(self.h), "ep_finalize")

    def reset_session(self):
        self._check(lib().lfm_reset_session(self.h), "reset_session")

    def snapshot_resident_cache(self, valid: int) -> bytes:
        n = ctypes.c_size_t()
        self._check(lib().lfm_snapshot_cache(self.h, valid, None, 0, ctypes.byref(n)), "snapshot")
        buf = np.empty(n.value, dtype=np.uint8)
        self._check(lib().lfm_snapshot_cache(self.h, valid, _p(buf), buf.size, ctypes.byref(n)), "snapshot")
        return buf.tobytes()

    def restore_session(self, valid: int, data: bytes):
        buf = np.frombuffer(data, dtype=np.uint8)
        self._check(lib().lfm_restore_cache(self.h, valid, _p(buf) if buf.size else None, buf.size), "restore")

    def snapshot_resident_logits(self) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        self._check(lib().lfm_snapshot_logits(self.h, _p(out)), "snapshot_logits")
        return out

    def counters(self) -> dict:
        c = Counters()
        lib().lfm_counters_get(self.h, ctypes.byref(c))
        return {k: int(getattr(c, k)) for k, _ in Counters._fields_}


class TextStreams:
    """Streaming text of many sessions (lfm_text_*): token pieces assembled
    into UTF-8 text and cleaned as the reference's StreamDecoder + DecodedText
    do. `pieces[t]` = bytes of token t (the tokenizer's token_to_piece)."""

    def __init__(self, pieces, n_sessions: int, clean_spaces: bool = True, replace_invalid: bool = False):
        blob = b"".join(pieces)
        off = np.zeros(len(pieces) + 1, dtype=np.uint64)
        off[1:] = np.cumsum([len(p) for p in pieces])
        self._blob = np.frombuffer(blob, dtype=np.uint8).copy() if blob else np.zeros(1, np.uint8)
        self._off = off
        h = ctypes.c_void_p()
        st = lib().lfm_text_create(_p(self._blob), _p(self._off), len(pieces), n_sessions, int(clean_spaces),
                                   int(replace_invalid), ctypes.byref(h))
        if st != 0:
            raise LfmError(f"lfm_text_create: {lib().lfm_text_error().decode()} (status {st})")
        self.h = h
        self._cap = 1 << 16
        self._buf = ctypes.create_string_buffer(self._cap)

    def close(self):
        if getattr(self, "h", None):
            lib().lfm_text_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def push(self, sessions, tokens):
        """One token per entry; returns the bytes each entry completed."""
        ss = np.ascontiguousarray(sessions, dtype=np.uint32)
        tt = np.ascontiguousarray(tokens, dtype=np.uint32)
        off = np.zeros(len(ss) + 1, dtype=np.uint64)
        st = lib().lfm_text_push(self.h, _p(ss), _p(tt), len(ss), self._buf, self._cap, _p(off))
        if st != 0:
            raise LfmError(f"lfm_text_push: {lib().lfm_text_error().decode()} (status {st})")
        raw = self._buf.raw
        return [raw[int(off[i]):int(off[i + 1])] for i in range(len(ss))]

    def finish(self, session: int) -> bytes:
        n = ctypes.c_size_t()
        st = lib().lfm_text_finish(self.h, session, self._buf, self._cap, ctypes.byref(n))
        if st != 0:
            raise LfmError(f"lfm_text_finish: {lib().lfm_text_error().decode()} (status {st})")
        return self._buf.raw[: n.value]

    def reset(self, session: int):
        st = lib().lfm_text_reset(self.h, session)
        if st != 0:
            raise LfmError(f"lfm_text_reset: {lib().lfm_text_error().decode()} (status {st})")

