"""ctypes wrapper of the CPU oracle (test infrastructure only).

The oracle (lfm_oracle.cpp) restates the reference's CPU path; see that file's
header for the cited reference lines. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this module.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liblfm_oracle.so")
CLI_PATH = os.path.join(HERE, "_build", "lfm2_greedy_cpu")

_lib = None


def build(quiet: bool = True) -> None:
    """Compile the oracle with its Makefile (system g++, OpenMP)."""
    subprocess.run(["make", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, F, U32, I32, SZ = ctypes.c_void_p, ctypes.c_float, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f16_to_f32.restype = F
        L.oracle_f32_to_f16.argtypes = [F]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_dequant_block.argtypes = [P, P]
        L.oracle_shader_dequant.argtypes = [P, U32]
        L.oracle_shader_dequant.restype = F
        L.oracle_dequant_rows.argtypes = [P, SZ, P]
        L.oracle_q6k_matvec_f64.argtypes = [P, I32, I32, P, P]
        L.oracle_q6k_matmul_f32.argtypes = [P, I32, I32, P, I32, P]
        L.oracle_argmax.argtypes = [P, SZ]
        L.oracle_argmax.restype = U32
        L.oracle_route.argtypes = [P, P, I32, I32, P, P]
        L.oracle_silu_mul.argtypes = [F, F]
        L.oracle_silu_mul.restype = F
        L.oracle_engine_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p, SZ]
        L.oracle_engine_create.restype = P
        L.oracle_engine_destroy.argtypes = [P]
        L.oracle_engine_set_ctx.argtypes = [P, SZ]
        L.oracle_engine_set_kv_f16.argtypes = [P, I32]
        L.oracle_engine_vocab.argtypes = [P]
        L.oracle_engine_vocab.restype = I32
        L.oracle_engine_eos.argtypes = [P]
        L.oracle_engine_eos.restype = U32
        L.oracle_engine_error.argtypes = [P]
        L.oracle_engine_error.restype = ctypes.c_char_p
        L.oracle_forward.argtypes = [P, P, I32, ctypes.c_int64, P]
        L.oracle_forward.restype = I32
        L.oracle_snapshot.argtypes = [P, SZ, P]
        L.oracle_snapshot.restype = SZ
        L.oracle_greedy.argtypes = [P, P, I32, I32, U32, P, P]
        L.oracle_greedy.restype = I32
        L.oracle_checkpoint.argtypes = [P]
        L.oracle_checkpoint.restype = None
        L.oracle_rollback.argtypes = [P]
        L.oracle_rollback.restype = None
        L.oracle_num_threads.restype = I32
        L.oracle_set_threads.argtypes = [I32]
        L.oracle_set_threads.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def dequant_blocks(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    nb = raw.size // 210
    out = np.empty(nb * 256, dtype=np.float32)
    lib().oracle_dequant_rows(_p(raw), nb, _p(out))
    return out


def shader_dequant(block: np.ndarray, k: int) -> float:
    block = np.ascontiguousarray(block, dtype=np.uint8)
    return lib().oracle_shader_dequant(_p(block), k)


def q6k_matvec_f64(w: np.ndarray, in_dim: int, out_dim: int, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(out_dim, dtype=np.float32)
    lib().oracle_q6k_matvec_f64(_p(w), in_dim, out_dim, _p(x), _p(out))
    return out


def q6k_matmul_f32(w: np.ndarray, in_dim: int, out_dim: int, x: np.ndarray, n: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(out_dim * n, dtype=np.float32)
    lib().oracle_q6k_matmul_f32(_p(w), in_dim, out_dim, _p(x), n, _p(out))
    return out


def argmax(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().oracle_argmax(_p(logits), logits.size))


def route(router: np.ndarray, bias: np.ndarray, n_used: int = 4):
    router = np.ascontiguousarray(router, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    sel = np.empty(n_used, dtype=np.int32)
    w = np.empty(n_used, dtype=np.float32)
    lib().oracle_route(_p(router), _p(bias), router.size, n_used, _p(sel), _p(w))
    return sel, w


def f32_to_f16_bits(x: float) -> int:
    return int(lib().oracle_f32_to_f16(x))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().oracle_f16_to_f32(h))


class OracleEngine:
    """The reference's CPU `Engine` (engine/src/lfm.rs:147-745), restated."""

    def __init__(self, path: str, kv_f16: bool = True):
        err = ctypes.create_string_buffer(512)
        self.h = lib().oracle_engine_create(path.encode(), err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        lib().oracle_engine_set_kv_f16(self.h, int(kv_f16))
        self.vocab = lib().oracle_engine_vocab(self.h)
        self.eos = lib().oracle_engine_eos(self.h)

    def close(self):
        if self.h:
            lib().oracle_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def set_ctx(self, ctx: int):
        lib().oracle_engine_set_ctx(self.h, ctx)

    def forward(self, ids, start_pos: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32)
        if lib().oracle_forward(self.h, _p(ids), ids.size, start_pos, _p(out)) != 0:
            raise RuntimeError(lib().oracle_engine_error(self.h).decode())
        return out

    def checkpoint(self):
        """Save the session state (K/V caches, conv states)."""
        lib().oracle_checkpoint(self.h)

    def rollback(self):
        """Put back the state saved by checkpoint()."""
        lib().oracle_rollback(self.h)

    def snapshot(self, valid: int) -> np.ndarray:
        n = lib().oracle_snapshot(self.h, valid, None)
        out = np.empty(n, dtype=np.float32)
        lib().oracle_snapshot(self.h, valid, _p(out))
        return out

    def greedy(self, prompt, n: int, eos: int, keep_logits: bool = True):
        """main.rs:174-195. Returns (tokens, per-forward logits [steps, vocab])."""
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        toks = np.empty(max(n, 1), dtype=np.uint32)
        logits = np.empty((n + 1, self.vocab), dtype=np.float32) if keep_logits else None
        cnt = lib().oracle_greedy(self.h, _p(prompt), prompt.size, n, eos, _p(toks),
                                  _p(logits) if keep_logits else None)
        if cnt < 0:
            raise RuntimeError(lib().oracle_engine_error(self.h).decode())
        return toks[:cnt].tolist(), (logits[:cnt + 1] if keep_logits else None)
