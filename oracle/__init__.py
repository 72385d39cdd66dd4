"""CPU oracle for the promptboot decode hot path -- TEST INFRASTRUCTURE ONLY.

A ctypes view of oracle/oracle.c, the plain-C restatement of the reference's
decode arithmetic (crates/promptboot-core/src/fp32_sse2.rs and inference.rs in
sulewicz/promptboot).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg may import this package, and only as the checker: the product
library (promptboot_b200) never loads it.

Parity pin: tests/test_oracle_golden.py checks every function used by the GPU
parity tests against the reference's own golden vectors.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess
import threading

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

VOCAB = 151936
HIDDEN = 896
FFN = 4864
ROPE_WORDS = 32768 * 32 * 2


class OracleError(ctypes.Structure):
    _fields_ = [("status", ctypes.c_uint32), ("domain", ctypes.c_uint32),
                ("layer", ctypes.c_uint32), ("position", ctypes.c_uint32),
                ("tensor_id", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("needed", ctypes.c_uint64), ("available", ctypes.c_uint64),
                ("detail", ctypes.c_uint64)]

    def tuple(self):
        return (self.status, self.domain, self.layer, self.position, self.tensor_id,
                self.needed, self.available, self.detail)


def build() -> pathlib.Path:
    """Compile oracle.c with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


_LIB = None
_INIT_LOCK = threading.RLock()


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    with _INIT_LOCK:
        return _load()


def _load():
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        sz = ctypes.c_size_t
        u32 = ctypes.c_uint32
        sig = {
            "orc_half_to_f32_bits": (u32, [ctypes.c_uint16]),
            "orc_f32_bits_to_half": (ctypes.c_uint16, [u32]),
            "orc_expf_bits": (u32, [u32]),
            "orc_expf4": (None, [P]),
            "orc_q4_row": (None, [P, sz, P, sz]),
            "orc_prepare_q8": (None, [P, P, sz]),
            "orc_q4_block_dot": (ctypes.c_int32, [P, P]),
            "orc_q8_block_dot": (ctypes.c_int32, [P, P]),
            "orc_q4_matvec": (None, [P, P, P, sz, sz]),
            "orc_q8_matvec": (None, [P, P, P, sz, sz]),
            "orc_rmsnorm": (None, [P, P, P, sz]),
            "orc_rope_table": (None, [P]),
            "orc_rope_in_place": (None, [P, sz, sz, P]),
            "orc_kv_word": (sz, [sz, sz, sz, sz, sz, sz]),
            "orc_attention": (None, [P, P, sz, sz, sz, sz, P, P, P, P]),
            "orc_swiglu": (None, [P, P, P, sz]),
            "orc_argmax": (u32, [P, sz]),
            "orc_next_24": (u32, [P, P]),
            "orc_sample_top_k_top_p": (u32, [P, sz, u32]),
            "orc_apply_repetition_penalty": (None, [P, P, sz, P]),
            "orc_sample_with_repetition": (u32, [P, sz, P, sz, P, sz, P, P, P, P]),
            "orc_tensor": (P, [P, u32]),
            "orc_forward": (u32, [P, P, sz, P, u32, u32, P, P]),
            "orc_generate": (u32, [P, P, sz, P, P, u32, u32, ctypes.c_uint64, ctypes.c_int,
                                   P, P, P, P]),
            "orc_generate_many": (u32, [P, sz, P, u32, P, u32, u32, P, u32, P]),
            "orc_bench_decode": (u32, [P, sz, P, u32, u32, u32, P, u32, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def f32(words) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(words, dtype=np.uint32)).view(np.float32)


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32)


def expf_bits(x: int) -> int:
    return lib().orc_expf_bits(x)


def expf4(words) -> np.ndarray:
    w = np.array(words, dtype=np.uint32)
    lib().orc_expf4(_p(w))
    return w


def prepare_q8(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros((x.size // 32) * 34, dtype=np.uint8)
    lib().orc_prepare_q8(_p(x), _p(out), x.size)
    return out


def q4_matvec(weights: np.ndarray, staging: np.ndarray, rows: int, columns: int) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_q4_matvec(_p(weights), _p(staging), _p(out), rows, columns)
    return out


def q8_matvec(weights: np.ndarray, staging: np.ndarray, rows: int, columns: int) -> np.ndarray:
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_q8_matvec(_p(weights), _p(staging), _p(out), rows, columns)
    return out


def q4_block_dot(packed16: np.ndarray, act32: np.ndarray) -> int:
    w = np.ascontiguousarray(packed16, dtype=np.uint8)
    a = np.ascontiguousarray(act32, dtype=np.int8)
    return lib().orc_q4_block_dot(_p(w), _p(a))


def q8_block_dot(w32: np.ndarray, act32: np.ndarray) -> int:
    w = np.ascontiguousarray(w32, dtype=np.int8)
    a = np.ascontiguousarray(act32, dtype=np.int8)
    return lib().orc_q8_block_dot(_p(w), _p(a))


def rmsnorm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), _p(out), x.size)
    return out


_ROPE = None


def rope_table() -> np.ndarray:
    """The inference RoPE table, built once per process.  Callers pass its raw
    address to C, so the table must never be replaced once published: threads
    that race here build it under a lock."""
    global _ROPE
    with _INIT_LOCK:
        if _ROPE is None:
            t = np.zeros(ROPE_WORDS, dtype=np.float32)
            lib().orc_rope_table(_p(t))
            _ROPE = t
    return _ROPE


def rope_in_place(values: np.ndarray, heads: int, position: int) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32).copy()
    lib().orc_rope_in_place(_p(v), heads, position, _p(rope_table()))
    return v


def kv_word(capacity, layer, kind, position, head, component) -> int:
    return lib().orc_kv_word(capacity, layer, kind, position, head, component)


def attention(query: np.ndarray, kv: np.ndarray, capacity: int, layer: int, current: int,
              span: int, capture: bool = False):
    q = np.ascontiguousarray(query, dtype=np.float32)
    out = np.zeros(896, dtype=np.float32)
    scores = np.zeros(max(span, 4), dtype=np.float32)
    raw = np.zeros(14 * span, dtype=np.float32) if capture else None
    prob = np.zeros(14 * span, dtype=np.float32) if capture else None
    lib().orc_attention(_p(q), _p(kv), capacity, layer, current, span, _p(out), _p(scores),
                        _p(raw) if capture else None, _p(prob) if capture else None)
    return (out, scores, raw, prob) if capture else (out, scores)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    out = np.zeros_like(g)
    lib().orc_swiglu(_p(g), _p(u), _p(out), g.size)
    return out


def argmax(logits: np.ndarray) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().orc_argmax(_p(x), x.size)


class SamplingState:
    """inference.rs:772-810 (xorshift64 draw generator)."""

    def __init__(self, seed: int):
        self.state = np.array([seed if seed != 0 else 0x9E3779B97F4A7C15], dtype=np.uint64)
        self.draws = np.zeros(1, dtype=np.uint64)

    def next_24(self) -> int:
        return lib().orc_next_24(_p(self.state), _p(self.draws))


def sample_top_k_top_p(logits: np.ndarray, random24: int) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().orc_sample_top_k_top_p(_p(x), x.size, random24)


def sample_with_repetition(logits: np.ndarray, tokens, state: SamplingState, seen=None):
    """inference.rs:919-965; mutates logits in place, returns (status, id, error)."""
    toks = np.ascontiguousarray(tokens, dtype=np.uint32)
    if seen is None:
        seen = np.zeros((logits.size + 7) // 8, dtype=np.uint8)
    err = OracleError()
    sel = np.zeros(1, dtype=np.uint32)
    st = lib().orc_sample_with_repetition(_p(logits), logits.size, _p(toks), toks.size,
                                          _p(seen), seen.size, _p(state.state),
                                          _p(state.draws), _p(sel), ctypes.byref(err))
    return st, int(sel[0]), err


def forward(model: np.ndarray, kv: np.ndarray, capacity: int, token: int, position: int,
            want_logits: bool = True):
    logits = np.zeros(VOCAB, dtype=np.float32) if want_logits else None
    err = OracleError()
    st = lib().orc_forward(_p(model), _p(kv), capacity, _p(rope_table()), token, position,
                           _p(logits) if want_logits else None, ctypes.byref(err))
    return st, logits, err


def generate(model: np.ndarray, prompt, decode_steps: int, seed: int, capacity: int,
             stop_at_eos: bool = False):
    prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
    kv = np.zeros(24 * 2 * 2 * capacity * 64, dtype=np.float32)
    out = np.zeros(max(decode_steps, 1), dtype=np.uint32)
    count = np.zeros(1, dtype=np.uint32)
    logits = np.zeros(VOCAB, dtype=np.float32)
    err = OracleError()
    st = lib().orc_generate(_p(model), _p(kv), capacity, _p(rope_table()), _p(prompt),
                            prompt.size, decode_steps, seed, int(stop_at_eos), _p(out),
                            _p(count), _p(logits), ctypes.byref(err))
    return st, out[: int(count[0])].copy(), logits, err


def generate_many(model: np.ndarray, prompts: np.ndarray, decode_steps: int, seeds,
                  capacity: int, threads: int) -> np.ndarray:
    prompts = np.ascontiguousarray(prompts, dtype=np.uint32)
    nseq, plen = prompts.shape
    seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
    out = np.zeros((nseq, decode_steps), dtype=np.uint32)
    st = lib().orc_generate_many(_p(model), capacity, _p(rope_table()), nseq, _p(prompts),
                                 plen, decode_steps, _p(seeds), threads, _p(out))
    if st:
        raise RuntimeError(f"oracle generation failed with status {st}")
    return out


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def bench_decode(model: np.ndarray, start_position: int, steps: int, nseq: int, threads: int,
                 seeds=None) -> float:
    """CPU baseline work: nseq sequences x `steps` decode tokens (forward +
    sampler) from start_position over a seeded KV, on `threads` threads.
    Returns the aggregate decode rate in tokens/s: all tokens over the summed
    per-sequence decode-loop time divided by the threads that ran at once (the
    seeded KV fill before each loop is not timed)."""
    seeds = np.ascontiguousarray(np.arange(nseq) if seeds is None else seeds, dtype=np.uint64)
    cap = ((start_position + steps + 3) // 4) * 4
    loop = np.zeros(nseq, dtype=np.float64)
    st = lib().orc_bench_decode(_p(model), cap, _p(rope_table()), start_position, steps, nseq,
                                _p(seeds), threads, None, _p(loop))
    if st:
        raise RuntimeError(f"oracle bench failed with status {st}")
    concurrent = max(1, min(threads, nseq))
    return nseq * steps / (float(loop.sum()) / concurrent)
