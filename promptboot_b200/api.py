"""Python mirror of promptboot-core's engine and sampler API over the C ABI.

Names, argument meaning and error behaviour follow the reference
(sulewicz/promptboot crates/promptboot-core/src/inference.rs:772-1371,
model.rs:371-720): logits are uint32 binary32 bit patterns, failures raise
InferenceError carrying the reference's 48-byte error fields, and failed calls
leave state untouched where the reference's prechecks do.
"""
from __future__ import annotations

import collections.abc
import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

VOCAB = 151_936
CONTEXT_LIMIT = 32_768
EOS = 151_645
SEEN_BYTES = 18_992
NO_LAYER = 0xFFFFFFFF
NO_TENSOR = 0xFFFFFFFF


class InferenceError(Exception):
    """InferenceError (inference.rs:226-264) raised from a failed call."""

    def __init__(self, err: _lib.PbError):
        self.status = err.status
        self.domain = err.domain
        self.layer = err.layer
        self.position = err.position
        self.tensor_id = err.tensor_id
        self.needed = err.needed
        self.available = err.available
        self.detail = err.detail
        super().__init__(f"InferenceError{tuple(self.tuple())}")

    def tuple(self):
        return [self.status, self.domain, self.layer, self.position, self.tensor_id,
                self.needed, self.available, self.detail]


class ModelError(Exception):
    def __init__(self, err: _lib.PbModelError):
        self.fields = err.tuple()
        self.status = err.status
        super().__init__(f"ModelError{tuple(self.fields)}")


class DeviceError(RuntimeError):
    pass


@dataclass(frozen=True)
class InferenceStep:
    position: int
    selected_token: int
    selected_logit_bits: int
    eos: int


def _step(s: _lib.PbStep) -> InferenceStep:
    return InferenceStep(s.position, s.selected_token, s.selected_logit_bits, s.eos)


class _Steps(collections.abc.Sequence):
    """The InferenceStep results of a batched call, converted on access (a
    batch of 256 converted eagerly costs more host time than a decode step's
    launches)."""

    def __init__(self, arr):
        self._a = arr

    def __len__(self):
        return len(self._a)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [_step(x) for x in self._a[i]]
        return _step(self._a[i])


def _check(status: int, err: _lib.PbError):
    if status == 0:
        return
    if status == 100:
        raise DeviceError(_lib.last_error())
    raise InferenceError(err)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class SamplingState:
    """SamplingState (inference.rs:772-810)."""

    def __init__(self, seed: int = 0):
        self._s = _lib.PbSamplingState()
        _lib.load().pb_sampling_state_init(ctypes.byref(self._s), seed & (2**64 - 1))

    @classmethod
    def new(cls, seed: int) -> "SamplingState":
        return cls(seed)

    def state(self) -> int:
        return int(self._s.state)

    def draws(self) -> int:
        return int(self._s.draws)

    def __eq__(self, other):
        return (self.state(), self.draws()) == (other.state(), other.draws())

    def copy(self) -> "SamplingState":
        c = SamplingState(1)
        c._s.state, c._s.draws = self._s.state, self._s.draws
        return c


class SamplingStates(collections.abc.Sequence):
    """A batch of SamplingState held in one contiguous array, the layout the
    batched entry points take: passing it to sample / generate costs no
    per-row copies.  Item i is a SamplingState sharing row i's memory."""

    def __init__(self, seeds):
        seeds = [int(x) for x in seeds]
        self._arr = (_lib.PbSamplingState * len(seeds))()
        init = _lib.load().pb_sampling_state_init
        for i, seed in enumerate(seeds):
            init(ctypes.byref(self._arr[i]), seed & (2**64 - 1))

    def __len__(self):
        return len(self._arr)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        if i < 0:
            i += len(self)
        if not 0 <= i < len(self):
            raise IndexError(i)
        view = SamplingState.__new__(SamplingState)
        view._s = _lib.PbSamplingState.from_buffer(self._arr, i * ctypes.sizeof(_lib.PbSamplingState))
        return view


def _state_array(states, n: int):
    if isinstance(states, SamplingStates):
        if len(states) != n:
            raise ValueError("one sampling state per sequence")
        return states._arr
    arr = (_lib.PbSamplingState * n)()
    for i, s in enumerate(states):
        arr[i] = s._s
    return arr


def _state_back(states, arr):
    if isinstance(states, SamplingStates):
        return
    for i, s in enumerate(states):
        s._s.state, s._s.draws = arr[i].state, arr[i].draws


def sample_token(logits, state: SamplingState) -> int:
    """inference.rs:914-917 (executed on the GPU)."""
    x = _u32(logits)
    out = ctypes.c_uint32()
    err = _lib.PbError()
    st = _lib.load().pb_sample_token(_ptr(x), x.size, ctypes.byref(state._s), ctypes.byref(out),
                                     ctypes.byref(err))
    _check(st, err)
    return out.value


def sample_token_with_repetition(logits: np.ndarray, tokens, seen: np.ndarray,
                                 state: SamplingState) -> int:
    """inference.rs:919-965; `logits` (uint32 array) and `seen` are mutated in place."""
    if logits.dtype != np.uint32 or not logits.flags.c_contiguous:
        raise TypeError("logits must be a contiguous uint32 array (binary32 bit patterns)")
    toks = _u32(tokens)
    out = ctypes.c_uint32()
    err = _lib.PbError()
    st = _lib.load().pb_sample_token_with_repetition(
        _ptr(logits), logits.size, _ptr(toks), toks.size, _ptr(seen), seen.size,
        ctypes.byref(state._s), ctypes.byref(out), ctypes.byref(err))
    _check(st, err)
    return out.value


def greedy_token(logits) -> int:
    """inference.rs:861-881."""
    x = _u32(logits)
    out = ctypes.c_uint32()
    err = _lib.PbError()
    st = _lib.load().pb_greedy_token(_ptr(x), x.size, ctypes.byref(out), ctypes.byref(err))
    _check(st, err)
    return out.value


def top_logits_8(logits):
    """inference.rs:814-859: list of (token, logit_bits)."""
    x = _u32(logits)
    out = (_lib.PbTopLogit * 8)()
    err = _lib.PbError()
    st = _lib.load().pb_top_logits_8(_ptr(x), x.size, out, ctypes.byref(err))
    _check(st, err)
    return [(o.token, o.logit_bits) for o in out]


class ModelView:
    """A PBTQW25 v1 image uploaded to one GPU (model.rs:371-720, layout-only open)."""

    def __init__(self, image: np.ndarray, device: int = 0):
        img = np.ascontiguousarray(image, dtype=np.uint8)
        handle = ctypes.c_void_p()
        err = _lib.PbModelError()
        st = _lib.load().pb_model_open(_ptr(img), img.size, 1, device, ctypes.byref(handle),
                                       ctypes.byref(err))
        if st == 100:
            raise DeviceError(_lib.last_error())
        if st:
            raise ModelError(err)
        self._h = handle
        self.device = device

    @classmethod
    def open_layout(cls, image: np.ndarray, device: int = 0) -> "ModelView":
        return cls(image, device)

    def tensor_device_ptr(self, tid: int) -> int:
        return _lib.load().pb_model_tensor_device(self._h, tid) or 0

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().pb_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class InferenceEngine:
    """InferenceEngine (inference.rs:967-1371) over `max_seqs` device-resident sequences.

    Single-sequence calls take `seq` (default 0) so that code written against the
    reference's one-engine-one-sequence API runs unchanged with seq=0.
    """

    def __init__(self, model: ModelView, max_seqs: int = 1, max_context: int = 4096):
        handle = ctypes.c_void_p()
        err = _lib.PbError()
        st = _lib.load().pb_engine_create(model._h, max_seqs, max_context, ctypes.byref(handle),
                                          ctypes.byref(err))
        _check(st, err)
        self._h = handle
        self._model = model
        self.max_seqs = max_seqs
        self.max_context = max_context

    @classmethod
    def build(cls, model: ModelView, max_seqs: int = 1, max_context: int = 4096):
        return cls(model, max_seqs, max_context)

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().pb_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _prefill_like(self, fn, seq, tokens, *args, logits=None):
        toks = _u32(tokens)
        step = _lib.PbStep()
        err = _lib.PbError()
        out = logits
        if out is not None and (out.dtype != np.uint32 or out.size != VOCAB):
            raise TypeError("logits must be a uint32 array of 151936 words")
        st = fn(self._h, seq, _ptr(toks), toks.size, *args, _ptr(out), ctypes.byref(step),
                ctypes.byref(err))
        _check(st, err)
        return _step(step)

    def prefill(self, tokens, generation_reserve: int, logits=None, seq: int = 0):
        return self._prefill_like(_lib.load().pb_engine_prefill, seq, tokens, generation_reserve,
                                  logits=logits)

    def prefill_with_prefix(self, tokens, prefix_tokens: int, generation_reserve: int,
                            logits=None, seq: int = 0):
        return self._prefill_like(_lib.load().pb_engine_prefill_with_prefix, seq, tokens,
                                  prefix_tokens, generation_reserve, logits=logits)

    def append_prefill(self, tokens, generation_reserve: int, logits=None, seq: int = 0):
        return self._prefill_like(_lib.load().pb_engine_append_prefill, seq, tokens,
                                  generation_reserve, logits=logits)

    def _decode(self, fn, token, logits, seq):
        step = _lib.PbStep()
        err = _lib.PbError()
        st = fn(self._h, seq, token, _ptr(logits), ctypes.byref(step), ctypes.byref(err))
        _check(st, err)
        return _step(step)

    def decode(self, token: int, logits=None, seq: int = 0):
        return self._decode(_lib.load().pb_engine_decode, token, logits, seq)

    def decode_selected(self, token: int, logits=None, seq: int = 0):
        return self._decode(_lib.load().pb_engine_decode_selected, token, logits, seq)

    def reset(self, seq: int = 0):
        _lib.load().pb_engine_reset(self._h, seq)

    def reset_to_prefix(self, seq: int = 0) -> int:
        out = ctypes.c_uint32()
        _lib.load().pb_engine_reset_to_prefix(self._h, seq, ctypes.byref(out))
        return out.value

    def usage(self, seq: int = 0) -> _lib.PbUsage:
        u = _lib.PbUsage()
        _lib.load().pb_engine_usage(self._h, seq, ctypes.byref(u))
        return u

    def position(self, seq: int = 0) -> int:
        return _lib.load().pb_engine_position(self._h, seq)

    def kv_device(self, seq: int = 0):
        """(device address, binary32 words) of slot `seq`'s KV region."""
        words = ctypes.c_uint64()
        addr = _lib.load().pb_engine_kv_device(self._h, seq, ctypes.byref(words))
        if not addr:
            raise IndexError(seq)
        return int(addr), int(words.value)

    def kv_tensor(self, seq: int = 0):
        """Slot `seq`'s KV region as a float32 torch tensor sharing the
        engine's memory (a view through __cuda_array_interface__)."""
        import torch
        addr, words = self.kv_device(seq)

        class _Region:
            __cuda_array_interface__ = {"shape": (words,), "typestr": "<f4",
                                        "data": (addr, False), "version": 3, "strides": None}
        return torch.as_tensor(_Region(), device=f"cuda:{self._model.device}")

    def stream(self) -> int:
        return int(_lib.load().pb_engine_stream(self._h) or 0)

    def restore(self, tokens, generation_reserve: int, seq: int = 0):
        """A RESET slot takes `tokens` whose KV the caller wrote into its region;
        it is then READY at position len(tokens) (decode_selected next)."""
        toks = _u32(tokens)
        err = _lib.PbError()
        st = _lib.load().pb_engine_restore(self._h, seq, _ptr(toks), toks.size,
                                           generation_reserve, ctypes.byref(err))
        _check(st, err)

    # ---- batched forms
    def prefill_batch(self, seqs, tokens: np.ndarray, generation_reserve: int):
        seqs = _u32(seqs)
        toks = _u32(tokens).reshape(seqs.size, -1)
        steps = (_lib.PbStep * seqs.size)()
        errs = (_lib.PbError * seqs.size)()
        st = _lib.load().pb_engine_prefill_batch(self._h, seqs.size, _ptr(seqs), _ptr(toks),
                                                 toks.shape[1], generation_reserve, steps, errs)
        if st == 100:
            raise DeviceError(_lib.last_error())
        return st, [_step(s) for s in steps], list(errs)

    def decode_batch(self, seqs, tokens, require_greedy: bool = False):
        """One decode step of every listed sequence; returns (status, steps,
        errors), steps and errors indexable per row."""
        seqs = _u32(seqs)
        toks = _u32(tokens)
        steps = (_lib.PbStep * seqs.size)()
        errs = (_lib.PbError * seqs.size)()
        st = _lib.load().pb_engine_decode_batch(self._h, seqs.size, _ptr(seqs), _ptr(toks),
                                                int(require_greedy), steps, errs)
        if st == 100:
            raise DeviceError(_lib.last_error())
        return st, _Steps(steps), errs

    def logits(self, row: int = 0) -> np.ndarray:
        out = np.zeros(VOCAB, dtype=np.uint32)
        st = _lib.load().pb_engine_logits(self._h, row, _ptr(out))
        if st:
            raise RuntimeError(f"no logits for batch row {row} (status {st})")
        return out

    def sample(self, seqs, states):
        """sample_token_with_repetition on the last step's rows, on the GPU.
        `states`: a SamplingStates batch (updated in place, no copies) or a
        list of SamplingState."""
        seqs = _u32(seqs)
        arr = _state_array(states, seqs.size)
        ids = np.zeros(seqs.size, dtype=np.uint32)
        errs = (_lib.PbError * seqs.size)()
        st = _lib.load().pb_engine_sample(self._h, seqs.size, _ptr(seqs), arr, _ptr(ids), errs)
        if st == 100:
            raise DeviceError(_lib.last_error())
        _state_back(states, arr)
        return st, ids, errs

    def generate(self, seqs, states, steps: int, want_tokens: bool = True):
        """Device-resident sample -> decode_selected loop (fixed length)."""
        seqs = _u32(seqs)
        arr = _state_array(states, seqs.size)
        out = np.zeros((steps, seqs.size), dtype=np.uint32) if want_tokens else None
        errs = (_lib.PbError * seqs.size)()
        st = _lib.load().pb_engine_generate(self._h, seqs.size, _ptr(seqs), arr, steps,
                                            _ptr(out), errs)
        if st == 100:
            raise DeviceError(_lib.last_error())
        _state_back(states, arr)
        return st, out, list(errs)
