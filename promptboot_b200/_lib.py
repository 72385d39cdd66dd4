"""ctypes binding of include/promptboot_b200.h (the library's C ABI).

The shared library is built in-tree (promptboot_b200/lib/libpromptboot_b200.so,
see promptboot_b200/build.py).  There is no fallback: if it is missing or fails
to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import pathlib

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libpromptboot_b200.so"

u8p = ctypes.POINTER(ctypes.c_uint8)
u32 = ctypes.c_uint32
u64 = ctypes.c_uint64
P = ctypes.c_void_p


class PbError(ctypes.Structure):
    """InferenceError (inference.rs:226-238), 48 bytes."""
    _fields_ = [("status", u32), ("domain", u32), ("layer", u32), ("position", u32),
                ("tensor_id", u32), ("reserved", u32), ("needed", u64),
                ("available", u64), ("detail", u64)]

    def tuple(self):
        """The 8-tuple the reference's tests compare (tests.rs:185-196)."""
        return [self.status, self.domain, self.layer, self.position, self.tensor_id,
                self.needed, self.available, self.detail]


class PbStep(ctypes.Structure):
    """InferenceStep (inference.rs:266-273)."""
    _fields_ = [("position", u32), ("selected_token", u32), ("selected_logit_bits", u32),
                ("eos", u32)]


class PbArenaUsage(ctypes.Structure):
    _fields_ = [("capacity", u64), ("requested", u64), ("committed", u64), ("current", u64),
                ("high_water", u64)]


class PbUsage(ctypes.Structure):
    """InferenceUsage (inference.rs:275-285), 136 bytes."""
    _fields_ = [("weights", PbArenaUsage), ("kv", PbArenaUsage), ("scratch", PbArenaUsage),
                ("position", u32), ("context_limit", u32), ("generation_reserve", u32),
                ("state", u32)]


class PbSamplingState(ctypes.Structure):
    """SamplingState (inference.rs:772-799), 16 bytes."""
    _fields_ = [("state", u64), ("draws", u64)]


class PbTopLogit(ctypes.Structure):
    _fields_ = [("token", u32), ("logit_bits", u32)]


class PbModelError(ctypes.Structure):
    """ModelError (model.rs:113-124), 48 bytes."""
    _fields_ = [("status", u32), ("domain", u32), ("index", u32), ("reserved", u32),
                ("offset", u64), ("needed", u64), ("available", u64), ("detail", u64)]

    def tuple(self):
        return [self.status, self.domain, self.index, self.offset, self.needed,
                self.available, self.detail]


E = ctypes.POINTER(PbError)
S = ctypes.POINTER(PbStep)

SIGNATURES = {
    "pb_abi_version": (u32, []),
    "pb_last_error_string": (ctypes.c_char_p, []),
    "pb_model_open": (u32, [P, u64, u32, ctypes.c_int, ctypes.POINTER(P),
                            ctypes.POINTER(PbModelError)]),
    "pb_model_close": (None, [P]),
    "pb_model_tensor_device": (P, [P, u32]),
    "pb_engine_create": (u32, [P, u32, u32, ctypes.POINTER(P), E]),
    "pb_engine_destroy": (None, [P]),
    "pb_engine_prefill": (u32, [P, u32, P, u32, u32, P, S, E]),
    "pb_engine_prefill_with_prefix": (u32, [P, u32, P, u32, u32, u32, P, S, E]),
    "pb_engine_append_prefill": (u32, [P, u32, P, u32, u32, P, S, E]),
    "pb_engine_decode": (u32, [P, u32, u32, P, S, E]),
    "pb_engine_decode_selected": (u32, [P, u32, u32, P, S, E]),
    "pb_engine_reset": (u32, [P, u32]),
    "pb_engine_reset_to_prefix": (u32, [P, u32, ctypes.POINTER(u32)]),
    "pb_engine_usage": (u32, [P, u32, ctypes.POINTER(PbUsage)]),
    "pb_engine_position": (u32, [P, u32]),
    "pb_engine_kv_device": (P, [P, u32, ctypes.POINTER(u64)]),
    "pb_engine_restore": (u32, [P, u32, P, u32, u32, E]),
    "pb_engine_prefill_batch": (u32, [P, u32, P, P, u32, u32, P, P]),
    "pb_engine_decode_batch": (u32, [P, u32, P, P, u32, P, P]),
    "pb_engine_logits": (u32, [P, u32, P]),
    "pb_engine_sample": (u32, [P, u32, P, P, P, P]),
    "pb_engine_generate": (u32, [P, u32, P, P, u32, P, P]),
    "pb_engine_stream": (P, [P]),
    "pb_engine_launch_count": (u64, [P]),
    "pb_engine_profile": (u32, [P, u32]),
    "pb_engine_profile_read": (u32, [P, P, P]),
    "pb_sampling_state_init": (None, [ctypes.POINTER(PbSamplingState), u64]),
    "pb_sample_token": (u32, [P, u64, ctypes.POINTER(PbSamplingState), P, E]),
    "pb_sample_token_with_repetition": (u32, [P, u64, P, u64, P, u64,
                                              ctypes.POINTER(PbSamplingState), P, E]),
    "pb_greedy_token": (u32, [P, u64, P, E]),
    "pb_top_logits_8": (u32, [P, u64, P, E]),
    "pb_sample_batch_device": (u32, [P, u64, u32, P, P, P, P, P, P]),
    "pb_qmatvec_device": (u32, [u32, P, u32, u32, P, u32, P, P]),
    "pb_model_matvec_device": (u32, [P, u32, P, u32, P, P]),
    "pb_model_matvec_status": (u32, [P, P]),
    "pb_qmatvec_device_noalloc": (u32, [u32, P, u32, u32, P, u32, P, P]),
    "pb_quantize_q8_device": (u32, [P, u32, u32, P, P]),
    "pb_rmsnorm_device": (u32, [P, P, u32, P, P]),
    "pb_swiglu_device": (u32, [P, P, u32, P, P]),
    "pb_rope_kv_device": (u32, [P, P, P, P, u32, P, u32, u32, P]),
    "pb_attention_device": (u32, [P, P, u32, u32, P, u32, u32, P, P, P]),
    "pb_rope_table": (u32, [P]),
    "pb_expf_device": (u32, [P, u64, P, P]),
}

_LIB = None


def load():
    """Load the in-tree library once and attach every C ABI signature."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m promptboot_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def last_error() -> str:
    return load().pb_last_error_string().decode()
