"""promptboot_b200: B200-native (sm_100a) decode hot path of sulewicz/promptboot.

The compute path is the CUDA library promptboot_b200/lib/libpromptboot_b200.so
behind the C ABI in include/promptboot_b200.h; this package is its Python
binding and the PBTQW25 v1 writer used to make seeded synthetic images.
"""
from .api import (CONTEXT_LIMIT, EOS, SEEN_BYTES, VOCAB, DeviceError, InferenceEngine,
                  InferenceError, InferenceStep, ModelError, ModelView, SamplingState,
                  greedy_token, sample_token, sample_token_with_repetition, top_logits_8)

__all__ = [
    "CONTEXT_LIMIT", "EOS", "SEEN_BYTES", "VOCAB", "DeviceError", "InferenceEngine",
    "InferenceError", "InferenceStep", "ModelError", "ModelView", "SamplingState",
    "greedy_token", "sample_token", "sample_token_with_repetition", "top_logits_8",
]
