"""C ABI and host-logic tests that need no GPU.

They load the sm_100a library, check that it exports every entry point that
include/promptboot_b200.h declares with the reference's struct layouts, and
exercise the host-side validation paths (length / finiteness / seen-capacity /
token checks, PBTQW25 layout checks) whose errors must equal the reference's
(inference.rs:737-965, model.rs:371-983).  None of these paths touches CUDA.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import pathlib
import re

import numpy as np
import pytest

import oracle
from promptboot_b200 import _lib, api, pbtqw25

ROOT = pathlib.Path(__file__).resolve().parents[1]
NO = 0xFFFFFFFF


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        for m in re.finditer(r"^PB_API\s+[^(]*?\b(pb_[a-z0-9_]+)\s*\(", header.read_text(), re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 30
    for name in sorted(names):
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no Python binding"


def test_abi_struct_layouts_match_reference():
    """tests.rs:313-366 sizes and offsets."""
    assert ctypes.sizeof(_lib.PbError) == 48
    assert _lib.PbError.needed.offset == 24 and _lib.PbError.detail.offset == 40
    assert ctypes.sizeof(_lib.PbStep) == 16
    assert ctypes.sizeof(_lib.PbUsage) == 136
    assert _lib.PbUsage.kv.offset == 40 and _lib.PbUsage.scratch.offset == 80
    assert _lib.PbUsage.position.offset == 120 and _lib.PbUsage.state.offset == 132
    assert ctypes.sizeof(_lib.PbSamplingState) == 16
    assert ctypes.sizeof(_lib.PbTopLogit) == 8
    assert ctypes.sizeof(_lib.PbModelError) == 48
    assert _lib.load().pb_abi_version() == 1


def test_rope_table_built_by_library_is_the_pinned_table():
    table = np.zeros(32768 * 64, dtype=np.float32)
    assert _lib.load().pb_rope_table(ctypes.c_void_p(table.ctypes.data)) == 0
    manifest = json.loads((ROOT / "tests" / "golden" / "manifest.json").read_text())
    assert hashlib.sha256(table.tobytes()).hexdigest() == manifest["rope-table"]["sha256"]
    assert np.array_equal(table.view(np.uint32), oracle.rope_table().view(np.uint32))


def test_sampling_state_zero_seed_replacement():
    assert api.SamplingState(0).state() == 0x9E3779B97F4A7C15
    s = api.SamplingState(7)
    assert (s.state(), s.draws()) == (7, 0)


def test_logits_length_and_finiteness_errors_match_reference():
    """tests.rs:368-418 (greedy_token error tuples)."""
    logits = np.full(api.VOCAB, np.float32(-100.0)).view(np.uint32)
    with pytest.raises(api.InferenceError) as e:
        api.greedy_token(logits[:-1])
    assert e.value.tuple() == [4, 18, NO, 0, NO, 151_936, 151_935, 51_539_607_552]
    with pytest.raises(api.InferenceError) as e:
        api.greedy_token(np.zeros(api.VOCAB + 1, dtype=np.uint32))
    assert e.value.tuple() == [4, 18, NO, 0, NO, 151_936, 151_937, 51_539_607_552]
    bad = logits.copy()
    bad[11] = 0x7FC00000
    with pytest.raises(api.InferenceError) as e:
        api.greedy_token(bad)
    assert e.value.tuple() == [7, 19, NO, 0, NO, 0, 2_143_289_344, 30_064_771_083]
    with pytest.raises(api.InferenceError) as e:
        api.top_logits_8(np.where(np.arange(api.VOCAB) == 42, 0x7F800000, logits).astype(np.uint32))
    assert e.value.status == 7 and e.value.domain == 19 and e.value.detail == (7 << 32) | 42


def test_sampler_rejections_are_transactional_on_host():
    """tests.rs:458-465 and 483-491: errors leave logits, seen and state unchanged."""
    logits = np.full(api.VOCAB, np.float32(-100.0)).view(np.uint32).copy()
    st = api.SamplingState(0x0123456789ABCDEF)
    before = st.copy()
    with pytest.raises(api.InferenceError) as e:
        api.sample_token(logits[:-1], st)
    assert e.value.status == 4 and st == before
    logits[17] = 0x7FC00000
    with pytest.raises(api.InferenceError) as e:
        api.sample_token(logits, st)
    assert e.value.status == 7 and st == before
    logits[17] = 0
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    snapshot = logits.copy()
    with pytest.raises(api.InferenceError) as e:
        api.sample_token_with_repetition(logits, [api.VOCAB], seen, st)
    assert e.value.status == 3 and e.value.available == api.VOCAB
    assert np.array_equal(logits, snapshot) and not seen.any() and st == before
    with pytest.raises(api.InferenceError) as e:
        api.sample_token_with_repetition(logits, [1], seen[:100], st)
    assert e.value.tuple() == [4, 19, NO, 0, NO, 18_992, 100, (4 << 32) | 2]


def test_synthetic_image_layout():
    img = pbtqw25.load_or_synthesize(0)
    assert img.size == pbtqw25.MODEL_BYTES
    assert bytes(img[:8]) == b"PBTQW25\0"
    offsets = pbtqw25.tensor_offsets()
    for tid in (0, 1, 100, 289, 290):
        view = pbtqw25.tensor_view(img, tid)
        assert view.size == pbtqw25.tensor_bytes(tid)
        assert offsets[tid] % 64 == 0
    norm = pbtqw25.tensor_view(img, pbtqw25.layer_tensor(3, 10)).view(np.float32)
    assert np.all(norm == 1.0)


def test_lm_head_is_the_reference_quantization_of_the_embedding():
    img = pbtqw25.load_or_synthesize(0)
    emb = pbtqw25.tensor_view(img, 0).reshape(api.VOCAB, 28, 18)
    out = pbtqw25.tensor_view(img, 290).reshape(api.VOCAB, 28, 34)
    rng = np.random.default_rng(3)
    for r in rng.integers(0, api.VOCAB, size=16):
        x = np.zeros(896, dtype=np.float32)
        oracle.lib().orc_q4_row(oracle._p(np.ascontiguousarray(emb[r])), 0, oracle._p(x), 896)
        assert np.array_equal(pbtqw25.dequantize_q4_rows(emb[r:r + 1])[0].view(np.uint32),
                              x.view(np.uint32))
        assert np.array_equal(oracle.prepare_q8(x), out[r].reshape(-1))


def test_quantizer_restatement_edge_inputs():
    x = np.zeros((1, 192), dtype=np.float32)
    x[0, 32:36] = [1, -1, 1, -1]
    x[0, 64:69] = [127, 0.5, -0.5, 1.5, -1.5]
    x[0, 96:99] = oracle.f32([0x34000000, 0x33800000, 0x33000000])
    x[0, 128:131] = [126.5, -126.5, 63.25]
    x[0, 160] = np.float32(-0.0)
    got = pbtqw25.quantize_q8_rows(x).reshape(-1)
    assert got.tobytes() == (ROOT / "tests" / "golden" / "q8.bin").read_bytes()


def test_model_open_rejects_bad_layout_before_touching_the_device():
    img = pbtqw25.load_or_synthesize(0)
    with pytest.raises(api.ModelError) as e:
        api.ModelView(img[:-1])
    assert e.value.fields[:3] == [1, 1, 0]
    bad = img.copy()
    bad[3] = ord("X")
    with pytest.raises(api.ModelError) as e:
        api.ModelView(bad)
    assert e.value.fields == [3, 1, 3, 3, ord("Q"), ord("X"), (4 << 32) | 3]
    bad = img.copy()
    bad[pbtqw25.TENSOR_DIR + 7 * 96 + 8] = 3  # tensor 7 dtype Q4_0 -> Q8_0
    with pytest.raises(api.ModelError) as e:
        api.ModelView(bad)
    assert e.value.fields == [17, 3, 7, pbtqw25.TENSOR_DIR + 7 * 96 + 8, 2, 3, 18 << 32]


def test_sampling_states_batch_shares_one_array():
    """SamplingStates keeps its rows in one pb_sampling_state array that the
    batched entry points take as is; items are views of those rows."""
    from promptboot_b200 import api
    batch = api.SamplingStates([0, 7, 8])
    assert len(batch) == 3
    assert batch[1] == api.SamplingState(7) and batch[-1] == api.SamplingState(8)
    assert batch[0] == api.SamplingState(0)             # seed 0 takes the replacement constant
    view = batch[2]
    view._s.state = 12345
    assert batch._arr[2].state == 12345                  # a view, not a copy
    assert api._state_array(batch, 3) is batch._arr
    with pytest.raises(ValueError):
        api._state_array(batch, 4)
    with pytest.raises(IndexError):
        batch[3]
    listed = [api.SamplingState(5), api.SamplingState(6)]
    arr = api._state_array(listed, 2)
    arr[0].draws = 9
    api._state_back(listed, arr)
    assert listed[0].draws() == 9 and listed[1] == api.SamplingState(6)


def test_step_views_convert_on_access():
    from promptboot_b200 import _lib, api
    arr = (_lib.PbStep * 3)()
    arr[1].position, arr[1].selected_token, arr[1].eos = 17, 42, 1
    steps = api._Steps(arr)
    assert len(steps) == 3
    assert steps[1].position == 17 and steps[1].selected_token == 42 and steps[1].eos == 1
    assert [s.position for s in steps] == [0, 17, 0]
    assert steps[1:][0].selected_token == 42
