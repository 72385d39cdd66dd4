"""Pin the CPU oracle to the reference's own golden vectors (CPU only).

Inputs restate crates/promptboot-core/src/tests.rs:4109-4435 of
sulewicz/promptboot; expected bytes are the reference's fixture files copied
into tests/golden/ by tests/golden/make_golden.py (SHA-256 checked).
"""
from __future__ import annotations

import hashlib
import json
import pathlib

import numpy as np
import pytest

import oracle

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def golden(name: str) -> bytes:
    return (GOLDEN / name).read_bytes()


def words(a) -> bytes:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).tobytes()


def test_golden_copies_match_manifest():
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    for name, entry in manifest.items():
        if name == "rope-table":
            continue
        data = golden(name)
        assert len(data) == entry["bytes"]
        assert hashlib.sha256(data).hexdigest() == entry["sha256"]


def quant_input() -> np.ndarray:
    x = np.zeros(32 * 6, dtype=np.float32)
    x[32], x[33], x[34], x[35] = 1.0, -1.0, 1.0, -1.0
    x[64], x[65], x[66], x[67], x[68] = 127.0, 0.5, -0.5, 1.5, -1.5
    x[96:99] = oracle.f32([0x34000000, 0x33800000, 0x33000000])
    x[128], x[129], x[130] = 126.5, -126.5, 63.25
    x[160] = np.float32(-0.0)
    x[161] = 0.0
    return x


def test_q8_quantizer_matches_fixture():
    stage = oracle.prepare_q8(quant_input())
    assert stage.tobytes() == golden("q8.bin")


def dot_inputs():
    mat = np.array([((i % 31) - 15) for i in range(64)], dtype=np.float32)
    mat[31], mat[63] = 127.0, -127.0
    q4 = np.zeros(36, dtype=np.uint8)
    q8 = np.zeros(68, dtype=np.uint8)
    for block in range(2):
        q4[block * 18:block * 18 + 2] = [0x00, 0x3C]
        for i in range(16):
            q4[block * 18 + 2 + i] = ((15 - i) << 4) | i
        q8[block * 34:block * 34 + 2] = [0x00, 0x3C]
        for i in range(32):
            q8[block * 34 + 2 + i] = ((i % 17) - 8) & 0xFF
    return mat, q4, q8


def test_q4_and_q8_matvec_match_fixture_words():
    mat, q4, q8 = dot_inputs()
    stage = oracle.prepare_q8(mat)
    y4 = oracle.q4_matvec(q4, stage, 1, 64)
    y8 = oracle.q8_matvec(q8, stage, 1, 64)
    assert oracle.bits(y4)[0] == 0x43E08000
    assert oracle.bits(y8)[0] == 0x44388000
    assert words(y4) + words(y8) == golden("dots.bin")


def test_rmsnorm_matches_fixture():
    x = np.array([((i % 17) - 8) / 8.0 for i in range(896)], dtype=np.float32)
    w = np.array([((i % 7) + 1) / 4.0 for i in range(896)], dtype=np.float32)
    y = oracle.rmsnorm(x, w)
    assert words(y) == golden("rms.bin")
    b = oracle.bits(y)
    assert (b[0], b[447], b[895]) == (0xBED15D27, 0xBF896521, 0x3F896521)


def test_swiglu_matches_fixture():
    g = np.array([((i % 33) - 16) / 16.0 for i in range(4864)], dtype=np.float32)
    u = np.array([((i % 19) - 9) / 8.0 for i in range(4864)], dtype=np.float32)
    y = oracle.swiglu(g, u)
    assert words(y) == golden("swiglu.bin")
    b = oracle.bits(y)
    assert (b[0], b[2431], b[4863]) == (0x3E9AE906, 0x3E800417, 0xBDFC2FB4)


def test_rope_table_is_the_pinned_table():
    table = oracle.rope_table()
    manifest = json.loads((GOLDEN / "manifest.json").read_text())["rope-table"]
    assert hashlib.sha256(table.tobytes()).hexdigest() == manifest["sha256"]
    b = table.view(np.uint32)
    for entry in manifest["selected_bits"]:
        at = (entry["position"] * 32 + entry["pair"]) * 2
        assert b[at] == int(entry["cos"], 16)
        assert b[at + 1] == int(entry["sin"], 16)


def test_rope_matches_fixture():
    v = np.array([(i - 32) / 16.0 for i in range(64)], dtype=np.float32)
    out = oracle.rope_in_place(v, 1, 511)
    assert words(out) == golden("rope.bin")
    last = oracle.rope_in_place(v, 1, 32767)
    assert hashlib.sha256(words(last)).hexdigest() == (
        "8121af7bd1111f604c69d651761737255b00bf43931b14c8fe64640bfd76aa61")


def attention_fixture_kv(capacity: int = 32768) -> np.ndarray:
    """tests.rs:4351-4368: rational K/V for positions 0..256 of layer 0."""
    kv = np.zeros(2 * 2 * capacity * 64, dtype=np.float32)
    p = np.arange(257)[:, None, None]
    h = np.arange(2)[None, :, None]
    c = np.arange(64)[None, None, :]
    kval = ((((p + c + h) % 29) - 14) / 32.0).astype(np.float32)
    vval = ((((p * 3 + c + h) % 31) - 15) / 32.0).astype(np.float32)
    value_words = 2 * capacity * 64
    kidx = ((h * (capacity // 4) + p // 4) * 64 + c) * 4 + p % 4
    vidx = value_words + (h * capacity + p) * 64 + c
    kv[kidx] = kval
    kv[vidx] = vval
    return kv


def attention_query() -> np.ndarray:
    return np.array([((i % 23) - 11) / 16.0 for i in range(896)], dtype=np.float32)


@pytest.mark.parametrize("capacity", [32768, 1024])
def test_attention_matches_fixtures(capacity):
    kv = attention_fixture_kv(capacity)
    q = attention_query()
    out, scores = oracle.attention(q, kv, capacity, 0, 2, 256)
    assert words(out) == golden("attention-256.bin")
    assert words(scores[:256]) == golden("scores-256.bin")
    q = np.roll(q, -7)
    out, scores = oracle.attention(q, kv, capacity, 0, 256, 512)
    assert words(out) == golden("attention-512.bin")
    assert words(scores[:512]) == golden("scores-512.bin")


def test_expf_edges_within_one_ulp():
    data = np.frombuffer(golden("expf-edge.u32le"), dtype=np.uint32).reshape(-1, 2)
    for x, expected in data:
        got = oracle.expf_bits(int(x))
        if expected & 0x7FFFFFFF == 0 or expected & 0x7F800000 == 0x7F800000:
            assert got == expected
        else:
            assert abs(int(got) - int(expected)) <= 1


def test_q4_block_dot_nibble_order_and_extrema():
    """tests.rs:3961-4023"""
    w = np.array([((15 - i) << 4) | i for i in range(16)], dtype=np.uint8)
    a = np.array([i + 1 if i < 16 else -(i - 15) for i in range(32)], dtype=np.int8)
    expected = sum(((int(w[i]) & 15) - 8) * int(a[i]) + ((int(w[i]) >> 4) - 8) * int(a[16 + i])
                   for i in range(16))
    assert oracle.q4_block_dot(w, a) == expected
    w = np.array([0x0F if i % 2 == 0 else 0xF0 for i in range(16)], dtype=np.uint8)
    a = np.array([-128 if (i < 16) == (i % 2 == 0) else 127 for i in range(32)], dtype=np.int8)
    expected = sum(((int(w[i]) & 15) - 8) * int(a[i]) + ((int(w[i]) >> 4) - 8) * int(a[16 + i])
                   for i in range(16))
    assert oracle.q4_block_dot(w, a) == expected


def test_block_dots_lcg_cases():
    """tests.rs:4053-4106 (256 LCG cases)"""
    state = 0x243F6A88

    def nxt():
        nonlocal state
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        return state >> 24

    for _ in range(256):
        q4w = np.array([nxt() for _ in range(16)], dtype=np.uint8)
        q8w = np.array([nxt() for _ in range(32)], dtype=np.uint8).view(np.int8)
        act = np.array([nxt() for _ in range(32)], dtype=np.uint8).view(np.int8)
        e4 = sum(((int(q4w[i]) & 15) - 8) * int(act[i]) + ((int(q4w[i]) >> 4) - 8) * int(act[16 + i])
                 for i in range(16))
        e8 = sum(int(q8w[i]) * int(act[i]) for i in range(32))
        assert oracle.q4_block_dot(q4w, act) == e4
        assert oracle.q8_block_dot(q8w, act) == e8
    w = np.array([-128 if i % 4 < 2 else 127 for i in range(32)], dtype=np.int8)
    a = np.array([-128 if i % 4 in (0, 2) else 127 for i in range(32)], dtype=np.int8)
    assert oracle.q8_block_dot(w, a) == 8


def kat_logits():
    logits = np.full(oracle.VOCAB, -100.0, dtype=np.float32)
    for t in range(41):
        logits[t] = np.float32(4.0) - np.float32(t) * np.float32(0.05)
    return logits


def test_sampler_state_known_answer():
    """tests.rs:424-466: 8 draws from 0x0123456789abcdef end in 0x37fe8664ce109d2f."""
    logits = kat_logits()
    st = oracle.SamplingState(0x0123456789ABCDEF)
    for _ in range(8):
        r = st.next_24()
        sel = oracle.sample_top_k_top_p(logits, r)
        assert sel < 20
    assert int(st.draws[0]) == 8
    assert int(st.state[0]) == 0x37FE8664CE109D2F
    assert int(oracle.SamplingState(0).state[0]) == 0x9E3779B97F4A7C15


def test_repetition_penalty_known_answer():
    """tests.rs:468-492"""
    logits = np.zeros(oracle.VOCAB, dtype=np.float32)
    logits[7], logits[9], logits[12] = 11.0, -2.0, np.float32(-0.0)
    seen = np.zeros(18992, dtype=np.uint8)
    st = oracle.SamplingState(1)
    status, _, _ = oracle.sample_with_repetition(logits, [7, 9, 7, 12, 9], st, seen)
    assert status == 0
    assert logits[7] == np.float32(11.0) / np.float32(1.1)
    assert logits[9] == np.float32(-2.0) * np.float32(1.1)
    assert oracle.bits(logits[12:13])[0] == 0x80000000
    assert not seen.any()
    assert int(st.draws[0]) == 1
    before = logits.copy()
    status, _, err = oracle.sample_with_repetition(logits, [oracle.VOCAB], st, seen)
    assert status == 3 and err.status == 3
    assert np.array_equal(before.view(np.uint32), logits.view(np.uint32))
    assert int(st.draws[0]) == 1


def test_sampler_selects_dominant_eos():
    """tests.rs:494-505"""
    logits = np.full(oracle.VOCAB, -100.0, dtype=np.float32)
    logits[151645] = 10.0
    logits[9] = 0.0
    for seed in [0, 1, 2**64 - 1, 0xFEEDFACEDEADBEEF]:
        st = oracle.SamplingState(seed)
        assert oracle.sample_top_k_top_p(logits, st.next_24()) == 151645


def test_kv_layout_matches_reference_formula():
    """tests.rs:612-676 at the reference capacity of 32768."""
    cap = 32768
    assert oracle.kv_word(cap, 23, 1, cap - 1, 1, 63) == 805306368 // 4 - 1
    for (layer, kind, pos, head, comp) in [(0, 0, 5, 1, 3), (23, 0, 32767, 0, 63), (1, 1, 256, 1, 7)]:
        base = layer * 2 * 2 * cap * 64
        if kind == 0:
            expected = base + (((head * (cap // 4) + pos // 4) * 64 + comp) * 4 + pos % 4)
        else:
            expected = base + 2 * cap * 64 + ((head * cap + pos) * 64 + comp)
        assert oracle.kv_word(cap, layer, kind, pos, head, comp) == expected
