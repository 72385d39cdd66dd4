"""Sampler parity on the GPU: the reference's known-answer tests
(tests.rs:368-599) through the host-buffer API, and a config-1-style batch
(N(0, 3^2) rows, five raised positions, 512-token histories, seed 7) through
the device batch API, every sampled id bit-exact to the CPU oracle."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import dev, ptr
from promptboot_b200 import _lib, api

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

V = api.VOCAB


def f32bits(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32)


def kat_logits():
    logits = np.full(V, -100.0, dtype=np.float32)
    for t in range(41):
        logits[t] = np.float32(4.0) - np.float32(t) * np.float32(0.05)
    return logits


def test_greedy_lowest_id_on_ties():
    logits = np.full(V, -100.0, dtype=np.float32)
    logits[7] = logits[3] = 1.5
    assert api.greedy_token(f32bits(logits)) == 3


@pytest.mark.parametrize("case", ["ties_across_threads", "signed_zero_max", "last_word", "random_dupes"])
def test_greedy_first_maximum_matches_oracle(case):
    """First maximum by strict > (lowest id among equal values, +0 == -0),
    across the vectorized scan's threads, iterations and tail."""
    rng = np.random.default_rng(sum(map(ord, case)))
    logits = (rng.standard_normal(V) * 2.0).astype(np.float32)
    if case == "ties_across_threads":
        for i in (4100, 4099, 151000, 4 * 1024 * 4 + 1):
            logits[i] = np.float32(9.5)
    elif case == "signed_zero_max":
        logits = -np.abs(logits) - np.float32(1.0)
        logits[77777] = np.float32(-0.0)
        logits[90001] = np.float32(0.0)
        logits[12] = np.float32(-0.0)
    elif case == "last_word":
        logits[V - 1] = np.float32(20.0)
    else:
        top = logits.max()
        logits[rng.choice(V, 6, replace=False)] = top
    assert api.greedy_token(f32bits(logits)) == oracle.argmax(logits)


def test_sampling_known_answer_state():
    logits = f32bits(kat_logits())
    first = api.SamplingState(0x0123456789ABCDEF)
    second = first.copy()
    ref = oracle.SamplingState(0x0123456789ABCDEF)
    for _ in range(8):
        a = api.sample_token(logits, first)
        assert a == api.sample_token(logits, second)
        assert a == oracle.sample_top_k_top_p(kat_logits(), ref.next_24())
        assert a < 20
    assert first == second and first.draws() == 8
    assert first.state() == 0x37FE8664CE109D2F


def test_repetition_penalty_known_answer():
    logits = np.zeros(V, dtype=np.float32)
    logits[7], logits[9], logits[12] = 11.0, -2.0, np.float32(-0.0)
    bits = f32bits(logits).copy()
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    st = api.SamplingState(1)
    api.sample_token_with_repetition(bits, [7, 9, 7, 12, 9], seen, st)
    assert bits[7] == f32bits(np.float32(11.0) / np.float32(1.1))
    assert bits[9] == f32bits(np.float32(-2.0) * np.float32(1.1))
    assert bits[12] == 0x80000000
    assert not seen.any() and st.draws() == 1


def test_dirty_seen_bitmap_follows_reference():
    """A token already marked in `seen` is not penalised, and is cleared after."""
    logits = np.linspace(-3, 3, V).astype(np.float32)
    a, b = f32bits(logits).copy(), logits.copy()
    seen_a = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    seen_a[5 // 8] |= 1 << (5 % 8)
    seen_b = seen_a.copy()
    s1, s2 = api.SamplingState(3), oracle.SamplingState(3)
    got = api.sample_token_with_repetition(a, [5, 6, 151935], seen_a, s1)
    status, ref, _ = oracle.sample_with_repetition(b, [5, 6, 151935], s2, seen_b)
    assert status == 0 and got == ref
    assert np.array_equal(a, f32bits(b)) and np.array_equal(seen_a, seen_b)


def test_dominant_eos_collapses_top_p():
    logits = np.full(V, -100.0, dtype=np.float32)
    logits[151645] = 10.0
    logits[9] = 0.0
    for seed in (0, 1, 2**64 - 1, 0xFEEDFACEDEADBEEF):
        st = api.SamplingState(seed)
        assert api.sample_token(f32bits(logits), st) == 151645 and st.draws() == 1


def test_top_logits_8_order_and_signed_zero():
    logits = np.full(V, -100.0, dtype=np.float32)
    for t, v in [(7, 9.0), (2, 9.0), (11, 8.0), (4, 7.0), (15, 6.0), (5, 5.0), (20, 4.0),
                 (6, 3.0), (30, 2.0)]:
        logits[t] = v
    got = api.top_logits_8(f32bits(logits))
    assert got == [(t, int(f32bits(np.float32(v)))) for t, v in
                   [(2, 9.0), (7, 9.0), (11, 8.0), (4, 7.0), (15, 6.0), (5, 5.0), (20, 4.0), (6, 3.0)]]
    logits = np.full(V, -100.0, dtype=np.float32)
    logits[1:9] = [-0.0, 0.0, -1, -2, -3, -4, -5, -6]
    got = api.top_logits_8(f32bits(logits))
    assert [t for t, _ in got] == [1, 2, 3, 4, 5, 6, 7, 8]
    assert got[0][1] == 0x80000000 and got[1][1] == 0


def config1_batch(rows: int, seed: int = 7):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    for r in range(rows):
        logits[r, rng.choice(V, size=5, replace=False)] += np.float32(12.0)
    history = rng.integers(0, V, size=(rows, 512), dtype=np.uint32)
    return logits, history


@pytest.mark.parametrize("rows", [1, 256])
def test_device_batch_sampler_matches_oracle(rows):
    logits, history = config1_batch(rows)
    lib = _lib.load()
    d_logits = dev(logits)
    d_hist = dev(history.reshape(-1))
    offsets = np.arange(rows, dtype=np.uint64) * 512
    lengths = np.full(rows, 512, dtype=np.uint32)
    # one SamplingState(7) drawn once per row in row order (row r uses draw r+1)
    master = oracle.SamplingState(7)
    states = np.zeros((rows, 2), dtype=np.uint64)
    draws = []
    for r in range(rows):
        st_before = int(master.state[0])
        draws.append(master.next_24())
        states[r] = [st_before, r]
    d_states = dev(states)
    out = torch.zeros((rows, 4), dtype=torch.int32, device="cuda")
    assert lib.pb_sample_batch_device(ptr(d_logits), V, rows, ptr(d_hist), ptr(dev(offsets)),
                                      ptr(dev(lengths)), ptr(d_states), ptr(out), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    mutated = d_logits.cpu().numpy()
    for r in range(rows):
        ref_logits = logits[r].copy()
        seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
        oracle.lib().orc_apply_repetition_penalty(oracle._p(ref_logits), oracle._p(history[r]),
                                                  512, oracle._p(seen))
        ref = oracle.sample_top_k_top_p(ref_logits, draws[r])
        assert got[r, 0] == 0 and got[r, 3] == ref, r
        assert got[r, 2] == draws[r]
        assert np.array_equal(f32bits(mutated[r]), f32bits(ref_logits)), r


def test_device_batch_sampler_rejects_rows_transactionally():
    logits, history = config1_batch(3, seed=8)
    logits[1, 1234] = np.inf
    history[2, 17] = V + 5
    lib = _lib.load()
    d_logits = dev(logits)
    states = np.array([[11, 0], [12, 0], [13, 0]], dtype=np.uint64)
    d_states = dev(states)
    out = torch.zeros((3, 4), dtype=torch.int32, device="cuda")
    assert lib.pb_sample_batch_device(ptr(d_logits), V, 3, ptr(dev(history.reshape(-1))),
                                      ptr(dev(np.arange(3, dtype=np.uint64) * 512)),
                                      ptr(dev(np.full(3, 512, dtype=np.uint32))), ptr(d_states),
                                      ptr(out), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    st = d_states.cpu().numpy().view(np.uint64)
    assert got[0, 0] == 0 and st[0, 1] == 1
    assert list(got[1, :3]) == [7, 1234, 0x7F800000] and list(st[1]) == [12, 0]
    assert list(got[2, :3]) == [3, 17, V + 5] and list(st[2]) == [13, 0]
    after = d_logits.cpu().numpy()
    assert np.array_equal(f32bits(after[1]), f32bits(logits[1]))
    assert np.array_equal(f32bits(after[2]), f32bits(logits[2]))


def test_device_batch_sampler_reports_first_nonfinite_word():
    """The first non-finite logit in index order (its bits as stored) across the
    row's warp segments and the unaligned tail; rows without one still sample."""
    logits, history = config1_batch(4, seed=9)
    nan_bits = np.array([0x7FC00123], dtype=np.uint32).view(np.float32)[0]
    logits[0, 150000] = nan_bits
    logits[0, 70001] = -np.inf
    logits[0, 90000] = np.inf
    logits[1, 5] = nan_bits
    logits[2, V - 1] = np.inf
    lib = _lib.load()
    d_logits = dev(logits)
    states = np.array([[21, 0], [22, 0], [23, 0], [24, 0]], dtype=np.uint64)
    d_states = dev(states)
    out = torch.zeros((4, 4), dtype=torch.int32, device="cuda")
    assert lib.pb_sample_batch_device(ptr(d_logits), V, 4, ptr(dev(history.reshape(-1))),
                                      ptr(dev(np.arange(4, dtype=np.uint64) * 512)),
                                      ptr(dev(np.full(4, 512, dtype=np.uint32))), ptr(d_states),
                                      ptr(out), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    st = d_states.cpu().numpy().view(np.uint64)
    assert list(got[0, :3]) == [7, 70001, 0xFF800000] and list(st[0]) == [21, 0]
    assert list(got[1, :3]) == [7, 5, 0x7FC00123] and list(st[1]) == [22, 0]
    assert list(got[2, :3]) == [7, V - 1, 0x7F800000] and list(st[2]) == [23, 0]
    assert got[3, 0] == 0 and st[3, 1] == 1
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    ref_logits = logits[3].copy()
    oracle.lib().orc_apply_repetition_penalty(oracle._p(ref_logits), oracle._p(history[3]), 512,
                                              oracle._p(seen))
    master = oracle.SamplingState(24)
    assert got[3, 3] == oracle.sample_top_k_top_p(ref_logits, master.next_24())


@pytest.mark.parametrize("case", ["all_equal", "signed_zero_top", "duplicate_top", "penalty_ties"])
def test_device_batch_sampler_ties_match_oracle(case):
    """Top-20 ties resolved by the lower id (strict >), signed zeros equal, and
    ties the repetition penalty creates, against the oracle for 4 rows."""
    rows = 4
    rng = np.random.default_rng(sum(map(ord, case)))
    logits = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    history = rng.integers(0, V, size=(rows, 512), dtype=np.uint32)
    if case == "all_equal":
        logits[:] = np.float32(1.25)
    elif case == "signed_zero_top":
        logits = -np.abs(logits) - np.float32(1.0)
        for r in range(rows):
            idx = rng.choice(V, 30, replace=False)
            logits[r, idx[:15]] = np.float32(0.0)
            logits[r, idx[15:]] = np.float32(-0.0)
    elif case == "duplicate_top":
        for r in range(rows):
            logits[r, rng.choice(V, 40, replace=False)] = np.float32(14.0)
    else:
        # x / 1.1 of a penalised token lands exactly on an unpenalised value
        for r in range(rows):
            t = int(history[r, 0])
            logits[r, t] = np.float32(11.0)
            logits[r, rng.choice(V, 25, replace=False)] = np.float32(np.float32(11.0) / np.float32(1.1))
    lib = _lib.load()
    d_logits = dev(logits)
    master = oracle.SamplingState(99)
    states = np.zeros((rows, 2), dtype=np.uint64)
    draws = []
    for r in range(rows):
        states[r] = [int(master.state[0]), r]
        draws.append(master.next_24())
    out = torch.zeros((rows, 4), dtype=torch.int32, device="cuda")
    assert lib.pb_sample_batch_device(ptr(d_logits), V, rows, ptr(dev(history.reshape(-1))),
                                      ptr(dev(np.arange(rows, dtype=np.uint64) * 512)),
                                      ptr(dev(np.full(rows, 512, dtype=np.uint32))), ptr(dev(states)),
                                      ptr(out), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint32)
    mutated = d_logits.cpu().numpy()
    for r in range(rows):
        ref_logits = logits[r].copy()
        seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
        oracle.lib().orc_apply_repetition_penalty(oracle._p(ref_logits), oracle._p(history[r]),
                                                  512, oracle._p(seen))
        assert got[r, 0] == 0 and got[r, 3] == oracle.sample_top_k_top_p(ref_logits, draws[r]), r
        assert np.array_equal(f32bits(mutated[r]), f32bits(ref_logits)), r


@pytest.mark.parametrize("case", ["all_equal", "signed_zero_top", "duplicate_top", "penalty_ties",
                                  "slice_edges", "nonfinite_late"])
def test_split_row_sampler_matches_oracle(case):
    """The host-buffer sampler, which splits the row's vocabulary over several
    CTAs and merges their top-20 lists: the tie cases above, the best values
    on the slice boundaries (ids 4863/4864, the last id), and a non-finite word
    in the last slice (the reference's first-non-finite error)."""
    rng = np.random.default_rng(sum(map(ord, case)) + 5)
    logits = (rng.standard_normal(V) * 3.0).astype(np.float32)
    history = rng.integers(0, V, size=300, dtype=np.uint32)
    if case == "all_equal":
        logits[:] = np.float32(1.25)
    elif case == "signed_zero_top":
        logits = -np.abs(logits) - np.float32(1.0)
        idx = rng.choice(V, 30, replace=False)
        logits[idx[:15]] = np.float32(0.0)
        logits[idx[15:]] = np.float32(-0.0)
    elif case == "duplicate_top":
        logits[rng.choice(V, 40, replace=False)] = np.float32(14.0)
    elif case == "penalty_ties":
        logits[int(history[0])] = np.float32(11.0)
        logits[rng.choice(V, 25, replace=False)] = np.float32(np.float32(11.0) / np.float32(1.1))
    elif case == "slice_edges":
        for i, t in enumerate([4863, 4864, 9727, 9728, V - 1, 0, 150783, 150784]):
            logits[t] = np.float32(13.0 - 0.25 * (i % 3))
        history[:3] = [4864, V - 1, 0]
    else:
        logits[V - 7] = np.float32(np.inf)
    bits = f32bits(logits).copy()
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    state = api.SamplingState(31)
    ref = logits.copy()
    ref_state = oracle.SamplingState(31)
    st_ref, id_ref, err_ref = oracle.sample_with_repetition(ref, history, ref_state)
    if case == "nonfinite_late":
        assert st_ref != 0
        with pytest.raises(api.InferenceError) as exc:
            api.sample_token_with_repetition(bits, history, seen, state)
        e = exc.value
        assert (e.status, e.domain, e.available, e.detail) == \
            (err_ref.status, err_ref.domain, err_ref.available, err_ref.detail)
        return
    assert st_ref == 0
    got = api.sample_token_with_repetition(bits, history, seen, state)
    assert got == id_ref
    assert state.state() == int(ref_state.state[0]) and state.draws() == 1
    assert np.array_equal(bits, f32bits(ref))
