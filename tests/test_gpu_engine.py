"""End-to-end engine parity on the GPU against the CPU oracle's restatement of
inference.rs:1454-1765, plus the state machine and error semantics of
inference.rs:967-1371 and host-side fault injection (a NaN planted in a weight
of the model image, never a device fault)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from promptboot_b200 import api, pbtqw25

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NO = 0xFFFFFFFF
CAP = 256


def prompt(n, seed=0x5EED0000):
    return np.random.default_rng(seed).integers(0, 151643, size=n, dtype=np.uint32)


@pytest.fixture(scope="module")
def engine(model_view):
    e = api.InferenceEngine(model_view, max_seqs=4, max_context=CAP)
    yield e
    e.close()


def oracle_prefill_logits(model_image, tokens):
    kv = np.zeros(24 * 2 * 2 * CAP * 64, dtype=np.float32)
    logits = None
    for i, t in enumerate(tokens):
        st, logits, err = oracle.forward(model_image, kv, CAP, int(t), i, i + 1 == len(tokens))
        assert st == 0
    return logits, kv


def test_prefill_and_decode_logits_bit_exact(engine, model_image):
    toks = prompt(6)
    engine.reset(0)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    step = engine.prefill(toks, 8, logits)
    ref, kv = oracle_prefill_logits(model_image, toks)
    assert np.array_equal(logits, ref.view(np.uint32))
    assert step.position == 6 and step.selected_token == oracle.argmax(ref)
    assert step.selected_logit_bits == int(ref.view(np.uint32)[step.selected_token])
    # decode_selected of an arbitrary token, then decode of the greedy one
    for i, token in enumerate([12345, None, None]):
        token = step.selected_token if token is None else token
        fn = engine.decode if i else engine.decode_selected
        step = fn(token, logits)
        st, ref, _ = oracle.forward(model_image, kv, CAP, token, 6 + i, True)
        assert st == 0
        assert np.array_equal(logits, ref.view(np.uint32)), i
        assert step.selected_token == oracle.argmax(ref) and step.position == 7 + i


def test_repl_generation_matches_oracle(engine, model_image):
    """src/model_repl.rs:927-1000 semantics: sample with the full history after
    every step, then decode_selected(sampled)."""
    toks = prompt(5, seed=3)
    engine.reset(1)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    engine.prefill(toks, 16, logits, seq=1)
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    state = api.SamplingState(1)
    history = list(toks)
    got = []
    for i in range(6):
        sel = api.sample_token_with_repetition(logits, history, seen, state)
        got.append(sel)
        history.append(sel)
        if i < 5:
            engine.decode_selected(sel, logits, seq=1)
    st, ref_tokens, _, _ = oracle.generate(model_image, toks, 6, 1, CAP)
    assert st == 0
    assert got == list(ref_tokens)
    assert state.draws() == 6


def test_batched_device_generation_matches_oracle(model_view, model_image):
    e = api.InferenceEngine(model_view, max_seqs=3, max_context=64)
    prompts = np.stack([prompt(7, seed=s) for s in (10, 11, 12)])
    status, steps, errs = e.prefill_batch([0, 1, 2], prompts, 32)
    assert status == 0
    states = [api.SamplingState(s) for s in (0, 5, 9)]
    status, out, errs = e.generate([0, 1, 2], states, 5)
    assert status == 0
    for i, seed in enumerate((0, 5, 9)):
        st, ref, _, _ = oracle.generate(model_image, prompts[i], 5, seed, 64)
        assert st == 0 and list(out[:, i]) == list(ref), i
        assert states[i].draws() == 5
        assert e.position(i) == 7 + 5
    e.close()


def test_tensor_core_batch_generation_matches_oracle(model_view, model_image):
    """12 sequences: every layer matvec and the lm_head run on the tcgen05 path."""
    n = 12
    e = api.InferenceEngine(model_view, max_seqs=n, max_context=32)
    prompts = np.stack([prompt(5, seed=100 + s) for s in range(n)])
    status, steps, errs = e.prefill_batch(list(range(n)), prompts, 16)
    assert status == 0
    rows = [e.logits(i) for i in range(n)]
    for i in (0, n - 1):
        ref, _ = oracle_prefill_logits(model_image, prompts[i])
        assert np.array_equal(rows[i], ref.view(np.uint32)), i
    states = [api.SamplingState(s) for s in range(n)]
    status, out, errs = e.generate(list(range(n)), states, 3)
    assert status == 0
    ref = oracle.generate_many(model_image, prompts, 4, np.arange(n), 32, oracle.cpu_cores())
    assert np.array_equal(out, ref[:, :3].T)
    e.close()


@pytest.mark.parametrize("batch", [False, True])
def test_engine_sample_matches_host_sampler(model_view, batch):
    """Per-row SamplingState objects, or one contiguous SamplingStates batch
    (updated in place)."""
    e = api.InferenceEngine(model_view, max_seqs=2, max_context=64)
    prompts = np.stack([prompt(4, seed=20), prompt(4, seed=21)])
    assert e.prefill_batch([0, 1], prompts, 8)[0] == 0
    rows = [e.logits(0), e.logits(1)]
    states = api.SamplingStates([7, 8]) if batch else [api.SamplingState(7), api.SamplingState(8)]
    st, ids, errs = e.sample([0, 1], states)
    assert st == 0
    for i in range(2):
        ref_state = api.SamplingState(7 + i)
        seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
        ref = api.sample_token_with_repetition(rows[i].copy(), prompts[i], seen, ref_state)
        assert ids[i] == ref and states[i] == ref_state
    e.close()


def test_state_machine_errors_match_reference(model_view):
    """inference.rs:1026-1371 prechecks (tests.rs:883-1768 shapes, synthetic model)."""
    e = api.InferenceEngine(model_view, max_seqs=1, max_context=64)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    with pytest.raises(api.InferenceError) as x:
        e.decode_selected(1, logits)
    assert x.value.tuple() == [1, 2, NO, 0, NO, 1, 0, (1 << 32) | 0]
    with pytest.raises(api.InferenceError) as x:
        e.append_prefill([1], 4, logits)
    assert x.value.tuple() == [1, 2, NO, 0, NO, 1, 0, (1 << 32) | 0]
    with pytest.raises(api.InferenceError) as x:
        e.prefill([1, 2], 0, logits)
    assert x.value.tuple() == [2, 2, NO, 0, NO, 1, 0, (11 << 32) | 0]
    with pytest.raises(api.InferenceError) as x:
        e.prefill([], 4, logits)
    assert x.value.tuple() == [2, 2, NO, 0, NO, 1, 0, (3 << 32) | 0]
    with pytest.raises(api.InferenceError) as x:
        e.prefill([1, 2, 3], 62, logits)
    assert x.value.tuple() == [2, 2, NO, 0, NO, 64, 65, (3 << 32) | 1]
    with pytest.raises(api.InferenceError) as x:
        e.prefill([1, 151936], 4, logits)
    assert x.value.tuple() == [3, 2, NO, 1, NO, 151936, 151936, (2 << 32) | 0]
    assert e.usage().state == 0 and e.position() == 0
    step = e.prefill([5, 6, 7], 2, logits)
    assert e.usage().state in (1, 2) and e.position() == 3
    with pytest.raises(api.InferenceError) as x:
        e.prefill([1], 4, logits)
    assert x.value.tuple()[:2] == [1, 2] and x.value.detail == (1 << 32) | 1
    wrong = (step.selected_token + 1) % api.VOCAB
    with pytest.raises(api.InferenceError) as x:
        e.decode(wrong, logits)
    assert x.value.tuple() == [1, 19, NO, 3, NO, step.selected_token, wrong, (14 << 32) | 0]
    with pytest.raises(api.InferenceError) as x:
        e.decode_selected(151936, logits)
    assert x.value.tuple() == [3, 2, NO, 3, NO, 151936, 151936, (2 << 32) | 1]
    e.decode_selected(9, logits)  # second prediction of reserve 2
    with pytest.raises(api.InferenceError) as x:
        e.decode_selected(9, logits)
    assert x.value.tuple() == [2, 2, NO, 4, NO, 2, 2, (11 << 32) | 1]
    u = e.usage()
    assert (u.position, u.context_limit, u.generation_reserve) == (4, 64, 2)
    assert u.kv.current == 4 * 24576 and u.kv.high_water == 4 * 24576
    e.reset()
    assert e.usage().state == 0 and e.position() == 0
    e.close()


def test_retained_prefix_reuse_is_exact(model_view, model_image):
    """prefill_with_prefix / reset_to_prefix (inference.rs:1044-1093, 1315-1335)."""
    e = api.InferenceEngine(model_view, max_seqs=1, max_context=64)
    a = np.concatenate([prompt(4, seed=30), prompt(3, seed=31)])
    b = np.concatenate([a[:4], prompt(2, seed=32)])
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    e.prefill_with_prefix(a, 4, 8, logits)
    e.decode_selected(17, logits)
    assert e.reset_to_prefix() == 4 and e.position() == 4
    e.prefill_with_prefix(b, 4, 8, logits)
    ref, _ = oracle_prefill_logits(model_image, b)
    assert np.array_equal(logits, ref.view(np.uint32))
    with pytest.raises(api.InferenceError) as x:
        e.prefill_with_prefix(b, 0, 8, logits)
    assert x.value.tuple() == [2, 2, NO, 0, NO, 1, 0, (3 << 32) | 3]
    assert e.position() == 0 and e.reset_to_prefix() == 0
    e.close()


def test_nonfinite_weight_faults_with_reference_error(model_image):
    """inference.rs:1889-1944: a NaN in layer 2's FFN norm weight faults the FFN_NORM
    stage of layer 2 at element 5; logits are zeroed and only reset recovers."""
    img = model_image.copy()
    tid = pbtqw25.layer_tensor(2, 14)
    off = int(np.frombuffer(img[pbtqw25.TENSOR_DIR + tid * 96 + 32:][:8].tobytes(), np.uint64)[0])
    img[off + 5 * 4:off + 6 * 4] = np.frombuffer(np.uint32(0x7FC00000).tobytes(), np.uint8)
    view = api.ModelView(img)
    e = api.InferenceEngine(view, max_seqs=1, max_context=64)
    logits = np.ones(api.VOCAB, dtype=np.uint32)
    with pytest.raises(api.InferenceError) as x:
        e.prefill([1, 2, 3], 4, logits)
    # status, domain, layer, position, tensor and index are the reference's; the
    # NaN's payload is the GPU's canonical NaN rather than x86's propagated one.
    t = x.value.tuple()
    assert t[:6] == [6, 12, 2, 0, tid, 0] and t[7] == (7 << 32) | 5
    assert t[6] & 0x7F800000 == 0x7F800000 and t[6] & 0x7FFFFF
    assert not logits.any()
    assert e.usage().state == 3
    with pytest.raises(api.InferenceError) as x:
        e.decode_selected(1, logits)
    assert x.value.tuple()[:2] == [1, 2] and x.value.detail == (1 << 32) | 3
    e.close()
    view.close()


def test_tensor_core_up_stage_fault_matches_cuda_core_path(model_image):
    """An infinite binary16 scale in one block of layer 1's up matrix (row 100)
    makes the UP stage fail at element 100.  The tensor-core path (12 sequences;
    its Q4_0 epilogue falls back from the fma form for a non-finite scale)
    reports the same error tuple, value bits included, as the CUDA-core path
    (1 sequence)."""
    img = model_image.copy()
    tid = pbtqw25.layer_tensor(1, 13)
    off = int(np.frombuffer(img[pbtqw25.TENSOR_DIR + tid * 96 + 32:][:8].tobytes(), np.uint64)[0])
    blk = off + (100 * 28 + 3) * 18
    img[blk:blk + 2] = np.frombuffer(np.uint16(0x7C00).tobytes(), np.uint8)
    view = api.ModelView(img)
    p = prompt(3, seed=5)
    e1 = api.InferenceEngine(view, max_seqs=1, max_context=64)
    with pytest.raises(api.InferenceError) as x:
        e1.prefill(p, 4, np.zeros(api.VOCAB, dtype=np.uint32))
    t1 = x.value.tuple()
    assert t1[:6] == [6, 14, 1, 0, tid, 0] and t1[7] == (7 << 32) | 100
    e1.close()
    n = 12
    e12 = api.InferenceEngine(view, max_seqs=n, max_context=64)
    seqs = np.arange(n, dtype=np.uint32)
    status, _, errs = e12.prefill_batch(seqs, np.stack([p] * n), 4)
    assert status != 0
    for er in errs:
        t = er.tuple()
        assert t[:6] == t1[:6] and t[7] == t1[7]
        assert t[6] & 0x7F800000 == 0x7F800000
        if t1[6] & 0x7FFFFF == 0:  # an infinity: identical bits on both paths
            assert t[6] == t1[6]
    e12.close()
    view.close()


def test_batched_prefill_faults_each_sequence_at_its_position(model_image):
    """Prompt positions but the last run as one batched forward of (sequence,
    position) rows.  A NaN embedding scale of token 777 faults each sequence at
    the EMBEDDING stage of the position where 777 first appears (0, 3, or the
    last position 7); a sequence without it still matches the oracle."""
    img = model_image.copy()
    off = int(np.frombuffer(img[pbtqw25.TENSOR_DIR + 0 * 96 + 32:][:8].tobytes(), np.uint64)[0])
    blk = off + 777 * 28 * 18
    img[blk:blk + 2] = np.frombuffer(np.uint16(0x7E00).tobytes(), np.uint8)
    view = api.ModelView(img)
    n, plen = 4, 8
    prompts = np.stack([prompt(plen, seed=700 + i) for i in range(n)])
    prompts[prompts == 777] = 778
    prompts[1, 3] = 777
    prompts[1, 5] = 777
    prompts[2, 0] = 777
    prompts[3, 7] = 777
    e = api.InferenceEngine(view, max_seqs=n, max_context=64)
    status, steps, errs = e.prefill_batch(np.arange(n), prompts, 4)
    assert status == 6
    assert errs[0].status == 0
    for i, p in [(1, 3), (2, 0), (3, 7)]:
        t = errs[i].tuple()
        assert t[:6] == [6, 3, NO, p, 0, 0] and t[7] == (7 << 32) | 0, (i, t)
        assert t[6] & 0x7F800000 == 0x7F800000 and t[6] & 0x7FFFFF
        assert e.usage(i).state == 3
    ref, _ = oracle_prefill_logits(model_image, prompts[0])
    assert np.array_equal(e.logits(0), ref.view(np.uint32))
    assert steps[0].selected_token == oracle.argmax(ref) and steps[0].position == plen
    e.close()
    view.close()


def test_batched_calls_reject_a_sequence_listed_twice(model_image):
    """Two rows of one slot would write the same KV position: the batched entry
    points refuse duplicates with PB_CAPACITY before touching any state."""
    view = api.ModelView(model_image)
    e = api.InferenceEngine(view, max_seqs=4, max_context=32)
    seqs = np.array([0, 1, 0], dtype=np.uint32)
    st, _, _ = e.prefill_batch(seqs, np.stack([prompt(3, seed=i) for i in range(3)]), 4)
    assert st == 4 and e.position(0) == 0 and e.position(1) == 0
    st, _, _ = e.prefill_batch(np.array([0, 1], dtype=np.uint32), np.stack([prompt(3), prompt(3, 9)]), 4)
    assert st == 0
    st, _, _ = e.decode_batch(seqs, np.array([1, 2, 3], dtype=np.uint32))
    assert st == 4 and e.position(0) == 3
    e.close()
    view.close()


def test_repl_loop_allocates_no_device_memory(model_view):
    """100 REPL-style iterations (sample_token_with_repetition on host logits,
    then decode_selected; src/model_repl.rs:945-967) leave the device's free
    memory unchanged once the first iteration has set up the thread's sampler
    buffers."""
    e = api.InferenceEngine(model_view, max_seqs=1, max_context=256)
    toks = prompt(8, seed=55)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    e.prefill(toks, 120, logits)
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    state = api.SamplingState(3)
    history = list(toks)

    def one():
        tok = api.sample_token_with_repetition(logits, history, seen, state)
        history.append(tok)
        e.decode_selected(tok, logits)
        api.greedy_token(logits)
        api.top_logits_8(logits)

    one()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(100):
        one()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    e.close()
