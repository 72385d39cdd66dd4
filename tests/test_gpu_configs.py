"""Engine parity on the GPU at the benchmark configurations' own scale, against
the CPU oracle's restatement of inference.rs:1454-1765 and the sampler of
inference.rs:914-965 / fp32_sse2.rs:1787-1876.

* config 0 as specified: the 64-token prompt of default_rng(0x5eed0000), then
  64 sampled tokens with seed 1 in the REPL's order (sample with the whole
  history, then decode_selected; src/model_repl.rs:945-967), and a greedy
  stream of the same length (decode of the previous greedy id, the
  validate_inference.rs:449-529 harness) -- every id and the final logits bit
  for bit;
* config 3's batch: 256 sequences in one engine (the tensor-core tiles of every
  width live together), checked against the oracle on a spread of rows;
* the engine past the 2,048 positions of the shared-memory attention path, at
  2,100 prefilled positions and at config 4's ~31,000 positions over a seeded
  KV cache restored into a slot;
* the split attention launches of a 20-sequence batch past 256 positions.
"""
from __future__ import annotations

import concurrent.futures

import numpy as np
import pytest

import oracle
from promptboot_b200 import api, shard

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _oracle_greedy(model_image, prompt, steps, capacity):
    """Prefill, then `steps` decode(greedy) forwards: (ids, final logits)."""
    kv = np.zeros(24 * 4 * capacity * 64, dtype=np.float32)
    logits = None
    for i, t in enumerate(prompt):
        st, logits, _ = oracle.forward(model_image, kv, capacity, int(t), i, i + 1 == len(prompt))
        assert st == 0
    ids = [oracle.argmax(logits)]
    for s in range(steps):
        st, logits, _ = oracle.forward(model_image, kv, capacity, ids[-1], len(prompt) + s, True)
        assert st == 0
        ids.append(oracle.argmax(logits))
    return ids, logits


def test_config0_sampled_and_greedy_streams_match_oracle(model_view, model_image):
    """Config 0: 64-token prompt, 64 sampled tokens (seed 1), and a 64-step
    greedy stream, each in its own slot."""
    cap = 160
    prompt = shard.prompt_for(0, 64)
    with concurrent.futures.ThreadPoolExecutor(2) as pool:
        sampled_ref = pool.submit(oracle.generate, model_image, prompt, 64, 1, cap)
        greedy_ref = pool.submit(_oracle_greedy, model_image, prompt, 64, cap)

        eng = api.InferenceEngine(model_view, max_seqs=2, max_context=cap)
        # sampled stream, slot 0
        logits = np.zeros(api.VOCAB, dtype=np.uint32)
        eng.prefill(prompt, 80, logits, seq=0)
        seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
        state = api.SamplingState(1)
        history = list(prompt)
        got = []
        for i in range(64):
            tok = api.sample_token_with_repetition(logits, history, seen, state)
            got.append(tok)
            history.append(tok)
            if i < 63:
                eng.decode_selected(tok, logits, seq=0)
        # greedy stream, slot 1
        glogits = np.zeros(api.VOCAB, dtype=np.uint32)
        step = eng.prefill(prompt, 80, glogits, seq=1)
        greedy = [step.selected_token]
        for _ in range(64):
            step = eng.decode(greedy[-1], glogits, seq=1)
            greedy.append(step.selected_token)
        eng.close()

        st, ref_tokens, ref_logits, _ = sampled_ref.result()
        ref_greedy, ref_glogits = greedy_ref.result()
    assert st == 0
    assert got == list(ref_tokens)
    assert state.draws() == 64
    # the logits of the 64th draw after its repetition penalty, in place
    assert np.array_equal(logits, ref_logits.view(np.uint32))
    assert greedy == ref_greedy
    assert np.array_equal(glogits, ref_glogits.view(np.uint32))


def _oracle_row(model_image, prompt, seed, steps, capacity):
    """The engine's generate order for one sequence: prompt, then `steps` x
    (sample with the whole history, forward of the sampled id).  Returns the ids
    and the raw logits of the last forward."""
    kv = np.zeros(24 * 4 * capacity * 64, dtype=np.float32)
    logits = None
    for i, t in enumerate(prompt):
        st, logits, _ = oracle.forward(model_image, kv, capacity, int(t), i, i + 1 == len(prompt))
        assert st == 0
    state = oracle.SamplingState(seed)
    history = list(prompt)
    ids = []
    for s in range(steps):
        st, tok, _ = oracle.sample_with_repetition(logits, history, state)
        assert st == 0
        ids.append(tok)
        history.append(tok)
        st, logits, _ = oracle.forward(model_image, kv, capacity, tok, len(prompt) + s, True)
        assert st == 0
    return ids, logits


def test_config3_batch_of_256_matches_oracle_on_spread_rows(model_view, model_image):
    """256 sequences in one engine: 12-token prompts of the bench's generator
    (default_rng(0x5eed0000 + s)), seeds 0-255, three generate steps; rows 0, 7,
    8, 127 and 255 (first and last of 8- and 64-sequence tiles) against the
    oracle, ids and last logits bit for bit."""
    n, plen, steps, cap = 256, 12, 3, 32
    prompts = np.stack([shard.prompt_for(s, plen) for s in range(n)])
    rows = [0, 7, 8, 127, 255]
    with concurrent.futures.ThreadPoolExecutor(len(rows)) as pool:
        refs = [pool.submit(_oracle_row, model_image, prompts[r], shard.sampling_seed(r), steps, cap)
                for r in rows]
        eng = api.InferenceEngine(model_view, max_seqs=n, max_context=cap)
        status, _, errs = eng.prefill_batch(np.arange(n), prompts, 8)
        assert status == 0
        states = api.SamplingStates([shard.sampling_seed(s) for s in range(n)])
        status, out, errs = eng.generate(np.arange(n), states, steps)
        assert status == 0
        got_logits = {r: eng.logits(r) for r in rows}
        results = [fut.result() for fut in refs]
        # the greedy id of the last generate step (launched after the step's
        # graph) is the one decode continues from
        eng.decode(oracle.argmax(results[-1][1]), seq=rows[-1])
        eng.close()
        for r, (ids, logits) in zip(rows, results):
            assert list(out[:, r]) == ids, r
            assert np.array_equal(got_logits[r], logits.view(np.uint32)), r
            assert states[r].draws() == steps


def _kv_positions(kv: np.ndarray, capacity: int, positions) -> np.ndarray:
    """The K and V words of the given positions, every layer and head."""
    words = []
    for layer in range(24):
        for kind in range(2):
            for head in range(2):
                for p in positions:
                    idx = [oracle.kv_word(capacity, layer, kind, p, head, c) for c in range(64)]
                    words.append(kv[idx])
    return np.concatenate(words)


def test_engine_past_2048_positions_matches_oracle(model_view, model_image):
    """A 2,100-token prompt (batched prefill rows attend over more than the
    2,048 positions of the shared-memory path), then two decode_selected steps:
    the first 8 positions' KV against a fresh oracle run, and the logits of the
    last prompt position and of both decode steps against oracle forwards over
    the engine's own cache."""
    cap, n = 2112, 2100
    prompt = shard.prompt_for(77, n)
    eng = api.InferenceEngine(model_view, max_seqs=1, max_context=cap)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    eng.prefill(prompt, 4, logits)
    torch.cuda.synchronize()
    kv = eng.kv_tensor(0).cpu().numpy().copy()

    fresh = np.zeros_like(kv)
    for i in range(8):
        assert oracle.forward(model_image, fresh, cap, int(prompt[i]), i, False)[0] == 0
    assert np.array_equal(_kv_positions(kv, cap, range(8)).view(np.uint32),
                          _kv_positions(fresh, cap, range(8)).view(np.uint32))

    # the last prompt position, over the engine's KV of positions < n - 1
    work = kv.copy()
    st, ref, _ = oracle.forward(model_image, work, cap, int(prompt[-1]), n - 1, True)
    assert st == 0
    assert np.array_equal(logits, ref.view(np.uint32))
    assert np.array_equal(_kv_positions(work, cap, [n - 1]).view(np.uint32),
                          _kv_positions(kv, cap, [n - 1]).view(np.uint32))
    for i, token in enumerate((4242, 151000)):
        eng.decode_selected(token, logits)
        st, ref, _ = oracle.forward(model_image, work, cap, token, n + i, True)
        assert st == 0
        assert np.array_equal(logits, ref.view(np.uint32)), i
    eng.close()


def test_engine_restored_long_context_matches_oracle(model_view, model_image):
    """Config 4 scale: a slot restored at 30,000 positions over a seeded KV
    cache (the values the bench uses in place of a 30,000-token prefill), then
    two decode_selected steps against oracle forwards over the same cache."""
    cap, n = 30008, 30000
    prompt = shard.prompt_for(1000, n)
    eng = api.InferenceEngine(model_view, max_seqs=1, max_context=cap)
    region = eng.kv_tensor(0)
    g = torch.Generator(device="cuda").manual_seed(4)
    region.copy_(torch.randn(region.numel(), device="cuda", generator=g) * 0.5)
    torch.cuda.synchronize()
    kv = region.cpu().numpy().copy()
    eng.restore(prompt, 4)
    assert eng.position(0) == n
    with pytest.raises(api.InferenceError):
        eng.decode(0)  # no greedy id after a restore
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    for i, token in enumerate((17, 90000)):
        eng.decode_selected(token, logits)
        st, ref, _ = oracle.forward(model_image, kv, cap, token, n + i, True)
        assert st == 0
        assert np.array_equal(logits, ref.view(np.uint32)), i
    # the engine wrote the same K/V for the decoded positions
    torch.cuda.synchronize()
    got = region.cpu().numpy()
    assert np.array_equal(_kv_positions(got, cap, [n, n + 1]).view(np.uint32),
                          _kv_positions(kv, cap, [n, n + 1]).view(np.uint32))
    eng.close()


def test_engine_split_attention_batch_matches_oracle(model_view, model_image):
    """20 sequences past 256 positions: the engine's decode step takes the split
    attention launches (scores, softmax, the two-group PV launch that also
    quantizes the o-projection input); rows 0, 9 and 19 against oracle
    forwards over the engine's own KV, logits bit for bit."""
    n, plen, cap = 20, 300, 320
    prompts = np.stack([shard.prompt_for(200 + s, plen) for s in range(n)])
    eng = api.InferenceEngine(model_view, max_seqs=n, max_context=cap)
    status, _, errs = eng.prefill_batch(np.arange(n), prompts, 8)
    assert status == 0
    torch.cuda.synchronize()
    rows = [0, 9, 19]
    kvs = {r: eng.kv_tensor(r).cpu().numpy().copy() for r in rows}
    tokens = np.array([(1000 + 37 * s) % 151936 for s in range(n)], dtype=np.uint32)
    status, _, errs = eng.decode_batch(np.arange(n), tokens, require_greedy=False)
    assert status == 0
    got = {r: eng.logits(r) for r in rows}
    eng.close()
    for r in rows:
        st, ref, _ = oracle.forward(model_image, kvs[r], cap, int(tokens[r]), plen, True)
        assert st == 0
        assert np.array_equal(got[r], ref.view(np.uint32)), r


def test_sampler_expf_matches_reference_edges_and_dense_sweep():
    """The device exponential of the top-k/top-p weights (fp32_sse2.rs:404-469)
    against the reference's edge table (expf-edge.u32le, tests.rs:3293-3308)
    and, bit for bit, against the oracle over every 2^10-th binary32 in
    [-104, 0] plus the special inputs."""
    import ctypes
    import pathlib
    from promptboot_b200 import _lib
    lib = _lib.load()
    edge = np.frombuffer((pathlib.Path(__file__).parent / "golden" / "expf-edge.u32le").read_bytes(),
                         dtype=np.uint32).reshape(-1, 2)
    sweep = np.arange(0x80000000, 0xC2D00001, 1 << 10, dtype=np.uint64).astype(np.uint32)
    special = np.array([0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0x42B17218,
                        0x42B17217, 0xC2CFF1B5, 0xC2CFF1B4, 0x3EB17218, 0x3F851592, 0x39000000,
                        0x39000001, 0x00000001, 0x80000001], dtype=np.uint32)
    xs = np.concatenate([edge[:, 0], sweep, special])
    x_d = torch.from_numpy(xs.view(np.int32)).cuda()
    y_d = torch.zeros_like(x_d)
    assert lib.pb_expf_device(ctypes.c_void_p(x_d.data_ptr()), xs.size,
                              ctypes.c_void_p(y_d.data_ptr()), None) == 0
    got = y_d.cpu().numpy().view(np.uint32)
    ref = np.array([oracle.expf_bits(int(x)) for x in xs], dtype=np.uint32)
    nan = (ref & 0x7FFFFFFF) > 0x7F800000
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.all((got[nan] & 0x7FFFFFFF) > 0x7F800000)
    # and the reference's own table: exact at zeros/infinities, within 1 ulp elsewhere
    for (x, expected), g in zip(edge, got[:len(edge)]):
        if expected & 0x7FFFFFFF == 0 or expected & 0x7F800000 == 0x7F800000:
            assert g == expected
        else:
            assert abs(int(g) - int(expected)) <= 1
