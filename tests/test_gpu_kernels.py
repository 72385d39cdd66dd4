"""Kernel parity on the GPU: each sm_100a kernel against the reference's golden
vectors (tests/golden) and against the CPU oracle on seeded random inputs.
The bar is bit-exact binary32 output."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import dev, ptr
from promptboot_b200 import _lib
from test_oracle_golden import (GOLDEN, attention_fixture_kv, attention_query, dot_inputs,
                                quant_input)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def sync():
    torch.cuda.synchronize()


def host(t) -> np.ndarray:
    return t.cpu().numpy()


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32)


def test_quantizer_matches_fixture_and_oracle():
    lib = _lib.load()
    x = quant_input()[None, :]
    out = torch.zeros(6 * 34, dtype=torch.uint8, device="cuda")
    assert lib.pb_quantize_q8_device(ptr(dev(x)), 1, 192, ptr(out), None) == 0
    sync()
    assert host(out).tobytes() == (GOLDEN / "q8.bin").read_bytes()
    rng = np.random.default_rng(11)
    for cols in (896, 4864):
        x = (rng.standard_normal((5, cols)) * rng.choice([1e-3, 1.0, 40.0], size=(5, 1))).astype(np.float32)
        x[0, :32] = 0.0
        out = torch.zeros(5 * cols // 32 * 34, dtype=torch.uint8, device="cuda")
        assert lib.pb_quantize_q8_device(ptr(dev(x)), 5, cols, ptr(out), None) == 0
        sync()
        got = host(out).reshape(5, -1)
        for r in range(5):
            assert np.array_equal(got[r], oracle.prepare_q8(x[r])), (cols, r)


def test_quantizer_extreme_scales_match_oracle():
    """Scales d = amax / 127 in the binary16 subnormal range, rounding to zero,
    overflowing binary16 to inf, and rows with inf / NaN words."""
    lib = _lib.load()
    rng = np.random.default_rng(12)
    rows = []
    for amax in (127 * 2.0 ** -20, 127 * 2.0 ** -23, 1e-40, 1e-30, 3e-3, 8.3e6, 1e7, 3e38):
        x = rng.uniform(-1.0, 1.0, 896) * amax
        x[::32] = amax
        rows.append(x.astype(np.float32))
    special = rng.standard_normal(896).astype(np.float32)
    special[5] = np.inf
    special[40] = np.nan
    special[70] = -np.inf
    rows.append(special)
    x = np.stack(rows)
    out = torch.zeros(len(rows) * 28 * 34, dtype=torch.uint8, device="cuda")
    assert lib.pb_quantize_q8_device(ptr(dev(x)), len(rows), 896, ptr(out), None) == 0
    sync()
    got = host(out).reshape(len(rows), -1)
    for r in range(len(rows)):
        assert np.array_equal(got[r], oracle.prepare_q8(x[r])), r


def test_rmsnorm_matches_fixture_and_oracle():
    lib = _lib.load()
    x = np.array([((i % 17) - 8) / 8.0 for i in range(896)], dtype=np.float32)
    w = np.array([((i % 7) + 1) / 4.0 for i in range(896)], dtype=np.float32)
    rng = np.random.default_rng(5)
    xs = np.stack([x] + [rng.standard_normal(896).astype(np.float32) * s for s in (1e-3, 1.0, 30.0)])
    y = torch.zeros((4, 896), dtype=torch.float32, device="cuda")
    assert lib.pb_rmsnorm_device(ptr(dev(xs)), ptr(dev(w)), 4, ptr(y), None) == 0
    sync()
    got = host(y)
    assert got[0].tobytes() == (GOLDEN / "rms.bin").read_bytes()
    for r in range(4):
        assert np.array_equal(u32(got[r]), u32(oracle.rmsnorm(xs[r], w)))


def test_rmsnorm_wide_exponent_range_matches_oracle():
    """Squares spanning more than 19 binades take the serial f64 sum (the
    reference's order); narrow rows take the exact tree sum.  Both bit-exact."""
    lib = _lib.load()
    rng = np.random.default_rng(77)
    rows = []
    for lo, hi in [(-60, 20), (-30, 0), (-8, 2), (-1, 1), (-126, -100)]:
        m = rng.uniform(1.0, 2.0, 896) * rng.choice([-1.0, 1.0], 896)
        rows.append((m * np.exp2(rng.integers(lo, hi + 1, 896))).astype(np.float32))
    rows[1][::7] = 0.0
    xs = np.stack(rows)
    w = rng.uniform(0.5, 1.5, 896).astype(np.float32)
    y = torch.zeros((len(rows), 896), dtype=torch.float32, device="cuda")
    assert lib.pb_rmsnorm_device(ptr(dev(xs)), ptr(dev(w)), len(rows), ptr(y), None) == 0
    sync()
    got = host(y)
    for r in range(len(rows)):
        assert np.array_equal(u32(got[r]), u32(oracle.rmsnorm(xs[r], w))), r


def test_swiglu_matches_fixture_and_oracle():
    lib = _lib.load()
    g = np.array([((i % 33) - 16) / 16.0 for i in range(4864)], dtype=np.float32)
    u = np.array([((i % 19) - 9) / 8.0 for i in range(4864)], dtype=np.float32)
    rng = np.random.default_rng(9)
    g2 = (rng.standard_normal(4864) * 30).astype(np.float32)
    g2[:4] = [-200.0, 200.0, 0.0, -0.0]
    u2 = rng.standard_normal(4864).astype(np.float32)
    out = torch.zeros((2, 4864), dtype=torch.float32, device="cuda")
    assert lib.pb_swiglu_device(ptr(dev(np.stack([g, g2]))), ptr(dev(np.stack([u, u2]))), 2,
                                ptr(out), None) == 0
    sync()
    got = host(out)
    assert got[0].tobytes() == (GOLDEN / "swiglu.bin").read_bytes()
    assert np.array_equal(u32(got[1]), u32(oracle.swiglu(g2, u2)))


def test_rope_and_kv_write_match_fixture_and_oracle():
    lib = _lib.load()
    cap = 1024
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 896)).astype(np.float32)
    q[0, :64] = [(i - 32) / 16.0 for i in range(64)]
    k = rng.standard_normal((2, 128)).astype(np.float32)
    v = rng.standard_normal((2, 128)).astype(np.float32)
    positions = np.array([511, 1023], dtype=np.uint32)
    kv = torch.zeros(2 * 24 * 4 * cap * 64, dtype=torch.float32, device="cuda")
    qd, kd = dev(q), dev(k)
    assert lib.pb_rope_kv_device(ptr(qd), ptr(kd), ptr(dev(v)), positions.ctypes.data_as(ctypes.c_void_p),
                                 2, ptr(kv), cap, 5, None) == 0
    sync()
    gq, gk, gkv = host(qd), host(kd), host(kv)
    assert gq[0, :64].tobytes() == (GOLDEN / "rope.bin").read_bytes()
    for r in range(2):
        assert np.array_equal(u32(gq[r]), u32(oracle.rope_in_place(q[r], 14, int(positions[r]))))
        kr = oracle.rope_in_place(k[r], 2, int(positions[r]))
        assert np.array_equal(u32(gk[r]), u32(kr))
        base = r * 24 * 4 * cap * 64
        for h in range(2):
            for c in range(64):
                kw = oracle.kv_word(cap, 5, 0, int(positions[r]), h, c)
                vw = oracle.kv_word(cap, 5, 1, int(positions[r]), h, c)
                assert u32(gkv[base + kw:base + kw + 1])[0] == u32(kr[h * 64 + c:h * 64 + c + 1])[0]
                assert gkv[base + vw] == v[r, h * 64 + c]


@pytest.mark.parametrize("path", ["0", "1"])
@pytest.mark.parametrize("current,span,fixture,rot", [(2, 256, "256", 0), (256, 512, "512", 7)])
def test_attention_matches_fixtures(monkeypatch, current, span, fixture, rot, path):
    """The reference's attention fixtures through the grouped (0) and the split
    (1) launches."""
    monkeypatch.setenv("PB_ATTN_SPLIT", path)
    lib = _lib.load()
    cap = 32768
    kv = attention_fixture_kv(cap)
    q = np.roll(attention_query(), -rot)
    out = torch.zeros(896, dtype=torch.float32, device="cuda")
    scores = torch.zeros(14 * span, dtype=torch.float32, device="cuda")
    pos = np.array([current], dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(dev(kv)), cap, 0,
                                   pos.ctypes.data_as(ctypes.c_void_p), 1, span, ptr(out),
                                   ptr(scores), None) == 0
    sync()
    assert host(out).tobytes() == (GOLDEN / f"attention-{fixture}.bin").read_bytes()
    last_head = host(scores)[13 * span:14 * span]
    assert last_head.tobytes() == (GOLDEN / f"scores-{fixture}.bin").read_bytes()


@pytest.mark.parametrize("positions,cap", [([0, 1, 2], 1024), ([3, 4, 5], 1024),
                                          ([29, 255, 256], 1024), ([511, 512, 600], 1024),
                                          ([63, 64, 65], 1024), ([1023, 2046, 2047], 2048),
                                          ([2048, 2100, 1], 2560)])
@pytest.mark.parametrize("path", ["0", "1"])
def test_attention_random_kv_matches_oracle(monkeypatch, positions, cap, path):
    """Edge spans (1..N positions, masked tails, tile boundaries at 64), the
    shared-memory path up to 2048 positions (forced with PB_ATTN_SPLIT=0) and
    the global-scores path (forced with 1, and taken beyond 2048 either way),
    and the reference's denormal / signed-zero query words (tests.rs:699-706)."""
    monkeypatch.setenv("PB_ATTN_SPLIT", path)
    lib = _lib.load()
    rows = len(positions)
    rng = np.random.default_rng(sum(positions))
    kv = np.zeros(rows * 24 * 4 * cap * 64, dtype=np.float32)
    layer = 3
    for r in range(rows):
        base = r * 24 * 4 * cap * 64 + layer * 4 * cap * 64
        kv[base:base + 4 * cap * 64] = rng.standard_normal(4 * cap * 64).astype(np.float32)
    q = rng.standard_normal((rows, 896)).astype(np.float32)
    q[0, :6] = oracle.f32([0x00000000, 0x80000000, 0x00000001, 0x007FFFFF, 0x00800000, 0x80000001])
    out = torch.zeros((rows, 896), dtype=torch.float32, device="cuda")
    pos = np.array(positions, dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(dev(kv)), cap, layer,
                                   pos.ctypes.data_as(ctypes.c_void_p), rows, 0, ptr(out), None,
                                   None) == 0
    sync()
    got = host(out)
    for r in range(rows):
        kvr = kv[r * 24 * 4 * cap * 64:(r + 1) * 24 * 4 * cap * 64]
        span = (positions[r] + 4) & ~3
        ref, _ = oracle.attention(q[r], kvr, cap, layer, positions[r], span)
        assert np.array_equal(u32(got[r]), u32(ref)), (r, positions[r])


def _same_bits_or_nan(got, ref):
    """Bit equality, except that a NaN only has to be a NaN (its payload is the
    device's, not the host's)."""
    g, r = u32(got), u32(ref)
    nan = np.isnan(ref)
    return np.array_equal(np.isnan(got), nan) and np.array_equal(g[~nan], r[~nan])


@pytest.mark.parametrize("case", ["overflowing_products", "overflowing_scores", "huge_but_finite",
                                  "inf_value", "nan_query", "nan_key", "tiny_products",
                                  "tiny_values", "wide_values"])
def test_attention_extreme_magnitudes_match_oracle(case):
    """Non-finite and extreme values through the grouped kernels against the
    oracle: products that overflow binary32, finite products whose f64 sum
    overflows the binary32 score, huge but finite products, infinite V, NaN
    queries and keys, products in the binary32 subnormal range, and V spread
    over 170 binades (the PV chain summed as scaled f64 images, and its exact
    fallback when a probability or a V word is not finite)."""
    lib = _lib.load()
    cap, layer = 256, 2
    positions = [0, 69, 130, 191]
    rows = len(positions)
    rng = np.random.default_rng(sum(map(ord, case)))
    kv = np.zeros(rows * 24 * 4 * cap * 64, dtype=np.float32)
    q = rng.standard_normal((rows, 896)).astype(np.float32)
    for r in range(rows):
        base = r * 24 * 4 * cap * 64 + layer * 4 * cap * 64
        kv[base:base + 4 * cap * 64] = rng.standard_normal(4 * cap * 64).astype(np.float32)
        kvr = kv[base:base + 4 * cap * 64]
        p = positions[r] // 2
        if case == "overflowing_products":      # |q k| > FLT_MAX in head 7
            q[r, 70:80] *= np.float32(3e19)
            q[r, 7 * 64 + 5] = np.float32(3e19)
            kvr[oracle.kv_word(cap, 0, 0, p, 1, 5)] = np.float32(2e20)
            kvr[oracle.kv_word(cap, 0, 0, p, 1, 9)] = np.float32(-2e20)
        elif case == "overflowing_scores":      # finite products, sum beyond FLT_MAX
            q[r, :64] = np.float32(1.2e19)
            for c in range(64):
                kvr[oracle.kv_word(cap, 0, 0, p, 0, c)] = np.float32(1.2e19)
        elif case == "huge_but_finite":         # max|q| max|k| >= 2^127, no product overflows
            q[r, 448] = np.float32(1e30)
            kvr[oracle.kv_word(cap, 0, 0, p, 1, 3)] = np.float32(1e10)
        elif case == "inf_value":
            kvr[oracle.kv_word(cap, 0, 1, p, 0, 17)] = np.float32(np.inf)
            kvr[oracle.kv_word(cap, 0, 1, positions[r], 1, 40)] = np.float32(-np.inf)
        elif case == "nan_query":
            q[r, 3 + 64 * r] = np.float32(np.nan)
        elif case == "nan_key":
            kvr[oracle.kv_word(cap, 0, 0, positions[r], 0, 63)] = np.float32(np.nan)
        elif case == "tiny_products":           # q.k products in the f32 subnormal range
            q[r] *= np.float32(2.0 ** -70)
            kvr[:2 * cap * 64] *= np.float32(2.0 ** -70)
        elif case == "tiny_values":             # p.v products subnormal or zero
            kvr[2 * cap * 64:] *= np.float32(2.0 ** -128)
        else:                                   # V over 170 binades: rounding in every f64 sum
            e = rng.integers(-140, 31, 2 * cap * 64)
            kvr[2 * cap * 64:] = (kvr[2 * cap * 64:] * np.exp2(e)).astype(np.float32)
    out = torch.zeros((rows, 896), dtype=torch.float32, device="cuda")
    pos = np.array(positions, dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(dev(kv)), cap, layer,
                                   pos.ctypes.data_as(ctypes.c_void_p), rows, 0, ptr(out), None,
                                   None) == 0
    sync()
    got = host(out)
    for r in range(rows):
        kvr = kv[r * 24 * 4 * cap * 64:(r + 1) * 24 * 4 * cap * 64]
        ref, _ = oracle.attention(q[r], kvr, cap, layer, positions[r], (positions[r] + 4) & ~3)
        assert _same_bits_or_nan(got[r], ref), (case, r, positions[r])


@pytest.mark.parametrize("groups", ["fed", "2", "4", "8", "16"])
@pytest.mark.parametrize("case", ["random", "wide_scores", "overflowing_products", "inf_value",
                                  "nan_key", "tiny_values", "wide_values"])
def test_attention_long_context_extremes_match_oracle(monkeypatch, case, groups):
    """The long-context path (probabilities in the global scratch, the softmax
    sum as an exact tree or its serial fallback, PV chains split into 2, 4, 8 or
    16 component groups, or fed by producer warps) against the oracle,
    probabilities included: random K/V
    (the tree sum holds), scores spread over ~200 units (subnormal
    exponentials: the serial fallback), and the non-finite and extreme cases of
    the grouped kernels."""
    monkeypatch.setenv("PB_ATTN_LONG_GROUPS", groups)
    lib = _lib.load()
    cap, layer = 3008, 0
    positions = [2100, 3000]
    rows = len(positions)
    rng = np.random.default_rng(sum(map(ord, case)) + sum(map(ord, groups)))
    slot = 24 * 4 * cap * 64
    kv = np.zeros(rows * slot, dtype=np.float32)
    q = rng.standard_normal((rows, 896)).astype(np.float32)
    for r in range(rows):
        kvr = kv[r * slot:r * slot + 4 * cap * 64]
        kvr[:] = rng.standard_normal(4 * cap * 64).astype(np.float32)
        p = positions[r] // 3
        if case == "wide_scores":
            q[r] *= np.float32(3.0)
            for c in range(64):
                for h in range(2):
                    kvr[oracle.kv_word(cap, 0, 0, p, h, c)] *= np.float32(40.0)
        elif case == "overflowing_products":
            q[r, 7 * 64 + 5] = np.float32(3e19)
            kvr[oracle.kv_word(cap, 0, 0, p, 1, 5)] = np.float32(2e20)
        elif case == "inf_value":
            kvr[oracle.kv_word(cap, 0, 1, p, 0, 17)] = np.float32(np.inf)
        elif case == "nan_key":
            kvr[oracle.kv_word(cap, 0, 0, positions[r], 0, 63)] = np.float32(np.nan)
        elif case == "tiny_values":
            kvr[2 * cap * 64:] *= np.float32(2.0 ** -128)
        elif case == "wide_values":
            e = rng.integers(-140, 31, 2 * cap * 64)
            kvr[2 * cap * 64:] = (kvr[2 * cap * 64:] * np.exp2(e)).astype(np.float32)
    span_max = (max(positions) + 4) & ~3
    out = torch.zeros((rows, 896), dtype=torch.float32, device="cuda")
    probs = torch.zeros((rows, 14, span_max), dtype=torch.float32, device="cuda")
    pos = np.array(positions, dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(dev(kv)), cap, layer,
                                   pos.ctypes.data_as(ctypes.c_void_p), rows, 0, ptr(out),
                                   ptr(probs), None) == 0
    sync()
    got, got_p = host(out), host(probs)
    for r in range(rows):
        span = (positions[r] + 4) & ~3
        ref, ref_p = oracle.attention(q[r], kv[r * slot:(r + 1) * slot], cap, layer, positions[r],
                                      span)
        assert _same_bits_or_nan(got[r], ref), (case, r, positions[r])
        assert _same_bits_or_nan(got_p[r, 13, :span], ref_p[:span]), (case, r)


@pytest.mark.parametrize("limit", [2300, 2040])
@pytest.mark.parametrize("case", ["random", "wide_values", "inf_value", "nan_key", "wide_scores"])
def test_attention_split_path_many_rows_matches_oracle(monkeypatch, case, limit):
    """The split launches (scores, global softmax, two-group one-chain PV)
    forced for every span at 64 rows, spans past 2,048 and up to 2,044, with
    the extreme cases that force every fallback (non-finite products in the
    integer-built score chains, the serial softmax sum); the final
    probabilities too."""
    monkeypatch.setenv("PB_ATTN_SPLIT", "1")
    lib = _lib.load()
    cap, layer, rows = (limit + 4) // 4 * 4, 0, 64
    rng = np.random.default_rng(sum(map(ord, case)) + limit)
    positions = [int(x) for x in rng.integers(0, limit, rows)]
    positions[:6] = [0, 1, 2, 3, 127, limit - 1]
    slot = 24 * 4 * cap * 64
    kv_d = torch.zeros(rows * slot, dtype=torch.float32, device="cuda")
    regions = []
    q = rng.standard_normal((rows, 896)).astype(np.float32)
    for r in range(rows):
        kvr = rng.standard_normal(4 * cap * 64).astype(np.float32)
        p = positions[r] // 2
        if case == "wide_values":
            e = rng.integers(-140, 31, 2 * cap * 64)
            kvr[2 * cap * 64:] = (kvr[2 * cap * 64:] * np.exp2(e)).astype(np.float32)
        elif case == "inf_value":
            kvr[oracle.kv_word(cap, 0, 1, p, r & 1, 17)] = np.float32(np.inf)
        elif case == "nan_key":
            kvr[oracle.kv_word(cap, 0, 0, p, r & 1, 63)] = np.float32(np.nan)
        elif case == "wide_scores":
            q[r] *= np.float32(3.0)
            for c in range(64):
                kvr[oracle.kv_word(cap, 0, 0, p, r & 1, c)] *= np.float32(40.0)
        regions.append(kvr)
        kv_d[r * slot:r * slot + kvr.size] = torch.from_numpy(kvr).to("cuda")
    out = torch.zeros((rows, 896), dtype=torch.float32, device="cuda")
    span_max = max((p + 4) & ~3 for p in positions)
    probs = torch.zeros((rows, 14, span_max), dtype=torch.float32, device="cuda")
    pos = np.array(positions, dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(kv_d), cap, layer,
                                   pos.ctypes.data_as(ctypes.c_void_p), rows, 0, ptr(out), ptr(probs),
                                   None) == 0
    sync()
    got, got_p = host(out), host(probs)
    full = np.zeros(slot, dtype=np.float32)
    for r in range(rows):
        full[:regions[r].size] = regions[r]
        span = (positions[r] + 4) & ~3
        ref, ref_p = oracle.attention(q[r], full, cap, layer, positions[r], span)
        assert _same_bits_or_nan(got[r], ref), (case, r, positions[r])
        assert _same_bits_or_nan(got_p[r, 13, :span], ref_p[:span]), (case, r)


def _q4_weights(rng, rows, cols):
    nb = rows * cols // 32
    scales = (np.abs(rng.standard_normal(nb) * 0.02) / 8).astype(np.float16)
    nib = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
    w = np.empty((nb, 18), dtype=np.uint8)
    w[:, :2] = scales.view(np.uint8).reshape(nb, 2)
    w[:, 2:] = nib[:, :16] | (nib[:, 16:] << 4)
    return w.reshape(-1)


def _q8_weights(rng, rows, cols):
    nb = rows * cols // 32
    scales = (np.abs(rng.standard_normal(nb) * 0.02) / 8).astype(np.float16)
    w = np.empty((nb, 34), dtype=np.uint8)
    w[:, :2] = scales.view(np.uint8).reshape(nb, 2)
    w[:, 2:] = rng.integers(-128, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    return w.reshape(-1)


def test_matvec_dot_fixture():
    lib = _lib.load()
    mat, q4, q8 = dot_inputs()
    rng = np.random.default_rng(1)
    w4 = np.concatenate([q4, _q4_weights(rng, 31, 64)])
    w8 = np.concatenate([q8, _q8_weights(rng, 31, 64)])
    y = torch.zeros(32, dtype=torch.float32, device="cuda")
    x = dev(mat[None, :])
    assert lib.pb_qmatvec_device(2, ptr(dev(w4)), 32, 64, ptr(x), 1, ptr(y), None) == 0
    sync()
    y4 = host(y).copy()
    assert lib.pb_qmatvec_device(3, ptr(dev(w8)), 32, 64, ptr(x), 1, ptr(y), None) == 0
    sync()
    y8 = host(y).copy()
    assert u32(y4[:1])[0] == 0x43E08000 and u32(y8[:1])[0] == 0x44388000
    st = oracle.prepare_q8(mat)
    assert np.array_equal(u32(y4), u32(oracle.q4_matvec(w4, st, 32, 64)))
    assert np.array_equal(u32(y8), u32(oracle.q8_matvec(w8, st, 32, 64)))


@pytest.mark.parametrize("wtype,rows,cols", [(2, 896, 896), (2, 128, 896), (2, 4864, 896),
                                             (2, 896, 4864), (3, 151936, 896)])
@pytest.mark.parametrize("batch", [1, 8, 9, 64, 256])
def test_matvec_shapes_match_oracle(wtype, rows, cols, batch):
    """B <= 8 runs the CUDA-core matvec, B > 8 the tcgen05 kind::i8 path (tile
    widths 16/32/64 chosen by grid size); both must equal the oracle bit for bit."""
    lib = _lib.load()
    rng = np.random.default_rng(rows * 7 + cols + batch)
    w = _q4_weights(rng, rows, cols) if wtype == 2 else _q8_weights(rng, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    y = torch.zeros((batch, rows), dtype=torch.float32, device="cuda")
    assert lib.pb_qmatvec_device(wtype, ptr(dev(w)), rows, cols, ptr(dev(x)), batch, ptr(y), None) == 0
    sync()
    got = host(y)
    check_rows = range(batch) if rows * batch <= 8 * 151936 else [0, batch - 1]
    for b in check_rows:
        st = oracle.prepare_q8(x[b])
        ref = oracle.q4_matvec(w, st, rows, cols) if wtype == 2 else oracle.q8_matvec(w, st, rows, cols)
        assert np.array_equal(u32(got[b]), u32(ref)), b


@pytest.mark.parametrize("tile", ["8", "16", "32", "64"])
@pytest.mark.parametrize("wtype,rows,cols,batch", [(2, 896, 4864, 100), (3, 1024, 896, 130),
                                                   (2, 1152, 896, 64)])
def test_tensor_core_every_tile_width(monkeypatch, tile, wtype, rows, cols, batch):
    """Each sequence-tile width of the tcgen05 path (forced through PB_TC_TILE),
    ragged last tiles included, equals the oracle bit for bit."""
    monkeypatch.setenv("PB_TC_TILE", tile)
    lib = _lib.load()
    rng = np.random.default_rng(rows + batch + int(tile))
    w = _q4_weights(rng, rows, cols) if wtype == 2 else _q8_weights(rng, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    y = torch.zeros((batch, rows), dtype=torch.float32, device="cuda")
    assert lib.pb_qmatvec_device(wtype, ptr(dev(w)), rows, cols, ptr(dev(x)), batch, ptr(y), None) == 0
    sync()
    got = host(y)
    for b in range(batch):
        st = oracle.prepare_q8(x[b])
        ref = oracle.q4_matvec(w, st, rows, cols) if wtype == 2 else oracle.q8_matvec(w, st, rows, cols)
        assert np.array_equal(u32(got[b]), u32(ref)), b


def test_tensor_core_widest_tile_matches_oracle():
    """4864 x 896 Q4_0 at 512 rows: 16 sequence tiles per weight tile."""
    lib = _lib.load()
    rng = np.random.default_rng(512)
    rows, cols, batch = 4864, 896, 512
    w = _q4_weights(rng, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    y = torch.zeros((batch, rows), dtype=torch.float32, device="cuda")
    assert lib.pb_qmatvec_device(2, ptr(dev(w)), rows, cols, ptr(dev(x)), batch, ptr(y), None) == 0
    sync()
    got = host(y)
    for b in (0, 63, 64, 300, 511):
        ref = oracle.q4_matvec(w, oracle.prepare_q8(x[b]), rows, cols)
        assert np.array_equal(u32(got[b]), u32(ref)), b


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 9, 64])
@pytest.mark.parametrize("layer,role", [(0, 19), (3, 16), (5, 21), (7, 17), (11, 12), (13, 13), (23, 11), (None, 290)])
def test_model_matvec_matches_oracle(model_view, model_image, layer, role, batch):
    """pb_model_matvec_device on the model's own tensors (the engine's matvec:
    CUDA-core below 9 rows, tensor-core tile image from 9) equals the oracle."""
    from promptboot_b200 import pbtqw25
    lib = _lib.load()
    tid = 290 if layer is None else pbtqw25.layer_tensor(layer, role)
    rows, cols = {19: (896, 896), 16: (128, 896), 21: (128, 896), 17: (896, 896), 12: (4864, 896),
                  13: (4864, 896), 11: (896, 4864), 290: (151936, 896)}[role]
    w = pbtqw25.tensor_view(model_image, tid)
    rng = np.random.default_rng(tid * 10 + batch)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    y = torch.zeros((batch, rows), dtype=torch.float32, device="cuda")
    assert lib.pb_model_matvec_device(model_view._h, tid, ptr(dev(x)), batch, ptr(y), None) == 0
    assert lib.pb_model_matvec_status(model_view._h, None) == 0
    got = host(y)
    for b in ([0, batch - 1] if role == 290 else range(batch)):
        st = oracle.prepare_q8(x[b])
        ref = oracle.q8_matvec(w, st, rows, cols) if role == 290 else oracle.q4_matvec(w, st, rows, cols)
        assert np.array_equal(u32(got[b]), u32(ref)), b
    assert lib.pb_model_matvec_device(model_view._h, 5, ptr(dev(x)), batch, ptr(y), None) != 0  # a norm


@pytest.mark.parametrize("position", [31023, 20001])
def test_attention_long_context_matches_oracle(position):
    """Config 4 scale (30,000-token prompts + 1,024 decode steps, up to 31,024
    positions): the long-context attention path over a seeded KV of slot 0,
    layer 0, against the oracle."""
    lib = _lib.load()
    cap = 31024
    rng = np.random.default_rng(position)
    kv = rng.standard_normal(4 * cap * 64).astype(np.float32)   # slot 0, layer 0 only
    q = rng.standard_normal((1, 896)).astype(np.float32)
    out = torch.zeros((1, 896), dtype=torch.float32, device="cuda")
    pos = np.array([position], dtype=np.uint32)
    assert lib.pb_attention_device(ptr(dev(q)), ptr(dev(kv)), cap, 0,
                                   pos.ctypes.data_as(ctypes.c_void_p), 1, 0, ptr(out), None,
                                   None) == 0
    sync()
    full = np.zeros(24 * 4 * cap * 64, dtype=np.float32)
    full[:kv.size] = kv
    ref, _ = oracle.attention(q[0], full, cap, 0, position, (position + 4) & ~3)
    assert np.array_equal(u32(host(out)[0]), u32(ref))


def test_swiglu_special_values_match_oracle():
    """Gate words at expf4's edges (overflow / underflow boundaries, infinities,
    NaN, signed zeros, subnormals, huge magnitudes) and up words with zeros and
    infinities; NaN results compared as NaN."""
    lib = _lib.load()
    rng = np.random.default_rng(31)
    g = (rng.standard_normal((3, 4864)) * 30).astype(np.float32)
    u = rng.standard_normal((3, 4864)).astype(np.float32)
    specials = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 1e-42, -1e-42, 88.72, -88.72,
                         88.73, -88.73, 103.9, -103.9, 104.0, -104.0, 1e30, -1e30, 3.4e38,
                         -3.4e38, 126.0, -126.0, 127.0, -127.0], dtype=np.float32)
    g[0, :specials.size] = specials
    g[1, 100:100 + specials.size] = specials
    u[1, 100:100 + specials.size] = np.float32(0.0)
    g[2, 4000:4000 + specials.size] = specials
    u[2, 4000:4000 + specials.size] = np.float32(np.inf)
    out = torch.zeros((3, 4864), dtype=torch.float32, device="cuda")
    assert lib.pb_swiglu_device(ptr(dev(g)), ptr(dev(u)), 3, ptr(out), None) == 0
    sync()
    got = host(out)
    for r in range(3):
        assert _same_bits_or_nan(got[r], oracle.swiglu(g[r], u[r])), r


def test_rmsnorm_special_rows_match_oracle():
    """All-zero, subnormal-only, overflowing squares, and rows holding inf or
    NaN words."""
    lib = _lib.load()
    rng = np.random.default_rng(32)
    rows = [np.zeros(896, dtype=np.float32),
            (rng.uniform(-1, 1, 896) * 1e-40).astype(np.float32),
            (rng.standard_normal(896) * 1e20).astype(np.float32),
            rng.standard_normal(896).astype(np.float32),
            rng.standard_normal(896).astype(np.float32),
            rng.standard_normal(896).astype(np.float32)]
    rows[3][17] = np.inf
    rows[4][800] = np.nan
    rows[5][:] = np.float32(-0.0)
    rows[5][3] = np.float32(2.0 ** -149)
    xs = np.stack(rows)
    w = rng.uniform(0.5, 1.5, 896).astype(np.float32)
    y = torch.zeros((len(rows), 896), dtype=torch.float32, device="cuda")
    assert lib.pb_rmsnorm_device(ptr(dev(xs)), ptr(dev(w)), len(rows), ptr(y), None) == 0
    sync()
    got = host(y)
    for r in range(len(rows)):
        assert _same_bits_or_nan(got[r], oracle.rmsnorm(xs[r], w)), r


@pytest.mark.parametrize("position", [0, 1, 32766, 32767])
def test_rope_extreme_positions_match_oracle(position):
    """The first and the last rows of the 32768-position table."""
    lib = _lib.load()
    cap = 32768
    rng = np.random.default_rng(position + 5)
    q = (rng.standard_normal((1, 896)) * 4).astype(np.float32)
    k = (rng.standard_normal((1, 128)) * 4).astype(np.float32)
    v = rng.standard_normal((1, 128)).astype(np.float32)
    kv = torch.zeros(24 * 4 * cap * 64 // 24, dtype=torch.float32, device="cuda")  # layer 0 only
    qd, kd = dev(q), dev(k)
    pos = np.array([position], dtype=np.uint32)
    assert lib.pb_rope_kv_device(ptr(qd), ptr(kd), ptr(dev(v)), pos.ctypes.data_as(ctypes.c_void_p),
                                 1, ptr(kv), cap, 0, None) == 0
    sync()
    assert np.array_equal(u32(host(qd)[0]), u32(oracle.rope_in_place(q[0], 14, position)))
    assert np.array_equal(u32(host(kd)[0]), u32(oracle.rope_in_place(k[0], 2, position)))


@pytest.mark.parametrize("case", ["tiny", "huge", "zero_block", "mixed"])
def test_matvec_extreme_activations_match_oracle(case):
    """Activations whose Q8_0 blocks hit the quantizer's edges (all-zero blocks,
    binary16-subnormal scales, scales rounding to inf in binary16) through both
    matvec paths."""
    lib = _lib.load()
    rng = np.random.default_rng(sum(map(ord, case)))
    rows, cols = 896, 896
    w = _q4_weights(rng, rows, cols)
    x = rng.standard_normal((12, cols)).astype(np.float32)
    if case == "tiny":
        x *= np.float32(1e-6)
    elif case == "huge":
        x *= np.float32(1e6)
    elif case == "zero_block":
        x[:, 64:128] = 0.0
        x[:, 320:352] = np.float32(-0.0)
    else:
        x[:, :32] *= np.float32(1e-7)
        x[:, 32:64] *= np.float32(3e6)
    for batch in (4, 12):
        y = torch.zeros((batch, rows), dtype=torch.float32, device="cuda")
        assert lib.pb_qmatvec_device(2, ptr(dev(w)), rows, cols, ptr(dev(x[:batch])), batch, ptr(y),
                                     None) == 0
        sync()
        got = host(y)
        for b in range(batch):
            ref = oracle.q4_matvec(w, oracle.prepare_q8(x[b]), rows, cols)
            assert _same_bits_or_nan(got[b], ref), (case, batch, b)
