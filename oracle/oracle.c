/*
 * CPU oracle for the promptboot decode hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's decode arithmetic.  Every function
 * cites the reference file:line (paths inside sulewicz/promptboot) whose
 * operation order it follows.  Built with -ffp-contract=off: each C operator is
 * one IEEE binary32/binary64 rounding, as each scalar SSE2 instruction in the
 * reference is.  Parity pin: tests/test_oracle_golden.py checks this file
 * against the reference's fixtures/inference/kernels/ golden files, the expf edge
 * table, the sampler known-answer tests and the RoPE table SHA-256.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <time.h>
#include <stdlib.h>
#include <string.h>

static inline float fbits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bitsf(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
static inline int finite_bits(uint32_t b) { return (b & 0x7f800000u) != 0x7f800000u; }

/* fp32_sse2.rs:362-376 */
uint32_t orc_half_to_f32_bits(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 0x1fu;
    uint32_t fraction = bits & 0x03ffu;
    if (exponent == 0) {
        if (fraction == 0) return sign;
        uint32_t shift = (uint32_t)__builtin_clz(fraction) - 21u;
        uint32_t normalized = fraction << shift;
        return sign | ((113u - shift) << 23) | ((normalized & 0x03ffu) << 13);
    }
    if (exponent == 31) return sign | 0x7f800000u | (fraction << 13);
    return sign | ((exponent + 112u) << 23) | (fraction << 13);
}

/* fp32_sse2.rs:924-943 (float-multiply round-to-nearest-even conversion) */
uint16_t orc_f32_bits_to_half(uint32_t bits) {
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    uint32_t magnitude = bits & 0x7fffffffu;
    float base = (fbits(magnitude) * fbits(0x77800000u)) * fbits(0x08800000u);
    uint32_t doubled = bits + bits;
    uint32_t bias = doubled & 0xff000000u;
    if (bias < 0x71000000u) bias = 0x71000000u;
    uint32_t rounded = bitsf(fbits((bias >> 1) + 0x07800000u) + base);
    uint32_t exponent = (rounded >> 13) & 0x7c00u;
    uint32_t mantissa = rounded & 0x0fffu;
    if (doubled > 0xff000000u) return (uint16_t)(sign | 0x7e00u);
    return (uint16_t)(sign | (uint16_t)(exponent + mantissa));
}

/* fp32_sse2.rs:378-402 */
static float scalbn_ref(float value, int32_t exponent) {
    if (exponent > 127) {
        value = value * fbits(0x7f000000u);
        exponent -= 127;
        if (exponent > 127) {
            value = value * fbits(0x7f000000u);
            exponent -= 127;
            if (exponent > 127) exponent = 127;
        }
    } else if (exponent < -126) {
        float step = fbits(0x00800000u) * fbits(0x4b800000u);
        value = value * step;
        exponent += 126 - 24;
        if (exponent < -126) {
            value = value * step;
            exponent += 126 - 24;
            if (exponent < -126) exponent = -126;
        }
    }
    return value * fbits((uint32_t)(0x7f + exponent) << 23);
}

/* fp32_sse2.rs:404-469: FreeBSD msun e_expf.c as carried by rust libm 0.2.11 */
uint32_t orc_expf_bits(uint32_t in) {
    float x = fbits(in);
    uint32_t magnitude = in & 0x7fffffffu;
    uint32_t sign = in >> 31;
    if (magnitude >= 0x42aeac50u) {
        if (magnitude > 0x7f800000u) return in;
        if (magnitude >= 0x42b17218u && sign == 0) return bitsf(x * fbits(0x7f000000u));
        if (sign != 0 && magnitude >= 0x42cff1b5u) return 0;
    }
    int32_t k;
    float hi, lo;
    if (magnitude > 0x3eb17218u) {
        if (magnitude > 0x3f851592u) {
            float half = sign == 0 ? 0.5f : -0.5f;
            k = (int32_t)(fbits(0x3fb8aa3bu) * x + half);
        } else {
            k = 1 - (int32_t)sign - (int32_t)sign;
        }
        float kf = (float)k;
        hi = x - kf * fbits(0x3f317200u);
        lo = kf * fbits(0x35bfbe8eu);
        x = hi - lo;
    } else if (magnitude > 0x39000000u) {
        k = 0;
        hi = x;
        lo = 0.0f;
    } else {
        return bitsf(1.0f + x);
    }
    float square = x * x;
    float c = x - square * (fbits(0x3e2aaa8fu) + square * fbits(0xbb355215u));
    float fraction = (x * c) / (2.0f - c);
    float y = 1.0f + ((fraction - lo) + hi);
    return k == 0 ? bitsf(y) : bitsf(scalbn_ref(y, k));
}

/* fp32_sse2.rs:1336-1372: ggml four-lane vector expf, -inf lanes map to +0 */
void orc_expf4(uint32_t v[4]) {
    for (int lane = 0; lane < 4; ++lane) {
        uint32_t in = v[lane];
        if (in == 0xff800000u) { v[lane] = 0; continue; }
        float x = fbits(in);
        float z = x * fbits(0x3fb8aa3bu) + fbits(0x4b400000u);
        float n = z - fbits(0x4b400000u);
        float b = (x - n * fbits(0x3f317200u)) - n * fbits(0x35bfbe8eu);
        uint32_t e = bitsf(z) << 23;
        uint32_t k = e + 0x3f800000u;
        float absn = fbits(bitsf(n) & 0x7fffffffu);
        float u = b * b;
        float first = fbits(0x3c072010u) * b + fbits(0x3d2b9f17u);
        float second = fbits(0x3e2aaf33u) * b + fbits(0x3efffedbu);
        float poly = first * u + second;
        float j = poly * u + fbits(0x3f7ffff6u) * b;
        float result;
        if (!(absn > fbits(0x42fc0000u))) {
            result = j * fbits(k) + fbits(k);
        } else {
            uint32_t g = !(n > 0.0f) ? 0x82000000u : 0u;
            float s1 = fbits(g + 0x7f000000u);
            float s2 = fbits(e - g);
            float exceptional = (s2 * j + s2) * s1;
            result = absn > fbits(0x43400000u) ? s1 * s1 : exceptional;
        }
        v[lane] = bitsf(result);
    }
}

/* fp32_sse2.rs:897-922: dequantize one Q4_0 row, low nibbles are elements 0-15 */
void orc_q4_row(const uint8_t *weights, size_t row, float *out, size_t columns) {
    size_t blocks = columns >> 5;
    const uint8_t *base = weights + row * blocks * 18;
    for (size_t b = 0; b < blocks; ++b) {
        const uint8_t *block = base + b * 18;
        float scale = fbits(orc_half_to_f32_bits((uint16_t)(block[0] | (block[1] << 8))));
        for (int e = 0; e < 32; ++e) {
            uint8_t packed = block[2 + (e & 15)];
            int q = e < 16 ? (packed & 0x0f) - 8 : (packed >> 4) - 8;
            out[b * 32 + e] = scale * (float)q;
        }
    }
}

/* fp32_sse2.rs:945-983: Q8_0 activation staging (34-byte blocks) */
void orc_prepare_q8(const float *input, uint8_t *staging, size_t columns) {
    for (size_t b = 0; b < (columns >> 5); ++b) {
        const float *x = input + b * 32;
        uint8_t *block = staging + b * 34;
        float maximum = 0.0f;
        for (int e = 0; e < 32; ++e) {
            float magnitude = fbits(bitsf(x[e]) & 0x7fffffffu);
            if (magnitude > maximum) maximum = magnitude;
        }
        float scale = maximum / 127.0f;
        uint16_t h = orc_f32_bits_to_half(bitsf(scale));
        block[0] = (uint8_t)(h & 0xff);
        block[1] = (uint8_t)(h >> 8);
        float inverse = bitsf(scale) == 0 ? 0.0f : 1.0f / scale;
        for (int e = 0; e < 32; ++e) {
            float v = x[e] * inverse;
            float half = (bitsf(v) >> 31) == 0 ? 0.5f : -0.5f;
            block[2 + e] = (uint8_t)(int8_t)(int32_t)(v + half);
        }
    }
}

/* fp32_sse2.rs:1001-1062 (SSE2) / 1116-1141 (AVX2): exact int32 nibble dot */
int32_t orc_q4_block_dot(const uint8_t *packed16, const int8_t *act32) {
    int32_t total = 0;
    for (int i = 0; i < 16; ++i) {
        total += ((int32_t)(packed16[i] & 0x0f) - 8) * (int32_t)act32[i];
        total += ((int32_t)(packed16[i] >> 4) - 8) * (int32_t)act32[16 + i];
    }
    return total;
}

/* fp32_sse2.rs:1064-1114 / 1143-1164 */
int32_t orc_q8_block_dot(const int8_t *weights32, const int8_t *act32) {
    int32_t total = 0;
    for (int i = 0; i < 32; ++i) total += (int32_t)weights32[i] * (int32_t)act32[i];
    return total;
}

static inline float half_at(const uint8_t *p) {
    return fbits(orc_half_to_f32_bits((uint16_t)(p[0] | (p[1] << 8))));
}

/* fp32_sse2.rs:1217-1248: total += (f32(i32) * dW) * dA, blocks in order */
void orc_q4_matvec(const uint8_t *weights, const uint8_t *staging, float *out,
                   size_t rows, size_t columns) {
    size_t blocks = columns >> 5;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = weights + r * blocks * 18;
        float total = 0.0f;
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *w = row + b * 18;
            const uint8_t *a = staging + b * 34;
            int32_t integer = orc_q4_block_dot(w + 2, (const int8_t *)(a + 2));
            total = total + ((float)integer * half_at(w)) * half_at(a);
        }
        out[r] = total;
    }
}

/* fp32_sse2.rs:1250-1281: total += f32(i32) * (dW * dA) -- note the association */
void orc_q8_matvec(const uint8_t *weights, const uint8_t *staging, float *out,
                   size_t rows, size_t columns) {
    size_t blocks = columns >> 5;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = weights + r * blocks * 34;
        float total = 0.0f;
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *w = row + b * 34;
            const uint8_t *a = staging + b * 34;
            int32_t integer = orc_q8_block_dot((const int8_t *)(w + 2), (const int8_t *)(a + 2));
            total = total + (float)integer * (half_at(w) * half_at(a));
        }
        out[r] = total;
    }
}

/* fp32_sse2.rs:1310-1334: f64 sum of squares, f32 mean, 1/sqrt(mean + 1e-6) */
void orc_rmsnorm(const float *input, const float *weight, float *out, size_t words) {
    double sum = 0.0;
    for (size_t i = 0; i < words; ++i) sum += (double)(input[i] * input[i]);
    float mean = (float)(sum / (double)(float)words);
    float inverse = 1.0f / sqrtf(mean + fbits(0x358637bdu));
    for (size_t i = 0; i < words; ++i) out[i] = (input[i] * inverse) * weight[i];
}

/* tests/fixtures/inference/generate_inference_rope_fixture.py:34-45: glibc
 * powf/cosf/sinf over a binary32 angle recurrence, theta base 1e6, 64-wide heads */
void orc_rope_table(float *table) {
    float theta_scale = powf(1000000.0f, -2.0f / 64.0f);
    size_t at = 0;
    for (int position = 0; position < 32768; ++position) {
        float theta = (float)position;
        for (int pair = 0; pair < 32; ++pair) {
            table[at++] = cosf(theta);
            table[at++] = sinf(theta);
            theta = theta * theta_scale;
        }
    }
}

/* fp32_sse2.rs:1413-1428: NeoX half-split rotation, pairs (i, i+32) */
void orc_rope_in_place(float *values, size_t heads, size_t position, const float *table) {
    for (size_t h = 0; h < heads; ++h) {
        float *v = values + h * 64;
        for (int pair = 0; pair < 32; ++pair) {
            float left = v[pair], right = v[pair + 32];
            float cosine = table[(position * 32 + pair) * 2];
            float sine = table[(position * 32 + pair) * 2 + 1];
            v[pair] = left * cosine - right * sine;
            v[pair + 32] = left * sine + right * cosine;
        }
    }
}

/* inference.rs:2035-2052 with the context capacity as a parameter (the reference
 * fixes it at 32768): K in 4-position tiles, V row-major per position. */
size_t orc_kv_word(size_t capacity, size_t layer, size_t kind, size_t position,
                   size_t head, size_t component) {
    size_t value_words = 2 * capacity * 64;
    size_t base = layer * 2 * value_words;
    if (kind == 0)
        return base + (((head * (capacity / 4) + position / 4) * 64 + component) * 4 + position % 4);
    return base + value_words + ((head * capacity + position) * 64 + component);
}

/* fp32_sse2.rs:1430-1454, 1527-1550, 1589-1672 (the SSE2 backend; the AVX2 one is
 * bit-identical by tests.rs:803-808) */
void orc_attention(const float *query, const float *kv, size_t capacity, size_t layer,
                   size_t current, size_t span, float *out, float *scores,
                   float *raw_capture, float *prob_capture) {
    size_t positions = current + 1;
    for (size_t qh = 0; qh < 14; ++qh) {
        size_t kh = qh / 7;
        for (size_t p = 0; p < positions; ++p) {
            double dot = 0.0;
            for (size_t c = 0; c < 64; ++c)
                dot += (double)(query[qh * 64 + c] * kv[orc_kv_word(capacity, layer, 0, p, kh, c)]);
            scores[p] = (float)dot * 0.125f;
        }
        float maximum = fbits(0xff800000u);
        for (size_t p = 0; p < positions; ++p)
            if (scores[p] > maximum) maximum = scores[p];
        for (size_t p = positions; p < span; ++p) scores[p] = fbits(0xff800000u);
        if (raw_capture) memcpy(raw_capture + qh * span, scores, span * 4);
        double sum = 0.0;
        for (size_t p = 0; p < span; p += 4) {
            uint32_t lanes[4];
            for (int l = 0; l < 4; ++l) lanes[l] = bitsf(scores[p + l] - maximum);
            orc_expf4(lanes);
            for (int l = 0; l < 4; ++l) scores[p + l] = fbits(lanes[l]);
            sum += (double)((fbits(lanes[0]) + fbits(lanes[1])) + (fbits(lanes[2]) + fbits(lanes[3])));
        }
        float normalizer = (float)(1.0 / sum);
        for (size_t p = 0; p < positions; ++p) scores[p] = scores[p] * normalizer;
        if (prob_capture) memcpy(prob_capture + qh * span, scores, span * 4);
        for (size_t c = 0; c < 64; ++c) {
            double total = 0.0;
            for (size_t p = 0; p < positions; ++p)
                total += (double)(scores[p] * kv[orc_kv_word(capacity, layer, 1, p, kh, c)]);
            out[qh * 64 + c] = (float)total;
        }
    }
}

/* fp32_sse2.rs:1751-1770: g / (1 + expf4(0 - g)) * u */
void orc_swiglu(const float *gate, const float *up, float *out, size_t words) {
    for (size_t i = 0; i < words; i += 4) {
        uint32_t e[4];
        for (int l = 0; l < 4; ++l) e[l] = bitsf(0.0f - gate[i + l]);
        orc_expf4(e);
        for (int l = 0; l < 4; ++l) {
            float silu = gate[i + l] / (1.0f + fbits(e[l]));
            out[i + l] = silu * up[i + l];
        }
    }
}

/* fp32_sse2.rs:1772-1784: first maximum by strict > */
uint32_t orc_argmax(const float *logits, size_t words) {
    size_t selected = 0;
    float best = logits[0];
    for (size_t i = 1; i < words; ++i)
        if (logits[i] > best) { best = logits[i]; selected = i; }
    return (uint32_t)selected;
}

/* inference.rs:801-809: xorshift64 then a multiplicative 24-bit draw */
uint32_t orc_next_24(uint64_t *state, uint64_t *draws) {
    uint64_t v = *state;
    v ^= v >> 12;
    v ^= v << 25;
    v ^= v >> 27;
    *state = v;
    *draws += 1;
    return (uint32_t)((v * 0x2545f4914f6cdd1dull) >> 40);
}

/* fp32_sse2.rs:1786-1846 */
uint32_t orc_sample_top_k_top_p(const float *logits, size_t words, uint32_t random24) {
    enum { K = 20 };
    uint32_t ids[K];
    float values[K];
    for (int i = 0; i < K; ++i) { ids[i] = 0xffffffffu; values[i] = fbits(0xff800000u); }
    for (size_t token = 0; token < words; ++token) {
        float v = logits[token];
        int insertion = K;
        for (int at = 0; at < K; ++at)
            if (ids[at] == 0xffffffffu || v > values[at]) { insertion = at; break; }
        if (insertion < K) {
            for (int at = K - 1; at > insertion; --at) { ids[at] = ids[at - 1]; values[at] = values[at - 1]; }
            ids[insertion] = (uint32_t)token;
            values[insertion] = v;
        }
    }
    float maximum = values[0];
    float weights[K];
    double total = 0.0;
    for (int at = 0; at < K; ++at) {
        weights[at] = fbits(orc_expf_bits(bitsf((values[at] - maximum) / fbits(0x3f333333u))));
        total += (double)weights[at];
    }
    float cutoff = (float)total * fbits(0x3f4ccccdu);
    int kept = K;
    double kept_total = 0.0;
    for (int at = 0; at < K; ++at) {
        kept_total += (double)weights[at];
        if (!(cutoff > (float)kept_total)) { kept = at + 1; break; }
    }
    float unit = (float)(random24 & 0x00ffffffu) / fbits(0x4b800000u);
    float target = (float)kept_total * unit;
    double cumulative = 0.0;
    for (int at = 0; at < kept; ++at) {
        cumulative += (double)weights[at];
        if ((float)cumulative > target) return ids[at];
    }
    return ids[kept - 1];
}

/* fp32_sse2.rs:1848-1876: once per distinct history token, bitmap cleared after */
void orc_apply_repetition_penalty(float *logits, const uint32_t *tokens, size_t count,
                                  uint8_t *seen) {
    for (size_t at = 0; at < count; ++at) {
        uint32_t token = tokens[at];
        uint8_t bit = (uint8_t)(1u << (token & 7));
        if ((seen[token / 8] & bit) == 0) {
            seen[token / 8] |= bit;
            uint32_t score = bitsf(logits[token]);
            float adjusted = ((score & 0x80000000u) && (score & 0x7fffffffu))
                                 ? logits[token] * fbits(0x3f8ccccdu)
                                 : logits[token] / fbits(0x3f8ccccdu);
            logits[token] = adjusted;
        }
    }
    for (size_t at = 0; at < count; ++at) {
        uint32_t token = tokens[at];
        seen[token / 8] &= (uint8_t)~(1u << (token & 7));
    }
}

static void set_error(orc_error *err, uint32_t status, uint32_t domain, uint32_t layer,
                      uint32_t position, uint32_t tensor, uint64_t needed, uint64_t available,
                      uint32_t kind, uint32_t sub) {
    if (!err) return;
    err->status = status; err->domain = domain; err->layer = layer; err->position = position;
    err->tensor_id = tensor; err->reserved = 0; err->needed = needed; err->available = available;
    err->detail = ((uint64_t)kind << 32) | sub;
}

/* inference.rs:919-965 (validate, penalty, one draw, top-k/top-p) */
uint32_t orc_sample_with_repetition(float *logits, size_t words, const uint32_t *tokens,
                                    size_t count, uint8_t *seen, size_t seen_len,
                                    uint64_t *state, uint64_t *draws, uint32_t *selected,
                                    orc_error *err) {
    if (words != ORC_VOCAB) {
        set_error(err, 4, 18, 0xffffffffu, 0, 0xffffffffu, ORC_VOCAB, words, 12, 0);
        return 4;
    }
    for (size_t i = 0; i < words; ++i)
        if (!finite_bits(bitsf(logits[i]))) {
            set_error(err, 7, 19, 0xffffffffu, 0, 0xffffffffu, 0, bitsf(logits[i]), 7, (uint32_t)i);
            return 7;
        }
    if (seen_len < (words + 7) / 8) {
        set_error(err, 4, 19, 0xffffffffu, 0, 0xffffffffu, (words + 7) / 8, seen_len, 4, 2);
        return 4;
    }
    for (size_t i = 0; i < count; ++i)
        if (tokens[i] >= words) {
            set_error(err, 3, 19, 0xffffffffu, 0, 0xffffffffu, words, tokens[i], 2, 0);
            return 3;
        }
    orc_apply_repetition_penalty(logits, tokens, count, seen);
    uint32_t r = orc_next_24(state, draws);
    *selected = orc_sample_top_k_top_p(logits, words, r);
    return 0;
}

/* ------------------------------------------------------------------ model */

/* model.rs:780-808: the 96-byte directory entry of tensor id inside section 6 */
const uint8_t *orc_tensor(const uint8_t *file, uint32_t id) {
    uint64_t offset;
    memcpy(&offset, file + 3952512 + (size_t)id * 96 + 32, 8);
    return file + offset;
}

static uint32_t layer_id(uint32_t layer, uint32_t role) { return 1 + layer * 12 + (role - 10); }

typedef struct {
    float hidden[896], residual[896], norm[896], q[896], k[128], v[128], attention[896];
    float gate[4864], up[4864], product[4864];
    uint8_t staging[5184];
    float *scores;
} orc_scratch;

/* inference.rs:1889-1936: first non-finite word of a stage output */
static int check_stage(const float *values, size_t words, uint32_t domain, uint32_t layer,
                       uint32_t tensor, uint32_t position, orc_error *err) {
    for (size_t i = 0; i < words; ++i) {
        uint32_t b = bitsf(values[i]);
        if (!finite_bits(b)) {
            set_error(err, domain <= 16 ? 6 : 7, domain, layer, position, tensor, 0, b, 7, (uint32_t)i);
            return 1;
        }
    }
    return 0;
}

static void add_into(float *values, const float *bias, size_t words) {
    for (size_t i = 0; i < words; ++i) values[i] = values[i] + bias[i];
}

/* inference.rs:1454-1765: one token through 24 layers and, on request, the lm_head */
static uint32_t forward_scratch(const uint8_t *file, float *kv, size_t capacity,
                                const float *rope, uint32_t token, uint32_t position,
                                float *logits, orc_error *err, orc_scratch *s) {
#define CHECK(buf, n, dom, lay, tid) \
    if (check_stage(buf, n, dom, lay, tid, position, err)) return err ? err->status : 6
    const uint32_t NO = 0xffffffffu;
    orc_q4_row(orc_tensor(file, 0), token, s->hidden, 896);
    CHECK(s->hidden, 896, 3, NO, 0);
    for (uint32_t layer = 0; layer < 24; ++layer) {
        memcpy(s->residual, s->hidden, sizeof s->hidden);
        orc_rmsnorm(s->hidden, (const float *)orc_tensor(file, layer_id(layer, 10)), s->norm, 896);
        CHECK(s->norm, 896, 4, layer, layer_id(layer, 10));
        orc_prepare_q8(s->norm, s->staging, 896);
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 19)), s->staging, s->q, 896, 896);
        add_into(s->q, (const float *)orc_tensor(file, layer_id(layer, 18)), 896);
        CHECK(s->q, 896, 5, layer, layer_id(layer, 19));
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 16)), s->staging, s->k, 128, 896);
        add_into(s->k, (const float *)orc_tensor(file, layer_id(layer, 15)), 128);
        CHECK(s->k, 128, 6, layer, layer_id(layer, 16));
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 21)), s->staging, s->v, 128, 896);
        add_into(s->v, (const float *)orc_tensor(file, layer_id(layer, 20)), 128);
        CHECK(s->v, 128, 7, layer, layer_id(layer, 21));
        orc_rope_in_place(s->q, 14, position, rope);
        orc_rope_in_place(s->k, 2, position, rope);
        CHECK(s->q, 896, 8, layer, layer_id(layer, 19));
        CHECK(s->k, 128, 8, layer, layer_id(layer, 16));
        CHECK(s->k, 128, 9, layer, layer_id(layer, 16));
        for (int h = 0; h < 2; ++h)
            for (int c = 0; c < 64; ++c) {
                kv[orc_kv_word(capacity, layer, 0, position, h, c)] = s->k[h * 64 + c];
                kv[orc_kv_word(capacity, layer, 1, position, h, c)] = s->v[h * 64 + c];
            }
        size_t span = ((size_t)position + 1 + 3) & ~(size_t)3;
        orc_attention(s->q, kv, capacity, layer, position, span, s->attention, s->scores, NULL, NULL);
        CHECK(s->attention, 896, 10, layer, NO);
        orc_prepare_q8(s->attention, s->staging, 896);
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 17)), s->staging, s->norm, 896, 896);
        for (int i = 0; i < 896; ++i) s->hidden[i] = s->residual[i] + s->norm[i];
        CHECK(s->hidden, 896, 11, layer, layer_id(layer, 17));
        memcpy(s->residual, s->hidden, sizeof s->hidden);
        orc_rmsnorm(s->hidden, (const float *)orc_tensor(file, layer_id(layer, 14)), s->norm, 896);
        CHECK(s->norm, 896, 12, layer, layer_id(layer, 14));
        orc_prepare_q8(s->norm, s->staging, 896);
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 12)), s->staging, s->gate, 4864, 896);
        CHECK(s->gate, 4864, 13, layer, layer_id(layer, 12));
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 13)), s->staging, s->up, 4864, 896);
        CHECK(s->up, 4864, 14, layer, layer_id(layer, 13));
        orc_swiglu(s->gate, s->up, s->product, 4864);
        CHECK(s->product, 4864, 15, layer, layer_id(layer, 12));
        orc_prepare_q8(s->product, s->staging, 4864);
        orc_q4_matvec(orc_tensor(file, layer_id(layer, 11)), s->staging, s->norm, 896, 4864);
        for (int i = 0; i < 896; ++i) s->hidden[i] = s->residual[i] + s->norm[i];
        CHECK(s->hidden, 896, 16, layer, layer_id(layer, 11));
    }
    if (logits) {
        orc_rmsnorm(s->hidden, (const float *)orc_tensor(file, 289), s->norm, 896);
        CHECK(s->norm, 896, 17, NO, 289);
        orc_prepare_q8(s->norm, s->staging, 896);
        orc_q8_matvec(orc_tensor(file, 290), s->staging, logits, 151936, 896);
        CHECK(logits, 151936, 18, NO, 290);
    }
    return 0;
#undef CHECK
}

uint32_t orc_forward(const uint8_t *file, float *kv, size_t capacity, const float *rope,
                     uint32_t token, uint32_t position, float *logits, orc_error *err) {
    orc_scratch *s = (orc_scratch *)calloc(1, sizeof *s);
    s->scores = (float *)calloc(capacity + 4, sizeof(float));
    uint32_t status = forward_scratch(file, kv, capacity, rope, token, position, logits, err, s);
    free(s->scores);
    free(s);
    return status;
}

/* src/model_repl.rs:927-1000: prefill, then sample_token_with_repetition over the
 * prompt plus every sampled token, then decode_selected(sampled) */
uint32_t orc_generate(const uint8_t *file, float *kv, size_t capacity, const float *rope,
                      const uint32_t *prompt, uint32_t prompt_len, uint32_t decode_steps,
                      uint64_t seed, int stop_at_eos, uint32_t *out_tokens,
                      uint32_t *out_count, float *last_logits, orc_error *err) {
    orc_scratch *s = (orc_scratch *)calloc(1, sizeof *s);
    s->scores = (float *)calloc(capacity + 4, sizeof(float));
    float *logits = (float *)malloc(151936 * sizeof(float));
    uint32_t *history = (uint32_t *)malloc(((size_t)prompt_len + decode_steps + 1) * 4);
    uint8_t *seen = (uint8_t *)calloc(18992, 1);
    uint64_t state = seed == 0 ? 0x9e3779b97f4a7c15ull : seed, draws = 0;
    uint32_t status = 0, count = 0, position = 0;
    memcpy(history, prompt, (size_t)prompt_len * 4);
    for (uint32_t i = 0; i < prompt_len && status == 0; ++i, ++position)
        status = forward_scratch(file, kv, capacity, rope, prompt[i], position,
                                 i + 1 == prompt_len ? logits : NULL, err, s);
    while (status == 0 && count < decode_steps) {
        uint32_t selected = 0;
        status = orc_sample_with_repetition(logits, 151936, history, prompt_len + count, seen,
                                            18992, &state, &draws, &selected, err);
        if (status) break;
        out_tokens[count] = selected;
        history[prompt_len + count] = selected;
        ++count;
        if (stop_at_eos && (selected == 151643u || selected == 151645u)) break;
        if (count == decode_steps) break;
        status = forward_scratch(file, kv, capacity, rope, selected, position, logits, err, s);
        ++position;
    }
    if (out_count) *out_count = count;
    if (last_logits) memcpy(last_logits, logits, 151936 * sizeof(float));
    free(seen); free(history); free(logits); free(s->scores); free(s);
    return status;
}

typedef struct {
    const uint8_t *file;
    size_t capacity;
    const float *rope;
    uint32_t nseq, prompt_len, decode_steps;
    const uint32_t *prompts;
    const uint64_t *seeds;
    uint32_t *out_tokens;
    uint32_t next;
    uint32_t status;
    pthread_mutex_t lock;
} orc_pool;

static void *pool_worker(void *arg) {
    orc_pool *pool = (orc_pool *)arg;
    float *kv = (float *)calloc(24 * 2 * 2 * pool->capacity * 64, sizeof(float));
    for (;;) {
        pthread_mutex_lock(&pool->lock);
        uint32_t seq = pool->next++;
        pthread_mutex_unlock(&pool->lock);
        if (seq >= pool->nseq) break;
        uint32_t count = 0;
        orc_error err;
        uint32_t st = orc_generate(pool->file, kv, pool->capacity, pool->rope,
                                   pool->prompts + (size_t)seq * pool->prompt_len,
                                   pool->prompt_len, pool->decode_steps, pool->seeds[seq], 0,
                                   pool->out_tokens + (size_t)seq * pool->decode_steps, &count,
                                   NULL, &err);
        if (st) {
            pthread_mutex_lock(&pool->lock);
            pool->status = st;
            pthread_mutex_unlock(&pool->lock);
        }
    }
    free(kv);
    return NULL;
}

uint32_t orc_generate_many(const uint8_t *file, size_t capacity, const float *rope,
                           uint32_t nseq, const uint32_t *prompts, uint32_t prompt_len,
                           uint32_t decode_steps, const uint64_t *seeds, uint32_t threads,
                           uint32_t *out_tokens) {
    orc_pool pool;
    memset(&pool, 0, sizeof pool);
    pool.file = file; pool.capacity = capacity; pool.rope = rope; pool.nseq = nseq;
    pool.prompt_len = prompt_len; pool.decode_steps = decode_steps; pool.prompts = prompts;
    pool.seeds = seeds; pool.out_tokens = out_tokens;
    pthread_mutex_init(&pool.lock, NULL);
    if (threads < 1) threads = 1;
    pthread_t *tid = (pthread_t *)malloc(threads * sizeof(pthread_t));
    for (uint32_t t = 0; t < threads; ++t) pthread_create(&tid[t], NULL, pool_worker, &pool);
    for (uint32_t t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    pthread_mutex_destroy(&pool.lock);
    return pool.status;
}

/* CPU baseline of one batched-decode step per sequence (the reference's per-token
 * work: inference.rs:1454-1765 forward + inference.rs:919-965 sampler) from a
 * context of start_position tokens.  The KV below start_position is filled with
 * seeded values: the decode arithmetic's cost does not depend on them. */
typedef struct {
    const uint8_t *file;
    size_t capacity;
    const float *rope;
    uint32_t start, steps, nseq;
    const uint64_t *seeds;
    uint32_t *out_tokens;
    double *loop_seconds;
    uint32_t next;
    pthread_mutex_t lock;
} orc_bench;

static double now_seconds(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static void *bench_worker(void *arg) {
    orc_bench *b = (orc_bench *)arg;
    size_t kv_words = 24 * 2 * 2 * b->capacity * 64;
    float *kv = (float *)malloc(kv_words * sizeof(float));
    float *logits = (float *)malloc(151936 * sizeof(float));
    uint32_t *history = (uint32_t *)malloc(((size_t)b->start + b->steps + 1) * 4);
    uint8_t *seen = (uint8_t *)calloc(18992, 1);
    orc_scratch *s = (orc_scratch *)calloc(1, sizeof *s);
    s->scores = (float *)calloc(b->capacity + 4, sizeof(float));
    for (;;) {
        pthread_mutex_lock(&b->lock);
        uint32_t seq = b->next++;
        pthread_mutex_unlock(&b->lock);
        if (seq >= b->nseq) break;
        uint64_t lcg = b->seeds[seq] * 6364136223846793005ull + 1442695040888963407ull;
        for (size_t i = 0; i < kv_words; ++i) {
            lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
            kv[i] = (float)((int32_t)(lcg >> 40) - (1 << 23)) * (1.0f / 8388608.0f);
        }
        for (uint32_t i = 0; i < b->start; ++i) {
            lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
            history[i] = (uint32_t)((lcg >> 33) % 151643u);
        }
        uint64_t state = b->seeds[seq] == 0 ? 0x9e3779b97f4a7c15ull : b->seeds[seq], draws = 0;
        uint32_t token = history[b->start - 1];
        orc_error err;
        const double t0 = now_seconds();
        for (uint32_t t = 0; t < b->steps; ++t) {
            uint32_t pos = b->start + t;
            history[pos] = token;
            if (forward_scratch(b->file, kv, b->capacity, b->rope, token, pos, logits, &err, s)) break;
            uint32_t sel = 0;
            if (orc_sample_with_repetition(logits, 151936, history, pos + 1, seen, 18992, &state,
                                           &draws, &sel, &err))
                break;
            if (b->out_tokens) b->out_tokens[(size_t)seq * b->steps + t] = sel;
            token = sel;
        }
        if (b->loop_seconds) b->loop_seconds[seq] = now_seconds() - t0;
    }
    free(s->scores); free(s); free(seen); free(history); free(logits); free(kv);
    return NULL;
}

uint32_t orc_bench_decode(const uint8_t *file, size_t capacity, const float *rope,
                          uint32_t start_position, uint32_t steps, uint32_t nseq,
                          const uint64_t *seeds, uint32_t threads, uint32_t *out_tokens,
                          double *loop_seconds) {
    if (start_position == 0 || start_position + steps > capacity) return 2;
    orc_bench b;
    memset(&b, 0, sizeof b);
    b.file = file; b.capacity = capacity; b.rope = rope; b.start = start_position;
    b.steps = steps; b.nseq = nseq; b.seeds = seeds; b.out_tokens = out_tokens;
    b.loop_seconds = loop_seconds;
    pthread_mutex_init(&b.lock, NULL);
    if (threads < 1) threads = 1;
    pthread_t *tid = (pthread_t *)malloc(threads * sizeof(pthread_t));
    for (uint32_t t = 0; t < threads; ++t) pthread_create(&tid[t], NULL, bench_worker, &b);
    for (uint32_t t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    pthread_mutex_destroy(&b.lock);
    return 0;
}
