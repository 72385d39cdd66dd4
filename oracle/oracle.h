/*
 * CPU oracle for the promptboot decode hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's decode arithmetic
 * (sulewicz/promptboot, crates/promptboot-core/src/fp32_sse2.rs and
 * inference.rs).  It exists so the CUDA implementation can be checked bit for
 * bit.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load it; the product library never links or calls it.
 *
 * Parity pin: every function here is checked against the reference's own
 * golden vectors (fixtures/inference/kernels/ golden files, the expf edge table, the
 * sampler known-answer tests and the RoPE table SHA-256) by tests/.
 *
 * All floating-point values cross this interface as IEEE binary32/binary64 in
 * memory; the build uses -ffp-contract=off so that every a*b+c below is two
 * roundings, exactly as the reference's scalar SSE2 operations.
 */
#ifndef PROMPTBOOT_ORACLE_H
#define PROMPTBOOT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_HIDDEN 896
#define ORC_FFN 4864
#define ORC_LAYERS 24
#define ORC_QHEADS 14
#define ORC_KVHEADS 2
#define ORC_HEAD_DIM 64
#define ORC_VOCAB 151936
#define ORC_CONTEXT 32768
#define ORC_ROPE_WORDS (32768 * 32 * 2)
#define ORC_EOS 151645

typedef struct orc_error {
    uint32_t status, domain, layer, position, tensor_id, reserved;
    uint64_t needed, available, detail;
} orc_error;

/* elementary functions */
uint32_t orc_half_to_f32_bits(uint16_t bits);
uint16_t orc_f32_bits_to_half(uint32_t bits);
uint32_t orc_expf_bits(uint32_t bits);
void orc_expf4(uint32_t values[4]);

/* kernels (fp32_sse2.rs) */
void orc_q4_row(const uint8_t *weights, size_t row, float *out, size_t columns);
void orc_prepare_q8(const float *input, uint8_t *staging, size_t columns);
int32_t orc_q4_block_dot(const uint8_t *packed16, const int8_t *act32);
int32_t orc_q8_block_dot(const int8_t *weights32, const int8_t *act32);
void orc_q4_matvec(const uint8_t *weights, const uint8_t *staging, float *out,
                   size_t rows, size_t columns);
void orc_q8_matvec(const uint8_t *weights, const uint8_t *staging, float *out,
                   size_t rows, size_t columns);
void orc_rmsnorm(const float *input, const float *weight, float *out, size_t words);
void orc_rope_table(float *table);
void orc_rope_in_place(float *values, size_t heads, size_t position, const float *table);
size_t orc_kv_word(size_t capacity, size_t layer, size_t kind, size_t position,
                   size_t head, size_t component);
void orc_attention(const float *query, const float *kv, size_t capacity, size_t layer,
                   size_t current, size_t span, float *out, float *scores,
                   float *raw_capture, float *prob_capture);
void orc_swiglu(const float *gate, const float *up, float *out, size_t words);
uint32_t orc_argmax(const float *logits, size_t words);

/* sampler (fp32_sse2.rs:1787-1876, inference.rs:774-965) */
uint32_t orc_next_24(uint64_t *state, uint64_t *draws);
uint32_t orc_sample_top_k_top_p(const float *logits, size_t words, uint32_t random24);
void orc_apply_repetition_penalty(float *logits, const uint32_t *tokens, size_t count,
                                  uint8_t *seen);
/* sample_token_with_repetition: returns status (0 ok) and fills *err on failure */
uint32_t orc_sample_with_repetition(float *logits, size_t words, const uint32_t *tokens,
                                    size_t count, uint8_t *seen, size_t seen_len,
                                    uint64_t *state, uint64_t *draws, uint32_t *selected,
                                    orc_error *err);

/* model (PBTQW25 v1 tensor directory) and the token forward (inference.rs:1454-1765) */
const uint8_t *orc_tensor(const uint8_t *file, uint32_t id);
uint32_t orc_forward(const uint8_t *file, float *kv, size_t capacity, const float *rope,
                     uint32_t token, uint32_t position, float *logits, orc_error *err);
/* REPL-style generation (prefill -> sample -> decode_selected ...); returns status */
uint32_t orc_generate(const uint8_t *file, float *kv, size_t capacity, const float *rope,
                      const uint32_t *prompt, uint32_t prompt_len, uint32_t decode_steps,
                      uint64_t seed, int stop_at_eos, uint32_t *out_tokens,
                      uint32_t *out_count, float *last_logits, orc_error *err);
/* independent sequences on worker threads (CPU baseline); tokens out [n][decode_steps] */
uint32_t orc_generate_many(const uint8_t *file, size_t capacity, const float *rope,
                           uint32_t nseq, const uint32_t *prompts, uint32_t prompt_len,
                           uint32_t decode_steps, const uint64_t *seeds, uint32_t threads,
                           uint32_t *out_tokens);

/* CPU baseline: nseq independent sequences on worker threads, each decoding
 * `steps` tokens (forward + sampler) from start_position over a seeded KV */
uint32_t orc_bench_decode(const uint8_t *file, size_t capacity, const float *rope,
                          uint32_t start_position, uint32_t steps, uint32_t nseq,
                          const uint64_t *seeds, uint32_t threads, uint32_t *out_tokens,
                          double *loop_seconds);

#ifdef __cplusplus
}
#endif
#endif
