/*
 * promptboot_b200 -- C ABI of the B200 (sm_100a) decode hot path.
 *
 * Drop-in boundary for promptboot-core's model-forward and sampler entry points
 * (sulewicz/promptboot).  Every call returns a u32 status (0 = OK) and reports
 * failures through the 48-byte pb_error, whose layout and numbering are the
 * reference's InferenceError (crates/promptboot-core/src/inference.rs:155-264).
 * Floats never cross this ABI as floats: logits are binary32 bit patterns in
 * uint32_t, as in the reference (fp32_sse2.rs:1-6).  No C++ or torch types
 * appear here; pointers are host pointers unless the name says _device.
 *
 * Threading: a pb_engine is single-owner (like the reference's &mut engine);
 * use one engine per GPU and one host thread per engine.
 */
#ifndef PROMPTBOOT_B200_H
#define PROMPTBOOT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PB_API __attribute__((visibility("default")))
#else
#define PB_API
#endif

#define PB_ABI_VERSION 1u
#define PB_VOCAB 151936u
#define PB_CONTEXT_LIMIT 32768u
#define PB_MODEL_BYTES 426762944ull
#define PB_SEEN_BYTES 18992u

/* InferenceStatus (inference.rs:155-169) */
enum {
    PB_OK = 0, PB_STATE = 1, PB_CONTEXT = 2, PB_TOKEN_ID = 3, PB_CAPACITY = 4,
    PB_ALIGNMENT = 5, PB_NONFINITE_INPUT = 6, PB_NONFINITE_OUTPUT = 7, PB_MODEL = 8,
    PB_ARITHMETIC = 9, PB_FAULTED = 10,
    PB_DEVICE = 100 /* CUDA runtime failure; no reference counterpart */
};

/* InferenceState (inference.rs:217-224) */
enum { PB_STATE_RESET = 0, PB_STATE_READY = 1, PB_STATE_EOS = 2, PB_STATE_FAULTED = 3 };

/* pb_model_open flags: the synthetic images used here carry zeroed tokenizer
 * sections, so only the layout (header, sections, tensor directory) is checked. */
enum { PB_MODEL_LAYOUT_ONLY = 1u };

/* InferenceError (inference.rs:226-238), 48 bytes */
typedef struct pb_error {
    uint32_t status, domain, layer, position, tensor_id, reserved;
    uint64_t needed, available, detail; /* detail = (field_kind << 32) | sub */
} pb_error;

/* InferenceStep (inference.rs:266-273), 16 bytes */
typedef struct pb_step {
    uint32_t position, selected_token, selected_logit_bits, eos;
} pb_step;

/* ArenaUsage (arena.rs) and InferenceUsage (inference.rs:275-285), 136 bytes */
typedef struct pb_arena_usage {
    uint64_t capacity, requested, committed, current, high_water;
} pb_arena_usage;
typedef struct pb_usage {
    pb_arena_usage weights, kv, scratch;
    uint32_t position, context_limit, generation_reserve, state;
} pb_usage;

/* SamplingState (inference.rs:772-799), 16 bytes */
typedef struct pb_sampling_state { uint64_t state, draws; } pb_sampling_state;

/* TopLogit (inference.rs:759-770), 8 bytes */
typedef struct pb_top_logit { uint32_t token, logit_bits; } pb_top_logit;

/* ModelError (model.rs:113-124), 48 bytes */
typedef struct pb_model_error {
    uint32_t status, domain, index, reserved;
    uint64_t offset, needed, available, detail;
} pb_model_error;

typedef struct pb_model pb_model;
typedef struct pb_engine pb_engine;

PB_API uint32_t pb_abi_version(void);
/* Text of the last CUDA/runtime failure seen on this thread ("" when none). */
PB_API const char *pb_last_error_string(void);

/* ------------------------------------------------------------------ model
 * Replaces ModelView::open_authenticated (model.rs:371-629) + tensor/tensor_for
 * (model.rs:652-720).  Validates the PBTQW25 v1 layout, then uploads section 7
 * (tensor data) to `device` unchanged, in PBTQW25 byte order. */
PB_API uint32_t pb_model_open(const uint8_t *bytes, uint64_t len, uint32_t flags, int device,
                       pb_model **out, pb_model_error *err);
PB_API void pb_model_close(pb_model *model);
/* Device pointer of tensor `id` (model.rs:652) or NULL. */
PB_API const void *pb_model_tensor_device(const pb_model *model, uint32_t id);

/* ----------------------------------------------------------------- engine
 * Replaces InferenceEngine (inference.rs:967-1371).  One engine owns
 * `max_seqs` independent sequences ("slots"), each with its own KV cache of
 * `max_context` positions (<= 32768; the reference's fixed KV is 32768) in the
 * reference's tiled layout, its own state machine and retained prefix. */
PB_API uint32_t pb_engine_create(pb_model *model, uint32_t max_seqs, uint32_t max_context,
                          pb_engine **out, pb_error *err);
PB_API void pb_engine_destroy(pb_engine *engine);

/* inference.rs:1026 prefill / :1044 prefill_with_prefix / :1095 append_prefill.
 * `logits` (optional) receives the 151936 binary32 words of the last token. */
PB_API uint32_t pb_engine_prefill(pb_engine *engine, uint32_t seq, const uint32_t *tokens, uint32_t n,
                           uint32_t generation_reserve, uint32_t *logits, pb_step *step,
                           pb_error *err);
PB_API uint32_t pb_engine_prefill_with_prefix(pb_engine *engine, uint32_t seq, const uint32_t *tokens,
                                       uint32_t n, uint32_t prefix_tokens,
                                       uint32_t generation_reserve, uint32_t *logits,
                                       pb_step *step, pb_error *err);
PB_API uint32_t pb_engine_append_prefill(pb_engine *engine, uint32_t seq, const uint32_t *tokens,
                                  uint32_t n, uint32_t generation_reserve, uint32_t *logits,
                                  pb_step *step, pb_error *err);
/* inference.rs:1205 decode (token must equal the last greedy id) / :1213 decode_selected */
PB_API uint32_t pb_engine_decode(pb_engine *engine, uint32_t seq, uint32_t token, uint32_t *logits,
                          pb_step *step, pb_error *err);
PB_API uint32_t pb_engine_decode_selected(pb_engine *engine, uint32_t seq, uint32_t token,
                                   uint32_t *logits, pb_step *step, pb_error *err);
/* inference.rs:1307 reset / :1315 reset_to_prefix / :1337 usage / :1369 position */
PB_API uint32_t pb_engine_reset(pb_engine *engine, uint32_t seq);
PB_API uint32_t pb_engine_reset_to_prefix(pb_engine *engine, uint32_t seq, uint32_t *prefix_out);
PB_API uint32_t pb_engine_usage(pb_engine *engine, uint32_t seq, pb_usage *out);
PB_API uint32_t pb_engine_position(pb_engine *engine, uint32_t seq);

/* KV snapshot access (no counterpart in the reference, whose KV is a caller-
 * owned byte slice: InferenceEngine::build, inference.rs:977-1011).
 * pb_engine_kv_device returns the device address of slot `seq`'s KV region,
 * *words binary32 words = max_context * 6144, in the reference's tiled layout
 * (inference.rs:2035-2052) with the slot's capacity C in place of 32768:
 * K at layer*4C*64 + ((h*C/4 + p/4)*64 + c)*4 + p%4, V at layer*4C*64 + 2C*64 +
 * (h*C + p)*64 + c.  Reads and writes through it are the caller's, ordered
 * against the engine by synchronizing pb_engine_stream.
 * pb_engine_restore makes a RESET slot hold `tokens` (n < context limit) whose
 * KV of positions [0, n) the caller has written there (a saved snapshot):
 * prefill's prechecks (inference.rs:1109-1191) on tokens and reserve, then the
 * slot is READY at position n with history = tokens and no greedy id, so the
 * next call is decode_selected (decode reports the selected-token state error). */
PB_API void *pb_engine_kv_device(pb_engine *engine, uint32_t seq, uint64_t *words);
PB_API uint32_t pb_engine_restore(pb_engine *engine, uint32_t seq, const uint32_t *tokens, uint32_t n,
                                  uint32_t generation_reserve, pb_error *err);

/* Batched forms: one forward step over n distinct sequences at their own
 * positions (a sequence listed twice: PB_CAPACITY).  prefill_batch runs `len`
 * prompt tokens per sequence (tokens is [n][len]; positions but the last as
 * batched (sequence, position) rows, results as the token-serial reference);
 * decode_batch evaluates tokens[i] for seqs[i] (require_greedy = 1 is decode, 0
 * is decode_selected).  Per-sequence results land in steps[i]/errs[i]; the call
 * returns PB_OK when every sequence succeeded, else the first failing status.
 * Logits stay on the device (row i = seqs[i]); see pb_engine_logits. */
PB_API uint32_t pb_engine_prefill_batch(pb_engine *engine, uint32_t n, const uint32_t *seqs,
                                 const uint32_t *tokens, uint32_t len,
                                 uint32_t generation_reserve, pb_step *steps, pb_error *errs);
PB_API uint32_t pb_engine_decode_batch(pb_engine *engine, uint32_t n, const uint32_t *seqs,
                                const uint32_t *tokens, uint32_t require_greedy,
                                pb_step *steps, pb_error *errs);
/* Copies the logits row of batch row `row` of the last step to host. */
PB_API uint32_t pb_engine_logits(pb_engine *engine, uint32_t row, uint32_t *logits);
/* sample_token_with_repetition (inference.rs:919-965) on batch rows 0..n-1 of the
 * last step, history = every token seqs[i] has evaluated; states are host
 * SamplingStates updated in place; ids[i] = sampled token. */
PB_API uint32_t pb_engine_sample(pb_engine *engine, uint32_t n, const uint32_t *seqs,
                          pb_sampling_state *states, uint32_t *ids, pb_error *errs);
/* Device-resident generation (benchmark mode: fixed length, EOS not honoured):
 * `steps` times { sample the current logits rows with repetition history, then
 * decode_selected(sampled) }, all on the GPU.  Requires every seq READY/EOS with
 * logits from its last step in batch row i.  out_tokens (optional, host) is
 * [steps][n]. */
PB_API uint32_t pb_engine_generate(pb_engine *engine, uint32_t n, const uint32_t *seqs,
                            pb_sampling_state *states, uint32_t steps, uint32_t *out_tokens,
                            pb_error *errs);

/* Engine instrumentation (no reference counterpart): the CUDA stream every
 * engine kernel runs on, the number of kernels launched so far, and optional
 * CUDA-event timing of selected kernel classes (bit i of class_mask = class i
 * below) accumulated on that stream; pb_engine_profile also resets the sums. */
enum {
    PB_KC_EMBED = 0, PB_KC_NORM = 1, PB_KC_GEMV = 2, PB_KC_ROPE_KV = 3, PB_KC_ATTENTION = 4,
    PB_KC_QUANT = 5, PB_KC_SWIGLU = 6, PB_KC_LM_HEAD = 7, PB_KC_ARGMAX = 8, PB_KC_SAMPLER = 9
};
PB_API void *pb_engine_stream(pb_engine *engine);
PB_API uint64_t pb_engine_launch_count(pb_engine *engine);
PB_API uint32_t pb_engine_profile(pb_engine *engine, uint32_t class_mask);
PB_API uint32_t pb_engine_profile_read(pb_engine *engine, double *ms16, uint64_t *launches16);

/* ---------------------------------------------------------------- sampler
 * Host-buffer forms of the reference's sampler entry points, executed on the
 * GPU (inference.rs:814-965).  Error fields match the reference. */
PB_API void pb_sampling_state_init(pb_sampling_state *state, uint64_t seed);
PB_API uint32_t pb_sample_token(const uint32_t *logits, uint64_t len, pb_sampling_state *state,
                         uint32_t *out, pb_error *err);
PB_API uint32_t pb_sample_token_with_repetition(uint32_t *logits, uint64_t len, const uint32_t *tokens,
                                         uint64_t count, uint8_t *seen, uint64_t seen_len,
                                         pb_sampling_state *state, uint32_t *out, pb_error *err);
PB_API uint32_t pb_greedy_token(const uint32_t *logits, uint64_t len, uint32_t *out, pb_error *err);
PB_API uint32_t pb_top_logits_8(const uint32_t *logits, uint64_t len, pb_top_logit *out8, pb_error *err);

/* Device batch sampler: rows of binary32 logits (row stride ld words) mutated in
 * place by the penalty; history for row r is history[offsets[r] .. +lengths[r]];
 * states [rows] updated; out [rows] receives {status, index, value, selected}
 * (status 0 ok, 3 TOKEN_ID at history index/value, 7 NONFINITE_OUTPUT at
 * logit index/bits).  Asynchronous on `stream` (a cudaStream_t, NULL = default). */
PB_API uint32_t pb_sample_batch_device(uint32_t *logits_device, uint64_t ld, uint32_t rows,
                                const uint32_t *history_device, const uint64_t *offsets_device,
                                const uint32_t *lengths_device,
                                pb_sampling_state *states_device, uint32_t *out_device,
                                void *stream);

/* --------------------------------------------------------- kernel operators
 * Device-pointer operators behind the engine, for tests and operator sweeps.
 * All are asynchronous on `stream`. */
/* y[b][r] = Q4_0 (wtype 2) or Q8_0 (wtype 3) weights [rows][cols] times the
 * Q8_0-quantized x[b] (fp32_sse2.rs:945-983, 1217-1281); x is f32 [batch][cols].
 * Scratch: the quantized x; allocated per call. */
PB_API uint32_t pb_qmatvec_device(uint32_t wtype, const uint8_t *w_device, uint32_t rows, uint32_t cols,
                           const float *x_device, uint32_t batch, float *y_device, void *stream);
/* The same operator without any device allocation (no counterpart in the
 * reference): for callers that cannot allocate device memory on this path,
 * e.g. hosts that own the GPU's memory budget through their own allocator,
 * latency-critical loops, or fixed-arena integrations like promptboot's own
 * firmware runtime.  Its scratch is one file-scope device array of 192 KiB
 * held by each GPU that loads the library; batch is limited to 32 rows and
 * cols to 4864 (PB_CAPACITY otherwise, see pb_last_error_string).  The first
 * call on a device sets it up and should come before any stream capture; all
 * calls share the array, so calls whose kernels overlap on the GPU (queued on
 * different streams, from any thread) race; calls queued on one stream are
 * ordered by it.  Unlike pb_qmatvec_device it does not wait: it returns once
 * the work is queued on `stream`, and y is ready when that stream has reached
 * it.  Non-finite outputs are not reported (y holds them as computed).  The
 * array's device address is looked up once per device for the process, so the
 * call must not be used after a cudaDeviceReset of that device. */
PB_API uint32_t pb_qmatvec_device_noalloc(uint32_t wtype, const uint8_t *w_device, uint32_t rows,
                                          uint32_t cols, const float *x_device, uint32_t batch,
                                          float *y_device, void *stream);
/* y[b] = model tensor `tensor_id` (a layer's q/k/v/o/gate/up/down matrix, the
 * Q8_0 output head, id 290, or the Q4_0 token embedding, id 0, as a tied
 * 896 -> 151936 head) times the Q8_0-quantized x[b], x f32 [batch][cols]:
 * the engine's own matvec (the tensor-core path on the model's tile image from
 * 9 rows, the CUDA-core path below).  Asynchronous on `stream`, no per-call
 * allocation once the model's scratch has grown to the batch (batch <= 256;
 * tensor 0's tile image is built on its first call from 9 rows);
 * pb_model_matvec_status synchronizes `stream` and reports a pipeline timeout of
 * any earlier call (PB_DEVICE) once.  Replaces the row loop of
 * inference_q4_matvec_rows_prepared / inference_q8_matvec_rows_prepared
 * (fp32_sse2.rs:1217-1281) over ModelView::tensor (model.rs:652). */
PB_API uint32_t pb_model_matvec_device(pb_model *model, uint32_t tensor_id, const float *x_device,
                                       uint32_t batch, float *y_device, void *stream);
PB_API uint32_t pb_model_matvec_status(pb_model *model, void *stream);
/* Q8_0 staging in the reference's 34-byte block format for [rows][cols] f32. */
PB_API uint32_t pb_quantize_q8_device(const float *x_device, uint32_t rows, uint32_t cols,
                               uint8_t *staging_device, void *stream);
/* RMSNorm (fp32_sse2.rs:1310-1334) of [rows][896] into y; x, w and y 16-byte
 * aligned (PB_CAPACITY otherwise). */
PB_API uint32_t pb_rmsnorm_device(const float *x_device, const float *w_device, uint32_t rows,
                           float *y_device, void *stream);
/* SwiGLU (fp32_sse2.rs:1751-1770) of [rows][4864]. */
PB_API uint32_t pb_swiglu_device(const float *gate_device, const float *up_device, uint32_t rows,
                          float *out_device, void *stream);
/* RoPE on q [rows][896] and k [rows][128] in place at positions[r]
 * (fp32_sse2.rs:1413-1428); v [rows][128]; both written to the KV of slot r. */
PB_API uint32_t pb_rope_kv_device(float *q_device, float *k_device, const float *v_device,
                           const uint32_t *positions_host, uint32_t rows, float *kv_device,
                           uint32_t capacity, uint32_t layer, void *stream);
/* GQA decode attention (fp32_sse2.rs:1430-1672) of q [rows][896] over the KV of
 * slot r at current positions[r]; span (0 = natural) pads the softmax span.
 * capacity and span at most 32768 (the reference's context), capacity a
 * multiple of 4 (PB_CAPACITY otherwise).
 * scores_device (optional) receives [rows][14][span_max] final probabilities. */
PB_API uint32_t pb_attention_device(const float *q_device, const float *kv_device, uint32_t capacity,
                             uint32_t layer, const uint32_t *positions_host, uint32_t rows,
                             uint32_t span, float *out_device, float *scores_device,
                             void *stream);
/* The 8 MiB RoPE table (32768 x 32 x {cos, sin}) the engine uploads; built from
 * glibc powf/cosf/sinf and checked against the reference's SHA-256. */
PB_API uint32_t pb_rope_table(float *table_host);
/* y[i] = the sampler's binary32 exponential of x[i] (bit patterns), the device
 * routine the top-k/top-p weights use: fp32_sse2.rs:378-469 (scalbnf, expf). */
PB_API uint32_t pb_expf_device(const uint32_t *x_device, uint64_t n, uint32_t *y_device, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* PROMPTBOOT_B200_H */
