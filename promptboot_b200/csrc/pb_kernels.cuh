// Launch-side declarations of the decode kernels (implemented in pb_kernels.cu
// and pb_sampler.cu).  Everything here is device pointers and sizes; the host
// engine (pb_engine.cu) sequences these per token step.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace pb {

// Launches `kernel` with programmatic stream serialization (the kernel begins
// with pdl_begin()), so its launch and prologue overlap the previous kernel.
// Kernel attributes belong to a device's context: `done` records the devices
// (bit per ordinal) whose attribute has been set.  Set first, then mark, so two
// threads at most both set it (idempotent).
inline bool attribute_needed(const std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return true;
  return !(done.load() & (1ull << dev));
}
inline void attribute_done(std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) done.fetch_or(1ull << dev);
}

// Whether this host thread's launch_pdl calls ask for programmatic
// serialization (PdlOff turns it off for a scope; the kernels' griddepcontrol
// instructions are then no-ops).
inline thread_local bool t_pdl_enabled = true;
struct PdlOff {
  bool saved;
  explicit PdlOff(bool off) : saved(t_pdl_enabled) { if (off) t_pdl_enabled = false; }
  ~PdlOff() { t_pdl_enabled = saved; }
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_pdl_enabled ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Per-row buffers of one forward batch; row b of every [B][...] array belongs to
// engine slot slots[b], which owns KV region slots[b] and writes position
// positions[b] this step.
struct Batch {
  int rows;                 // B
  const int* slots;         // [B]
  const int* positions;     // [B]
  const uint32_t* tokens;   // [B] token evaluated this step
  float* hidden;            // [B][896] residual stream
  int8_t* aq;               // [B][4864] Q8_0 activation quants
  float* ad;                // [B][152] activation scales (binary16 value as f32)
  int* asum;                // [B][152] sum of the 32 quants of each block
  float* q;                 // [B][896]
  float* k;                 // [B][128]
  float* v;                 // [B][128]
  float* attn;              // [B][896]
  float* gate;              // [B][4864]
  float* up;                // [B][4864]
  float* logits;            // [B][151936]
  float* scores;            // [B][14][score_stride] attention scratch
  size_t score_stride;
  float* kv;                // slot-major KV cache
  size_t capacity;          // positions per slot
  uint32_t* history;        // [slots][capacity] tokens evaluated so far
  unsigned long long* err;  // [B] ranked first stage failure
  float* norm_out = nullptr;     // optional [B][896] RMSNorm output (operator API)
  float* product_out = nullptr;  // optional [B][4864] SwiGLU output (operator API)
  int span_min = 0;              // minimum softmax span (operator API; 0 = natural)
  float* probs_out = nullptr;    // optional [B][14][score_stride] final probabilities
  // Every V word below each row's position came from this engine's own
  // forwards, whose v-projection stage check faults a row on a non-finite
  // word before it is written (rows read after such a fault are discarded),
  // so attention need not re-check V.
  bool kv_checked = false;
  // Tensor-core activation layout, written by the quantizers when aq_tc is set
  // (instead of the row-major aq/ad/asum),
  // chunk-major (4 Q-blocks per chunk) so one chunk of one sequence tile is one
  // contiguous copy: [K / 128][tc_seqs / 8][kTcGroupBytes], each 8-sequence
  // group = 4 blocks x 256 B of quants (bytes 0-15 of the 8 rows, then bytes
  // 16-31) followed by the [4 blocks][8 sequences] binary32 scales.
  int8_t* aq_tc = nullptr;
  int tc_seqs = 0;               // multiple of 64, >= rows
};

// Longest softmax span the shared-memory attention path holds; longer contexts
// keep the probabilities in the global score scratch.
constexpr int kAttnMaxPositions = 2048;
// Batches of at most kAttnSplitRows rows over more than kAttnSplitMinSpan
// positions take the split (global-scratch) path at any span.
constexpr int kAttnSplitRows = 64;
constexpr int kAttnSplitMinSpan = 256;

enum EpiMode : int { EPI_STORE = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2 };

struct Epilogue {
  int mode;
  float* out;             // output base (row b at out + b * ld)
  size_t ld;
  const float* bias;      // EPI_BIAS
  unsigned long long* err;
  uint32_t layer_ordinal;
  uint32_t domain;
};

enum WeightType : int { W_Q4_0 = 2, W_Q8_0 = 3 };

// Kernel launchers (stream-ordered, asynchronous).
void launch_embed(const Batch& b, const uint8_t* embedding, cudaStream_t s);
void launch_rmsnorm_quant(const Batch& b, const float* weight, uint32_t layer_ordinal,
                          uint32_t domain, cudaStream_t s);
void launch_quant(const Batch& b, const float* x, size_t ld, int columns, cudaStream_t s);
void launch_qgemv(int wtype, const uint8_t* w, int rows, int columns, const Batch& b,
                  const Epilogue& ep, cudaStream_t s);

// tcgen05 kind::i8 path (pb_gemm_tc.cu) for batches above 8 rows.  The weights
// are read from a tile image (launch_tc_repack): per 128-row tile and chunk of
// 4 Q-blocks, kTcChunkBytes = 4 canonical int8 tiles + 128 x 4 f32 scales.
constexpr int kTcChunkBytes = 18432;
constexpr int kTcGroupBytes = 4 * 256 + 4 * 8 * 4;  // 1152
// Bytes of the tensor-core activation layout for tc_seqs sequences and K columns.
constexpr size_t tc_act_bytes(int tc_seqs, int columns) {
  return (size_t)(columns / 128) * (tc_seqs / 8) * kTcGroupBytes;
}
constexpr int kTcMinBatch = 9;
bool tc_shape_supported(int rows, int columns);
size_t tc_image_bytes(int rows, int columns);
void launch_tc_repack(int wtype, const uint8_t* w, int rows, int columns, uint8_t* out,
                      cudaStream_t s);
// Up to three matrices stacked by row tiles in one image and one launch (q/k/v,
// gate/up); segment i covers row tiles [seg[i-1].rtile_end, seg[i].rtile_end)
// and writes through its own epilogue with rows numbered from 0.
struct TcSegment {
  int rtile_end;
  Epilogue ep;
};
struct TcGemm {
  int wtype;
  const uint8_t* tiles;
  int rtiles;
  int nb;  // Q-blocks per row (K / 32)
  int nseg;
  TcSegment seg[3];
  // Bits of -0.0f, passed at run time: fl(a * b) is formed as fma(a, b, -0.0)
  // with an addend the assembler cannot see, so it can never merge that product
  // with the following accumulation into one fused operation.
  uint32_t neg_zero_bits = 0x80000000u;
};
int tc_pick_config(int rtiles, int batch);
// Sets *status (device word) if a pipeline wait timed out.
void launch_tc_gemm(const TcGemm& g, const Batch& b, unsigned int* status, cudaStream_t s);
// Small-batch (B <= 8) matvec on CUDA cores (pb_gemv_small.cu): up to three
// matrices stacked by rows (segment i covers launch rows [seg[i-1].rows_end,
// seg[i].rows_end) and reads seg[i].w from its row 0), or in SwiGLU mode a
// gate/up pair (seg[0] gate, seg[1] up, the same 4864 rows) whose products are
// SwiGLU'd and quantized to the row-major Q8_0 activation.  rt rows per CTA
// (32 in SwiGLU mode) must divide every segment.
struct SmallGemv {
  int wtype;
  int cols;
  int rt;
  int nseg;
  struct Seg {
    const uint8_t* w;
    int rows_end;
    Epilogue ep;
  } seg[3];
  int swiglu;
  uint32_t swiglu_ordinal;
  // Optional RMSNorm + Q8_0 prologue (cols 896): the activations are computed
  // from Batch::hidden with this norm weight instead of read from Batch::aq,
  // every CTA repeating the small exact computation instead of a separate launch.
  const float* norm_weight = nullptr;
  uint32_t norm_ordinal = 0, norm_domain = 0;
};
bool small_gemv_supported(const SmallGemv& g, int batch);
// Sets *status (device word) if a weight copy did not land in time.
void launch_small_gemv(const SmallGemv& g, const Batch& b, unsigned int* status, cudaStream_t s);
void launch_rope_kv(const Batch& b, int layer, const float* rope, cudaStream_t s);
// max_span: the largest softmax span of the batch, (position + 4) & ~3 (or span_min).
// quantize: also write the Q8_0 activation of the output (the o-projection input).
// rope (optional): apply RoPE to q/k and write this step's K/V first (what
// launch_rope_kv does), fused into the attention launch; only when every row
// of the batch has its own slot.
// Both return the number of kernels they launched.
int launch_attention(const Batch& b, int layer, int max_span, bool quantize, const float* rope,
                     cudaStream_t s);
int launch_attention_grouped(const Batch& b, int layer, int span_cap, bool quantize, const float* rope,
                             cudaStream_t s);
// Beyond kAttnMaxPositions: scores, then the softmax and the PV chains over
// probabilities kept in the global score scratch (Batch::scores).
int launch_attention_long(const Batch& b, int layer, int span_cap, bool quantize, const float* rope,
                          cudaStream_t s);
void launch_swiglu_quant(const Batch& b, uint32_t layer_ordinal, cudaStream_t s);
void launch_argmax(const float* logits, size_t ld, int rows, int words, uint32_t* ids,
                   uint32_t* bits, unsigned long long* first_nonfinite, cudaStream_t s);
void launch_topk8(const float* logits, size_t ld, int rows, int words, uint32_t* out_pairs,
                  unsigned long long* first_nonfinite, cudaStream_t s);

// Sampler: rows of logits mutated in place by the repetition penalty, then one
// draw per row from states[row]; out[row] = selected id.  status[row] != 0 marks
// a rejected row (nothing mutated, no draw); detail[row] carries the reference's
// error fields (see pb_sampler.cu).
struct SamplerRow {
  uint32_t status;       // 0 ok, 3 TOKEN_ID, 7 NONFINITE_OUTPUT
  uint32_t index;        // offending logit index or history position
  uint32_t value;        // offending bits or token id
  uint32_t selected;
};
void launch_sampler(float* logits, size_t ld, int rows, int words, const uint32_t* history,
                    const uint64_t* hist_offset, const uint32_t* hist_len,
                    const uint8_t* initial_seen, unsigned long long* states, SamplerRow* out,
                    cudaStream_t s);
// The same sampler for few rows: each row's vocabulary split over kSplitParts
// CTAs, then one merge CTA per row (two launches).  cand: device scratch of
// split_sampler_words(rows) 64-bit words.
constexpr int kSplitParts = 32;
constexpr int kSplitSamplerMaxRows = 32;
constexpr size_t split_sampler_words(int rows) { return (size_t)rows * kSplitParts * 21; }
void launch_sampler_split(float* logits, size_t ld, int rows, int words, const uint32_t* history,
                          const uint64_t* hist_offset, const uint32_t* hist_len,
                          const uint8_t* initial_seen, unsigned long long* states, SamplerRow* out,
                          unsigned long long* cand, cudaStream_t s);

void init_kernel_attributes();

}  // namespace pb
