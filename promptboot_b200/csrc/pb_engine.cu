// The decode engine: per-sequence state machine of the reference's
// InferenceEngine (sulewicz/promptboot crates/promptboot-core/src/inference.rs:
// 967-1371) over a batched, device-resident forward (inference.rs:1454-1765).
//
// One pb_engine owns `max_seqs` slots.  Every slot has its own KV cache in the
// reference's tiled layout (inference.rs:2035-2052, context capacity as a
// parameter), token history, position, reserve and retained prefix.  A forward
// step evaluates one token for each of n slots with one launch per kernel; the
// stage checks of inference.rs:1889-1936 are folded into the kernels as a
// ranked per-row error word read back after the step.
#include "pb_common.cuh"
#include "pb_host.h"
#include "pb_kernels.cuh"

#include <algorithm>
#include <cstdlib>
#include <initializer_list>
#include <vector>

namespace {

constexpr uint32_t NO_LAYER = 0xffffffffu;
constexpr uint32_t NO_TENSOR = 0xffffffffu;
constexpr uint32_t kMaxPrefix = 599;  // tokenizer.rs:35 MAX_TOKENS

// InferenceDomain / InferenceFieldKind numbering (inference.rs:171-215)
enum : uint32_t { DOM_PROMPT = 2, DOM_KV = 9, DOM_LOGITS = 18, DOM_ARGMAX = 19 };
enum : uint32_t {
  K_STATE = 1, K_TOKEN = 2, K_CONTEXT = 3, K_BYTES = 4, K_FINITE = 7, K_RESERVE = 11,
  K_LOGITS = 12, K_SELECTED = 14,
};

pb_error make_error(uint32_t status, uint32_t domain, uint32_t layer, uint32_t position,
                    uint32_t tensor, uint64_t needed, uint64_t available, uint32_t kind,
                    uint32_t sub) {
  pb_error e;
  e.status = status; e.domain = domain; e.layer = layer; e.position = position;
  e.tensor_id = tensor; e.reserved = 0; e.needed = needed; e.available = available;
  e.detail = ((uint64_t)kind << 32) | sub;
  return e;
}

uint32_t layer_tensor(uint32_t layer, uint32_t role) { return 1 + layer * 12 + (role - 10); }

// Decodes the ranked stage-failure word written by the kernels (see
// pb_common.cuh error_key) into the reference's InferenceError for that stage.
pb_error stage_error(unsigned long long key, uint32_t position) {
  uint64_t rank = key >> 50;
  uint32_t index = (uint32_t)((key >> 32) & 0x3ffffu);
  uint32_t bits = (uint32_t)key;
  uint32_t sub = rank & 1u;
  uint32_t domain = (uint32_t)((rank >> 1) & 31u);
  uint32_t ordinal = (uint32_t)(rank >> 6);
  uint32_t layer = (ordinal >= 1 && ordinal <= 24) ? ordinal - 1 : NO_LAYER;
  uint32_t tensor = NO_TENSOR;
  switch (domain) {
    case pb::D_EMBEDDING: tensor = 0; break;
    case pb::D_ATTN_NORM: tensor = layer_tensor(layer, 10); break;
    case pb::D_Q: tensor = layer_tensor(layer, 19); break;
    case pb::D_K: tensor = layer_tensor(layer, 16); break;
    case pb::D_V: tensor = layer_tensor(layer, 21); break;
    case pb::D_ROPE: tensor = layer_tensor(layer, sub ? 16 : 19); break;
    case pb::D_KV: tensor = layer_tensor(layer, 16); break;
    case pb::D_ATTENTION: tensor = NO_TENSOR; break;
    case pb::D_ATTN_OUTPUT: tensor = layer_tensor(layer, 17); break;
    case pb::D_FFN_NORM: tensor = layer_tensor(layer, 14); break;
    case pb::D_GATE: tensor = layer_tensor(layer, 12); break;
    case pb::D_UP: tensor = layer_tensor(layer, 13); break;
    case pb::D_SWIGLU: tensor = layer_tensor(layer, 12); break;
    case pb::D_DOWN: tensor = layer_tensor(layer, 11); break;
    case pb::D_OUTPUT_NORM: tensor = 289; break;
    case pb::D_LOGITS: tensor = 290; break;
    default: break;
  }
  uint32_t status = domain <= pb::D_DOWN ? PB_NONFINITE_INPUT : PB_NONFINITE_OUTPUT;
  return make_error(status, domain, layer, position, tensor, 0, bits, K_FINITE, index);
}

struct Slot {
  uint32_t state = PB_STATE_RESET;
  uint32_t position = 0;
  uint32_t reserve = 0;
  uint32_t emitted = 0;
  uint32_t last_selected = 0;
  std::vector<uint32_t> prefix;  // retained prefix (inference.rs:689-704)
  uint64_t kv_high_water = 0;
  uint64_t scratch_high_water = 0;
};

template <typename T>
cudaError_t dalloc(T** p, size_t count) {
  return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T));
}

// The generate loop's per-step bookkeeping kernels.  A row's step index
// within the current chunk is positions[i] - base[i] (base = its position when
// the chunk began), so every step enqueues the same launches with the same
// arguments and one captured CUDA graph replays any step.
__global__ void take_sample_kernel(const pb::SamplerRow* sampled, uint32_t* tokens,
                                   const int* positions, const int* base,
                                   unsigned long long* status_log, uint32_t* token_log, int n) {
  pb::pdl_begin();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const pb::SamplerRow r = sampled[i];
  const size_t at = (size_t)(positions[i] - base[i]) * n + i;
  tokens[i] = r.selected;
  token_log[at] = r.selected;
  status_log[at] = r.status ? (((unsigned long long)r.status << 56) |
                               ((unsigned long long)r.index << 32) | r.value)
                            : pb::kNoError;
}

__global__ void finish_step_kernel(int* positions, const int* base, const unsigned long long* err,
                                   unsigned long long* err_log, int n) {
  pb::pdl_begin();
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  err_log[(size_t)(positions[i] - base[i]) * n + i] = err[i];
  positions[i] += 1;
}

}  // namespace

struct pb_engine {
  pb_model* model = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t max_seqs = 0;
  // Rows of one forward: the decode batch (max_seqs) or a prefill chunk of
  // (sequence, prompt position) rows, whichever is larger.
  uint32_t rows_cap = 0;
  static constexpr uint32_t kPrefillRows = 512;
  uint32_t capacity = 0;       // positions per slot (KV)
  uint32_t context_limit = 0;  // min(32768, capacity)
  std::vector<Slot> slots;

  // device buffers
  float* kv = nullptr;
  uint32_t* history = nullptr;
  float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
  float *gate = nullptr, *up = nullptr, *logits = nullptr, *scores = nullptr;
  int8_t* aq = nullptr;
  float* ad = nullptr;
  int* asum = nullptr;
  int8_t* aq_tc = nullptr;  // tensor-core activation layout (pb_kernels.cuh Batch)
  int tc_seqs = 0;
  int *d_slots = nullptr, *d_positions = nullptr;
  uint32_t* d_tokens = nullptr;
  unsigned long long* d_err = nullptr;      // [kErrSteps][max_seqs]
  uint32_t *d_greedy = nullptr, *d_greedy_bits = nullptr;
  unsigned long long* d_states = nullptr;   // [max_seqs][2]
  uint64_t* d_hist_offset = nullptr;
  uint32_t* d_hist_len = nullptr;
  pb::SamplerRow* d_sampled = nullptr;
  unsigned long long* d_samp_status = nullptr;  // [kErrSteps][max_seqs]
  uint32_t* d_token_log = nullptr;              // [kErrSteps][max_seqs]
  unsigned int* d_tc_status = nullptr;          // tensor-core pipeline timeout flag
  unsigned int* h_tc_status = nullptr;
  int* d_base = nullptr;                        // [max_seqs] positions at the chunk's start
  unsigned long long* d_cand = nullptr;         // split sampler's per-part top-20 lists
  unsigned long long* d_err_cur = nullptr;      // [max_seqs] this step's stage errors

  // CUDA graphs of whole steps.  A step's launches depend on the host only
  // through the key below (the softmax span is rounded up to 64 positions for
  // this: wider shared-memory tiles, the same results), so a step whose key was
  // seen before replays its graph.  The first occurrence of a key runs
  // directly (kernel attributes are set there), the second is captured.
  struct GraphKey {
    uint32_t rows;
    int span;
    int kind;  // 0 decode forward, 1 generate step (its greedy argmax runs outside the graph)
    bool operator==(const GraphKey& o) const {
      return rows == o.rows && span == o.span && kind == o.kind;
    }
  };
  struct GraphEntry {
    GraphKey key;
    cudaGraphExec_t exec = nullptr;  // null: seen once, not captured yet
    uint64_t launches = 0;
    uint64_t used = 0;
  };
  std::vector<GraphEntry> graphs;
  uint64_t graph_clock = 0;
  bool graphs_enabled = true;
  static constexpr size_t kMaxGraphs = 16;
  // Steps of up to this many rows replay graphs: measured +1% per step at 256
  // rows, +3% at 128 and more below; a key's capture (~ms) falls into the
  // second step of each span bucket, once per 128 positions.
  static constexpr uint32_t kGraphMaxRows = 256;
  // Graphs of steps of at most this many rows are captured without
  // programmatic dependent launch: measured 3-12% faster per step at 1-32 rows
  // (and 4.7% slower at 64), while PDL pays in stream-launched steps.
  static constexpr uint32_t kGraphNoPdlRows = 32;
  // Span bucket of the graph key: one capture per kGraphSpanBucket positions.
  static constexpr int kGraphSpanBucket = 128;

  // pinned host staging
  int *h_slots = nullptr, *h_positions = nullptr;
  uint32_t* h_tokens = nullptr;
  unsigned long long* h_err = nullptr;
  uint32_t *h_greedy = nullptr, *h_greedy_bits = nullptr;

  uint32_t last_rows = 0;  // rows of the last forward (logits rows valid)
  int max_span = 4;        // largest softmax span of the step being enqueued
  static constexpr uint32_t kErrSteps = 256;

  // Launch accounting and optional per-class CUDA-event timing on `stream`.
  uint64_t launches = 0;
  uint32_t prof_mask = 0;
  std::vector<cudaEvent_t> prof_events;
  std::vector<int> prof_class;
  size_t prof_used = 0;
  double prof_ms[16] = {};
  uint64_t prof_count[16] = {};

  void prof_mark(int cls) {
    if (!((prof_mask >> cls) & 1u)) return;
    if (prof_used == prof_events.size()) {
      cudaEvent_t ev;
      if (cudaEventCreate(&ev) != cudaSuccess) return;
      prof_events.push_back(ev);
      prof_class.push_back(cls);
    }
    prof_class[prof_used] = cls;
    cudaEventRecord(prof_events[prof_used++], stream);
  }
  // Accumulates the elapsed time of every recorded (begin, end) pair; call after
  // the stream is synchronized.
  void prof_resolve() {
    for (size_t i = 0; i + 1 < prof_used; i += 2) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, prof_events[i], prof_events[i + 1]) == cudaSuccess) {
        prof_ms[prof_class[i]] += ms;
        prof_count[prof_class[i]] += 1;
      }
    }
    prof_used = 0;
  }

  size_t scratch_bytes_per_slot() const {
    return (size_t)(896 * 4 + 4864 + 152 * 8 + 896 * 4 + 256 * 4 + 896 * 4 + 4864 * 8 +
                    151936 * 4) + (size_t)14 * (capacity + 4) * 4;
  }

#define PB_LAUNCH(cls, call) \
  do {                       \
    prof_mark(cls);          \
    call;                    \
    prof_mark(cls);          \
    ++launches;              \
  } while (0)
// For a launcher that returns how many kernels it launched.
#define PB_LAUNCH_N(cls, call) \
  do {                         \
    prof_mark(cls);            \
    launches += (call);        \
    prof_mark(cls);            \
  } while (0)

  pb::Batch batch(uint32_t rows, unsigned long long* err) const {
    pb::Batch b;
    b.rows = (int)rows; b.slots = d_slots; b.positions = d_positions; b.tokens = d_tokens;
    b.hidden = hidden; b.aq = aq; b.ad = ad; b.asum = asum; b.q = q; b.k = k; b.v = v;
    b.attn = attn; b.gate = gate; b.up = up; b.logits = logits; b.scores = scores;
    b.score_stride = capacity + 4; b.kv = kv; b.capacity = capacity; b.history = history;
    b.err = err;
    b.kv_checked = true;
    if ((int)rows >= pb::kTcMinBatch) {
      b.aq_tc = aq_tc; b.tc_seqs = tc_seqs;
    }
    return b;
  }

  // One matvec over the batch: the tensor-core path (tile image, up to three
  // stacked matrices in one launch) from kTcMinBatch rows, else one CUDA-core
  // matvec launch per matrix.
  struct Mat {
    const uint8_t* w;
    int rows;
    pb::Epilogue ep;
  };
  // The RMSNorm + Q8_0 stage that produces a matvec's input (weight, layer
  // ordinal, stage domain).
  struct Norm {
    const float* w = nullptr;
    uint32_t ord = 0, domain = 0;
  };
  void norm_launch(const pb::Batch& b, const Norm& n) {
    PB_LAUNCH(PB_KC_NORM, pb::launch_rmsnorm_quant(b, n.w, n.ord, n.domain, stream));
  }

  // With `norm` given, the matvec's input is that stage of Batch::hidden: fused
  // into the small-batch matvec's prologue, else a separate launch first.
  void matvec(int wtype, const pb::Batch& b, int columns, const uint8_t* tc_image,
              std::initializer_list<Mat> mats, int cls, int rt = 32, const Norm* norm = nullptr) {
    using namespace pb;
    if (!b.aq_tc) {
      SmallGemv g{};
      g.wtype = wtype; g.cols = columns; g.rt = rt;
      int rows = 0;
      for (const Mat& m : mats) {
        rows += m.rows;
        g.seg[g.nseg].w = m.w;
        g.seg[g.nseg].rows_end = rows;
        g.seg[g.nseg].ep = m.ep;
        ++g.nseg;
      }
      if (norm) {
        g.norm_weight = norm->w;
        g.norm_ordinal = norm->ord;
        g.norm_domain = norm->domain;
      }
      if (small_gemv_supported(g, b.rows)) {
        PB_LAUNCH(cls, launch_small_gemv(g, b, d_tc_status, stream));
        return;
      }
    }
    if (norm) norm_launch(b, *norm);
    if (b.aq_tc) {
      TcGemm g{};
      g.wtype = wtype; g.tiles = tc_image; g.nb = columns / 32;
      int rt = 0;
      for (const Mat& m : mats) {
        rt += m.rows / 128;
        g.seg[g.nseg].rtile_end = rt;
        g.seg[g.nseg].ep = m.ep;
        ++g.nseg;
      }
      g.rtiles = rt;
      PB_LAUNCH(cls, launch_tc_gemm(g, b, d_tc_status, stream));
    } else {
      for (const Mat& m : mats) PB_LAUNCH(cls, launch_qgemv(wtype, m.w, m.rows, columns, b, m.ep, stream));
    }
  }

  // The sampler over the first n logits rows (history of row i: the slot's
  // first hist_len[i] tokens); few rows split every row over several CTAs.
  // Returns the launches made.
  int sample_rows(uint32_t n, const uint32_t* hist_len) {
    if (n <= (uint32_t)pb::kSplitSamplerMaxRows) {
      pb::launch_sampler_split(logits, 151936, (int)n, 151936, history, d_hist_offset, hist_len,
                               nullptr, d_states, d_sampled, d_cand, stream);
      return 2;
    }
    pb::launch_sampler(logits, 151936, (int)n, 151936, history, d_hist_offset, hist_len, nullptr,
                       d_states, d_sampled, stream);
    return 1;
  }

  // Runs `enqueue` (the launches of one step) directly or as a CUDA graph
  // keyed by `key`; returns false when a CUDA call failed.
  template <class F>
  bool run_step(const GraphKey& key, F&& enqueue) {
    if (!graphs_enabled || prof_mask || key.rows > kGraphMaxRows) {
      enqueue();
      return true;
    }
    GraphEntry* entry = nullptr;
    for (GraphEntry& g : graphs)
      if (g.key == key) entry = &g;
    if (!entry) {
      if (graphs.size() == kMaxGraphs) {
        auto oldest = std::min_element(graphs.begin(), graphs.end(),
                                       [](const GraphEntry& a, const GraphEntry& b) {
                                         return a.used < b.used;
                                       });
        if (oldest->exec) cudaGraphExecDestroy(oldest->exec);
        graphs.erase(oldest);
      }
      graphs.push_back(GraphEntry{key});
      graphs.back().used = ++graph_clock;
      enqueue();  // first occurrence: direct
      return true;
    }
    entry->used = ++graph_clock;
    if (!entry->exec) {
      const uint64_t l0 = launches;
      if (cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        graphs_enabled = false;
        enqueue();
        return true;
      }
      {
        pb::PdlOff off(key.rows <= kGraphNoPdlRows);
        enqueue();
      }
      cudaGraph_t graph = nullptr;
      cudaError_t e = cudaStreamEndCapture(stream, &graph);
      if (e == cudaSuccess) e = cudaGraphInstantiate(&entry->exec, graph, 0);
      if (graph) cudaGraphDestroy(graph);
      entry->launches = launches - l0;
      launches = l0;
      if (e != cudaSuccess) {
        // not capturable here: run without graphs from now on
        cudaGetLastError();
        entry->exec = nullptr;
        graphs_enabled = false;
        enqueue();
        return true;
      }
    }
    launches += entry->launches;
    return cudaGraphLaunch(entry->exec, stream) == cudaSuccess;
  }

  // The softmax span rounded up for the graph key.  The kernels bound their
  // work by each row's own position, and the attention path is chosen from
  // (rows, rounded span), so every replay of a key takes the same launches.
  int graph_span(int span, uint32_t rows) const {
    return graphs_enabled && rows <= kGraphMaxRows
               ? (span + kGraphSpanBucket - 1) / kGraphSpanBucket * kGraphSpanBucket
               : span;
  }

  // Small batches: gate and up rows of one 32-row block per CTA, SwiGLU and the
  // Q8_0 quantization of the products fused into the matvec.
  bool gateup_swiglu(const pb::Batch& b, const uint8_t* gate_w, const uint8_t* up_w,
                     const pb::Epilogue& eg, const pb::Epilogue& eu, uint32_t ord,
                     const Norm& norm) {
    using namespace pb;
    SmallGemv g{};
    g.wtype = W_Q4_0; g.cols = kHidden; g.rt = 32; g.nseg = 2;
    g.seg[0] = {gate_w, kFfn, eg};
    g.seg[1] = {up_w, kFfn, eu};
    g.swiglu = 1;
    g.swiglu_ordinal = ord;
    g.norm_weight = norm.w;
    g.norm_ordinal = norm.ord;
    g.norm_domain = norm.domain;
    if (!small_gemv_supported(g, b.rows)) return false;
    PB_LAUNCH(PB_KC_GEMV, launch_small_gemv(g, b, d_tc_status, stream));
    return true;
  }

  // Enqueues one forward step for rows already staged in d_slots/d_positions/
  // d_tokens; stage failures land in err[0..rows).
  // distinct_slots: no two rows share a slot (decode); RoPE and the KV write
  // then run inside the attention launch.
  void enqueue_forward(uint32_t rows, bool want_logits, unsigned long long* err,
                       bool want_greedy = true, bool distinct_slots = true) {
    using namespace pb;
    const pb_model* m = model;
    Batch b = batch(rows, err);
    cudaMemsetAsync(err, 0xff, rows * sizeof(unsigned long long), stream);
    PB_LAUNCH(PB_KC_EMBED, launch_embed(b, m->tensor(0), stream));
    for (int layer = 0; layer < kLayers; ++layer) {
      const uint32_t ord = layer + 1;
      auto T = [&](uint32_t role) { return m->tensor(layer_tensor(layer, role)); };
      const Norm attn_norm{reinterpret_cast<const float*>(T(10)), ord, D_ATTN_NORM};
      const Epilogue eq{EPI_BIAS, q, kHidden, reinterpret_cast<const float*>(T(18)), err, ord, D_Q};
      const Epilogue ek{EPI_BIAS, k, 128, reinterpret_cast<const float*>(T(15)), err, ord, D_K};
      const Epilogue ev{EPI_BIAS, v, 128, reinterpret_cast<const float*>(T(20)), err, ord, D_V};
      matvec(W_Q4_0, b, 896, m->tc + m->tc_qkv[layer],
             {{T(19), 896, eq}, {T(16), 128, ek}, {T(21), 128, ev}}, PB_KC_GEMV, 32, &attn_norm);
      if (distinct_slots) {
        PB_LAUNCH_N(PB_KC_ATTENTION, launch_attention(b, layer, max_span, true, m->rope, stream));
      } else {
        PB_LAUNCH(PB_KC_ROPE_KV, launch_rope_kv(b, layer, m->rope, stream));
        PB_LAUNCH_N(PB_KC_ATTENTION, launch_attention(b, layer, max_span, true, nullptr, stream));
      }
      const Epilogue eo{EPI_RESIDUAL, hidden, kHidden, nullptr, err, ord, D_ATTN_OUTPUT};
      matvec(W_Q4_0, b, 896, m->tc + m->tc_o[layer], {{T(17), 896, eo}}, PB_KC_GEMV, 8);
      const Norm ffn_norm{reinterpret_cast<const float*>(T(14)), ord, D_FFN_NORM};
      const Epilogue eg{EPI_STORE, gate, kFfn, nullptr, err, ord, D_GATE};
      const Epilogue eu{EPI_STORE, up, kFfn, nullptr, err, ord, D_UP};
      if (!b.aq_tc && gateup_swiglu(b, T(12), T(13), eg, eu, ord, ffn_norm)) {
        // RMSNorm, gate/up, SwiGLU and its quantization in one small-batch launch
      } else {
        matvec(W_Q4_0, b, 896, m->tc + m->tc_gateup[layer], {{T(12), 4864, eg}, {T(13), 4864, eu}},
               PB_KC_GEMV, 32, &ffn_norm);
        PB_LAUNCH(PB_KC_SWIGLU, launch_swiglu_quant(b, ord, stream));
      }
      const Epilogue ed{EPI_RESIDUAL, hidden, kHidden, nullptr, err, ord, D_DOWN};
      matvec(W_Q4_0, b, 4864, m->tc + m->tc_down[layer], {{T(11), 896, ed}}, PB_KC_GEMV, 8);
    }
    if (want_logits) {
      PB_LAUNCH(PB_KC_NORM, launch_rmsnorm_quant(b, reinterpret_cast<const float*>(m->tensor(289)),
                                                 25, D_OUTPUT_NORM, stream));
      const Epilogue el{EPI_STORE, logits, (size_t)kVocab, nullptr, err, 25, D_LOGITS};
      matvec(W_Q8_0, b, 896, m->tc + m->tc_head, {{m->tensor(290), kVocab, el}}, PB_KC_LM_HEAD);
      if (want_greedy)
        PB_LAUNCH(PB_KC_ARGMAX, launch_argmax(logits, kVocab, rows, kVocab, d_greedy, d_greedy_bits,
                                              nullptr, stream));
    }
  }

  // One synchronous step over explicit rows; fills per-row stage errors (~0 = ok)
  // and, with logits, greedy ids/bits in h_greedy/h_greedy_bits.
  uint32_t step(uint32_t rows, const int* slot_ids, const uint32_t* toks, const int* pos,
                bool want_logits, bool distinct_slots = true) {
    std::copy(slot_ids, slot_ids + rows, h_slots);
    std::copy(toks, toks + rows, h_tokens);
    std::copy(pos, pos + rows, h_positions);
    PB_CUDA(cudaMemcpyAsync(d_slots, h_slots, rows * 4, cudaMemcpyHostToDevice, stream));
    PB_CUDA(cudaMemcpyAsync(d_tokens, h_tokens, rows * 4, cudaMemcpyHostToDevice, stream));
    PB_CUDA(cudaMemcpyAsync(d_positions, h_positions, rows * 4, cudaMemcpyHostToDevice, stream));
    max_span = 4;
    for (uint32_t i = 0; i < rows; ++i) max_span = std::max(max_span, (pos[i] + 4) & ~3);
    if (distinct_slots && want_logits) {
      max_span = graph_span(max_span, rows);
      if (!run_step(GraphKey{rows, max_span, 0},
                    [&] { enqueue_forward(rows, true, d_err, true, true); }))
        PB_CUDA(cudaGetLastError());
    } else {
      enqueue_forward(rows, want_logits, d_err, true, distinct_slots);
    }
    PB_CUDA(cudaGetLastError());
    PB_CUDA(cudaMemcpyAsync(h_err, d_err, rows * 8, cudaMemcpyDeviceToHost, stream));
    PB_CUDA(cudaMemcpyAsync(h_tc_status, d_tc_status, 4, cudaMemcpyDeviceToHost, stream));
    if (want_logits) {
      PB_CUDA(cudaMemcpyAsync(h_greedy, d_greedy, rows * 4, cudaMemcpyDeviceToHost, stream));
      PB_CUDA(cudaMemcpyAsync(h_greedy_bits, d_greedy_bits, rows * 4, cudaMemcpyDeviceToHost, stream));
      last_rows = rows;
    }
    PB_CUDA(cudaStreamSynchronize(stream));
    prof_resolve();
    return check_tc_status();
  }

  // A tensor-core pipeline wait that timed out (never expected) poisons the
  // engine's results: report it as a device failure.
  uint32_t check_tc_status() {
    if (*h_tc_status) {
      pb::set_last_error("tensor-core matvec pipeline timed out waiting for an MMA");
      return PB_DEVICE;
    }
    return PB_OK;
  }

  uint64_t kv_bytes_per_slot() const { return (uint64_t)capacity * 24576ull; }

  pb_error state_error(const Slot& s, uint32_t needed, uint32_t sub) const {
    return make_error(PB_STATE, DOM_PROMPT, NO_LAYER, s.position, NO_TENSOR, needed, s.state,
                      K_STATE, sub);
  }

  void reset_state(Slot& s) {
    s.position = 0; s.reserve = 0; s.emitted = 0; s.last_selected = 0;
    s.state = PB_STATE_RESET; s.prefix.clear();
  }

  // inference.rs:1938-1944
  pb_error fault(Slot& s, const pb_error& e, uint32_t* host_logits) {
    if (host_logits) std::fill(host_logits, host_logits + kVocabWords, 0u);
    s.state = PB_STATE_FAULTED;
    s.prefix.clear();
    return e;
  }
  static constexpr uint32_t kVocabWords = 151936;

  // inference.rs:1387-1411 (after a successful evaluate of row `row`)
  pb_step publish(Slot& s, uint32_t row) {
    uint32_t selected = h_greedy[row];
    s.last_selected = selected;
    uint32_t eos = selected == (uint32_t)pb::kEos;
    s.state = eos ? PB_STATE_EOS : PB_STATE_READY;
    pb_step st{s.position, selected, h_greedy_bits[row], eos};
    return st;
  }

  void advance(Slot& s) {
    s.position += 1;
    s.kv_high_water = std::max<uint64_t>(s.kv_high_water, (uint64_t)s.position * 24576ull);
    s.scratch_high_water = scratch_bytes_per_slot();
  }

  // Validation of inference.rs:1109-1191 (prefill_inner prechecks).
  bool prefill_checks(const Slot& s, const uint32_t* tokens, uint32_t n, uint32_t reserve,
                      bool append, pb_error* err) const {
    const uint32_t start = s.position;
    if (reserve < 1 || reserve > context_limit) {
      *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, start, NO_TENSOR,
                        reserve == 0 ? 1 : context_limit, reserve, K_RESERVE, 0);
      return false;
    }
    if (n == 0) {
      *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, start, NO_TENSOR, 1, 0, K_CONTEXT, 0);
      return false;
    }
    if (!append && n >= context_limit) {
      *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, 0, NO_TENSOR, context_limit - 1, n,
                        K_CONTEXT, 0);
      return false;
    }
    uint64_t total = (uint64_t)start + n + reserve;
    if (total > context_limit) {
      *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, start, NO_TENSOR, context_limit, total,
                        K_CONTEXT, 1);
      return false;
    }
    for (uint32_t i = 0; i < n; ++i)
      if (tokens[i] >= kVocabWords) {
        *err = make_error(PB_TOKEN_ID, DOM_PROMPT, NO_LAYER, start + i, NO_TENSOR, kVocabWords,
                          tokens[i], K_TOKEN, 0);
        return false;
      }
    return true;
  }

  // Lockstep prefill of `len` tokens for each of `n` slots (all already
  // validated); per-slot failures fault only that slot.
  uint32_t run_prefill(uint32_t n, const uint32_t* seq_ids, const uint32_t* tokens, uint32_t len,
                       uint32_t reserve, uint32_t* host_logits, pb_step* steps, pb_error* errs,
                       const char* active_in) {
    std::vector<char> active(n);
    for (uint32_t i = 0; i < n; ++i) {
      active[i] = active_in ? active_in[i] : 1;
      if (active[i]) {
        Slot& s = slots[seq_ids[i]];
        s.reserve = reserve;
        s.emitted = 0;
      }
    }
    std::vector<int> rs, ps;
    std::vector<uint32_t> ts, map, tmap;
    uint32_t first_status = PB_OK;
    // Every prompt position but the last runs batched: rows are (sequence,
    // position) pairs, position-major, up to rows_cap per forward.  Each row
    // evaluates exactly the reference's per-token arithmetic (rows are
    // independent; attention reads the slot's KV of positions <= its own, all
    // written by this or an earlier forward).  A row's stage failure faults its
    // sequence at the earliest failing position (rows of a sequence appear in
    // increasing position order); later rows of that sequence are discarded.
    std::vector<uint32_t> base(n);
    for (uint32_t i = 0; i < n; ++i) base[i] = slots[seq_ids[i]].position;
    const uint32_t batched = len > 0 ? len - 1 : 0;
    for (uint32_t t_cur = 0, i_cur = 0; t_cur < batched;) {
      rs.clear(); ps.clear(); ts.clear(); map.clear(); tmap.clear();
      while (t_cur < batched && rs.size() < rows_cap) {
        if (active[i_cur]) {
          rs.push_back((int)seq_ids[i_cur]);
          ps.push_back((int)(base[i_cur] + t_cur));
          ts.push_back(tokens[(size_t)i_cur * len + t_cur]);
          map.push_back(i_cur);
          tmap.push_back(t_cur);
        }
        if (++i_cur == n) { i_cur = 0; ++t_cur; }
      }
      if (rs.empty()) break;
      // rows of one sequence at several positions: the KV writes of all rows
      // must land before any row's attention (separate RoPE/KV launch)
      uint32_t st = step((uint32_t)rs.size(), rs.data(), ts.data(), ps.data(), false, false);
      if (st) return st;
      for (size_t r = 0; r < rs.size(); ++r) {
        const uint32_t i = map[r];
        if (!active[i] || h_err[r] == pb::kNoError) continue;
        Slot& s = slots[seq_ids[i]];
        while (s.position < base[i] + tmap[r]) advance(s);
        errs[i] = fault(s, stage_error(h_err[r], s.position), n == 1 ? host_logits : nullptr);
        active[i] = 0;
        if (!first_status) first_status = errs[i].status;
      }
    }
    for (uint32_t i = 0; i < n; ++i) {
      if (!active[i]) continue;
      Slot& s = slots[seq_ids[i]];
      while (s.position < base[i] + batched) advance(s);
    }
    // The last prompt position of every sequence: one forward with logits.
    for (uint32_t t = batched; t < len; ++t) {
      rs.clear(); ps.clear(); ts.clear(); map.clear();
      for (uint32_t i = 0; i < n; ++i) {
        if (!active[i]) continue;
        rs.push_back((int)seq_ids[i]);
        ps.push_back((int)slots[seq_ids[i]].position);
        ts.push_back(tokens[(size_t)i * len + t]);
        map.push_back(i);
      }
      if (rs.empty()) break;
      const bool last = t + 1 == len;
      uint32_t st = step((uint32_t)rs.size(), rs.data(), ts.data(), ps.data(), last);
      if (st) return st;
      for (size_t r = 0; r < rs.size(); ++r) {
        uint32_t i = map[r];
        Slot& s = slots[seq_ids[i]];
        if (h_err[r] != pb::kNoError) {
          errs[i] = fault(s, stage_error(h_err[r], s.position), n == 1 ? host_logits : nullptr);
          active[i] = 0;
          if (!first_status) first_status = errs[i].status;
          continue;
        }
        advance(s);
        if (last) {
          s.emitted = 1;
          steps[i] = publish(s, (uint32_t)r);
          if (n == 1 && host_logits) {
            PB_CUDA(cudaMemcpyAsync(host_logits, logits + (size_t)r * kVocabWords, kVocabWords * 4,
                                    cudaMemcpyDeviceToHost, stream));
            PB_CUDA(cudaStreamSynchronize(stream));
          }
        }
      }
    }
    return first_status;
  }

  bool decode_checks(const Slot& s, uint32_t token, bool require_greedy, pb_error* err) const {
    switch (s.state) {
      case PB_STATE_FAULTED: *err = state_error(s, PB_STATE_RESET, 3); return false;
      case PB_STATE_EOS:
        if (require_greedy) { *err = state_error(s, PB_STATE_READY, 2); return false; }
        break;
      case PB_STATE_RESET: *err = state_error(s, PB_STATE_READY, 0); return false;
      default: break;
    }
    if (token >= kVocabWords) {
      *err = make_error(PB_TOKEN_ID, DOM_PROMPT, NO_LAYER, s.position, NO_TENSOR, kVocabWords,
                        token, K_TOKEN, 1);
      return false;
    }
    if (require_greedy && token != s.last_selected) {
      *err = make_error(PB_STATE, DOM_ARGMAX, NO_LAYER, s.position, NO_TENSOR, s.last_selected,
                        token, K_SELECTED, 0);
      return false;
    }
    if (s.emitted >= s.reserve) {
      *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, s.position, NO_TENSOR, s.reserve,
                        s.emitted, K_RESERVE, 1);
      return false;
    }
    if (s.position >= context_limit) {
      *err = make_error(PB_CONTEXT, DOM_KV, NO_LAYER, s.position, NO_TENSOR, context_limit,
                        s.position, K_CONTEXT, 2);
      return false;
    }
    return true;
  }
};

namespace {

bool seq_ok(const pb_engine* e, uint32_t seq) { return e && seq < e->max_seqs; }

// The batched entry points evaluate one row per listed sequence; a sequence
// listed twice would have two rows write the same KV position.
bool distinct_seqs(const pb_engine* e, uint32_t n, const uint32_t* seqs) {
  std::vector<char> seen(e->max_seqs, 0);
  for (uint32_t i = 0; i < n; ++i) {
    if (seqs[i] >= e->max_seqs) continue;  // reported per sequence by the caller
    if (seen[seqs[i]]) return false;
    seen[seqs[i]] = 1;
  }
  return true;
}

pb_error bad_seq(uint32_t seq, uint32_t max) {
  return make_error(PB_CAPACITY, DOM_PROMPT, NO_LAYER, 0, NO_TENSOR, max, seq, K_STATE, 7);
}

}  // namespace

extern "C" {

uint32_t pb_engine_create(pb_model* model, uint32_t max_seqs, uint32_t max_context,
                          pb_engine** out, pb_error* err) {
  if (out) *out = nullptr;
  if (!model || !out || max_seqs == 0 || max_context == 0 || max_context > PB_CONTEXT_LIMIT ||
      (max_context & 3)) {
    if (err) *err = make_error(PB_CAPACITY, 1, NO_LAYER, 0, NO_TENSOR, PB_CONTEXT_LIMIT,
                               max_context, K_BYTES, 0);
    return PB_CAPACITY;
  }
  pb_engine* e = new pb_engine();
  e->model = model;
  e->device = model->device;
  e->max_seqs = max_seqs;
  e->capacity = max_context;
  e->context_limit = std::min<uint32_t>(PB_CONTEXT_LIMIT, max_context);
  e->slots.resize(max_seqs);
  const size_t S = max_seqs;
  e->rows_cap = std::max<uint32_t>(max_seqs, pb_engine::kPrefillRows);
  const size_t R = e->rows_cap;
  cudaError_t c = cudaSetDevice(e->device);
  auto chk = [&](cudaError_t r) { if (c == cudaSuccess) c = r; };
  chk(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  chk(dalloc(&e->kv, S * (size_t)max_context * 6144));
  chk(dalloc(&e->history, S * (size_t)max_context));
  chk(dalloc(&e->hidden, R * 896));
  chk(dalloc(&e->q, R * 896));
  chk(dalloc(&e->k, R * 128));
  chk(dalloc(&e->v, R * 128));
  chk(dalloc(&e->attn, R * 896));
  chk(dalloc(&e->gate, R * 4864));
  chk(dalloc(&e->up, R * 4864));
  chk(dalloc(&e->logits, S * 151936));
  chk(dalloc(&e->scores, R * 14 * ((size_t)max_context + 4)));
  chk(dalloc(&e->aq, R * 4864));
  chk(dalloc(&e->ad, R * 152));
  chk(dalloc(&e->asum, R * 152));
  e->tc_seqs = (int)((R + 63) / 64 * 64);
  chk(dalloc(&e->aq_tc, pb::tc_act_bytes(e->tc_seqs, 4864)));
  chk(dalloc(&e->d_slots, R));
  chk(dalloc(&e->d_positions, R));
  chk(dalloc(&e->d_tokens, R));
  chk(dalloc(&e->d_err, std::max(R, S * pb_engine::kErrSteps)));
  chk(dalloc(&e->d_greedy, S));
  chk(dalloc(&e->d_greedy_bits, S));
  chk(dalloc(&e->d_states, S * 2));
  chk(dalloc(&e->d_hist_offset, S));
  chk(dalloc(&e->d_hist_len, S));
  chk(dalloc(&e->d_sampled, S));
  chk(dalloc(&e->d_samp_status, S * pb_engine::kErrSteps));
  chk(dalloc(&e->d_token_log, S * pb_engine::kErrSteps));
  chk(dalloc(&e->d_tc_status, 1));
  chk(dalloc(&e->d_base, S));
  chk(dalloc(&e->d_cand, pb::split_sampler_words(std::min<int>((int)S, pb::kSplitSamplerMaxRows))));
  chk(dalloc(&e->d_err_cur, R));
  chk(cudaMallocHost(&e->h_tc_status, 4));
  chk(cudaMallocHost(&e->h_slots, R * 4));
  chk(cudaMallocHost(&e->h_positions, R * 4));
  chk(cudaMallocHost(&e->h_tokens, R * 4));
  chk(cudaMallocHost(&e->h_err, 8 * std::max(R, S * pb_engine::kErrSteps)));
  chk(cudaMallocHost(&e->h_greedy, S * 4));
  chk(cudaMallocHost(&e->h_greedy_bits, S * 4));
  if (c == cudaSuccess) pb::init_kernel_attributes();
  if (const char* f = std::getenv("PB_GRAPHS")) e->graphs_enabled = std::atoi(f) != 0;
  if (c == cudaSuccess) c = cudaMemsetAsync(e->kv, 0, S * (size_t)max_context * 6144 * 4, e->stream);
  if (c == cudaSuccess) c = cudaMemsetAsync(e->history, 0, S * (size_t)max_context * 4, e->stream);
  if (c == cudaSuccess) c = cudaMemsetAsync(e->d_tc_status, 0, 4, e->stream);
  if (c == cudaSuccess) c = cudaMemsetAsync(e->aq_tc, 0, pb::tc_act_bytes(e->tc_seqs, 4864), e->stream);
  if (c == cudaSuccess) c = cudaStreamSynchronize(e->stream);
  if (c == cudaSuccess) *e->h_tc_status = 0;
  if (c != cudaSuccess) {
    pb::record_cuda_error(c, "pb_engine_create");
    if (err) *err = make_error(PB_DEVICE, 1, NO_LAYER, 0, NO_TENSOR, 0, (uint64_t)c, K_BYTES, 1);
    pb_engine_destroy(e);
    return PB_DEVICE;
  }
  *out = e;
  return PB_OK;
}

void pb_engine_destroy(pb_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  void* dev[] = {e->kv, e->history, e->hidden, e->q, e->k, e->v, e->attn, e->gate, e->up,
                 e->logits, e->scores, e->aq, e->ad, e->asum, e->d_slots, e->d_positions,
                 e->d_tokens, e->d_err, e->d_greedy, e->d_greedy_bits, e->d_states,
                 e->d_hist_offset, e->d_hist_len, e->d_sampled, e->d_samp_status,
                 e->d_token_log, e->d_tc_status, e->aq_tc, e->d_base, e->d_err_cur, e->d_cand};
  for (void* p : dev) if (p) cudaFree(p);
  void* host[] = {e->h_slots, e->h_positions, e->h_tokens, e->h_err, e->h_greedy, e->h_greedy_bits,
                  e->h_tc_status};
  for (void* p : host) if (p) cudaFreeHost(p);
  for (cudaEvent_t ev : e->prof_events) cudaEventDestroy(ev);
  for (auto& g : e->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

static uint32_t prefill_common(pb_engine* e, uint32_t seq, const uint32_t* tokens, uint32_t n,
                               uint32_t reserve, uint32_t* logits, pb_step* step, pb_error* err,
                               bool append) {
  Slot& s = e->slots[seq];
  pb_error local;
  pb_error* er = err ? err : &local;
  if (!e->prefill_checks(s, tokens, n, reserve, append, er)) return er->status;
  cudaSetDevice(e->device);
  pb_step st{};
  uint32_t status = e->run_prefill(1, &seq, tokens, n, reserve, logits, &st, er, nullptr);
  if (status == PB_OK && step) *step = st;
  return status;
}

uint32_t pb_engine_prefill(pb_engine* e, uint32_t seq, const uint32_t* tokens, uint32_t n,
                           uint32_t reserve, uint32_t* logits, pb_step* step, pb_error* err) {
  if (!seq_ok(e, seq)) { if (err) *err = bad_seq(seq, e ? e->max_seqs : 0); return PB_CAPACITY; }
  Slot& s = e->slots[seq];
  if (s.state == PB_STATE_FAULTED) { if (err) *err = e->state_error(s, PB_STATE_RESET, 3); return PB_STATE; }
  if (s.state != PB_STATE_RESET) { if (err) *err = e->state_error(s, PB_STATE_RESET, 1); return PB_STATE; }
  return prefill_common(e, seq, tokens, n, reserve, logits, step, err, false);
}

uint32_t pb_engine_prefill_with_prefix(pb_engine* e, uint32_t seq, const uint32_t* tokens,
                                       uint32_t n, uint32_t prefix_tokens, uint32_t reserve,
                                       uint32_t* logits, pb_step* step, pb_error* err) {
  if (!seq_ok(e, seq)) { if (err) *err = bad_seq(seq, e ? e->max_seqs : 0); return PB_CAPACITY; }
  Slot& s = e->slots[seq];
  const uint32_t prefix = prefix_tokens;
  if (prefix == 0 || prefix >= n || prefix > kMaxPrefix) {
    e->reset_state(s);
    if (err) *err = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, 0, NO_TENSOR, 1, prefix_tokens,
                               K_CONTEXT, 3);
    return PB_CONTEXT;
  }
  if (!s.prefix.empty()) {
    if (s.state == PB_STATE_RESET && s.position == s.prefix.size() && s.prefix.size() == prefix &&
        std::equal(s.prefix.begin(), s.prefix.end(), tokens))
      return prefill_common(e, seq, tokens + prefix, n - prefix, reserve, logits, step, err, true);
    if (s.state != PB_STATE_RESET) {
      pb_error er = e->state_error(s, PB_STATE_RESET, 4);
      e->reset_state(s);
      if (err) *err = er;
      return er.status;
    }
    e->reset_state(s);
  }
  uint32_t status = pb_engine_prefill(e, seq, tokens, n, reserve, logits, step, err);
  if (status == PB_OK) s.prefix.assign(tokens, tokens + prefix);
  return status;
}

uint32_t pb_engine_append_prefill(pb_engine* e, uint32_t seq, const uint32_t* tokens, uint32_t n,
                                  uint32_t reserve, uint32_t* logits, pb_step* step,
                                  pb_error* err) {
  if (!seq_ok(e, seq)) { if (err) *err = bad_seq(seq, e ? e->max_seqs : 0); return PB_CAPACITY; }
  Slot& s = e->slots[seq];
  if (s.state == PB_STATE_FAULTED) { if (err) *err = e->state_error(s, PB_STATE_RESET, 3); return PB_STATE; }
  if (s.state == PB_STATE_RESET) { if (err) *err = e->state_error(s, PB_STATE_READY, 0); return PB_STATE; }
  return prefill_common(e, seq, tokens, n, reserve, logits, step, err, true);
}

uint32_t pb_engine_decode_batch(pb_engine* e, uint32_t n, const uint32_t* seqs,
                                const uint32_t* tokens, uint32_t require_greedy, pb_step* steps,
                                pb_error* errs) {
  if (!e || n == 0 || n > e->max_seqs) return PB_CAPACITY;
  if (!distinct_seqs(e, n, seqs)) return PB_CAPACITY;
  cudaSetDevice(e->device);
  std::vector<int> rs, ps;
  std::vector<uint32_t> ts, map;
  uint32_t first = PB_OK;
  for (uint32_t i = 0; i < n; ++i) {
    if (!seq_ok(e, seqs[i])) { errs[i] = bad_seq(seqs[i], e->max_seqs); first = first ? first : PB_CAPACITY; continue; }
    Slot& s = e->slots[seqs[i]];
    if (!e->decode_checks(s, tokens[i], require_greedy != 0, &errs[i])) {
      if (!first) first = errs[i].status;
      continue;
    }
    rs.push_back((int)seqs[i]);
    ps.push_back((int)s.position);
    ts.push_back(tokens[i]);
    map.push_back(i);
  }
  if (rs.empty()) return first;
  uint32_t st = e->step((uint32_t)rs.size(), rs.data(), ts.data(), ps.data(), true);
  if (st) return st;
  for (size_t r = 0; r < rs.size(); ++r) {
    uint32_t i = map[r];
    Slot& s = e->slots[seqs[i]];
    if (e->h_err[r] != pb::kNoError) {
      errs[i] = e->fault(s, stage_error(e->h_err[r], s.position), nullptr);
      if (!first) first = errs[i].status;
      continue;
    }
    e->advance(s);
    s.emitted += 1;
    steps[i] = e->publish(s, (uint32_t)r);
    std::memset(&errs[i], 0, sizeof(pb_error));
  }
  return first;
}

static uint32_t decode_one(pb_engine* e, uint32_t seq, uint32_t token, uint32_t* logits,
                           pb_step* step, pb_error* err, uint32_t greedy) {
  if (!seq_ok(e, seq)) { if (err) *err = bad_seq(seq, e ? e->max_seqs : 0); return PB_CAPACITY; }
  pb_step st{};
  pb_error er{};
  uint32_t status = pb_engine_decode_batch(e, 1, &seq, &token, greedy, &st, &er);
  if (status == PB_OK) {
    if (step) *step = st;
    if (logits) {
      PB_CUDA(cudaMemcpyAsync(logits, e->logits, 151936 * 4, cudaMemcpyDeviceToHost, e->stream));
      PB_CUDA(cudaStreamSynchronize(e->stream));
    }
  } else {
    if (err) *err = er;
    if (logits && er.status >= PB_NONFINITE_INPUT && e->slots[seq].state == PB_STATE_FAULTED)
      std::fill(logits, logits + 151936, 0u);
  }
  return status;
}

uint32_t pb_engine_decode(pb_engine* e, uint32_t seq, uint32_t token, uint32_t* logits,
                          pb_step* step, pb_error* err) {
  return decode_one(e, seq, token, logits, step, err, 1);
}

uint32_t pb_engine_decode_selected(pb_engine* e, uint32_t seq, uint32_t token, uint32_t* logits,
                                   pb_step* step, pb_error* err) {
  return decode_one(e, seq, token, logits, step, err, 0);
}

uint32_t pb_engine_prefill_batch(pb_engine* e, uint32_t n, const uint32_t* seqs,
                                 const uint32_t* tokens, uint32_t len, uint32_t reserve,
                                 pb_step* steps, pb_error* errs) {
  if (!e || n == 0 || n > e->max_seqs) return PB_CAPACITY;
  if (!distinct_seqs(e, n, seqs)) return PB_CAPACITY;
  cudaSetDevice(e->device);
  std::vector<char> active(n, 0);
  uint32_t first = PB_OK;
  for (uint32_t i = 0; i < n; ++i) {
    if (!seq_ok(e, seqs[i])) { errs[i] = bad_seq(seqs[i], e->max_seqs); first = first ? first : PB_CAPACITY; continue; }
    Slot& s = e->slots[seqs[i]];
    if (s.state == PB_STATE_FAULTED) { errs[i] = e->state_error(s, PB_STATE_RESET, 3); first = first ? first : PB_STATE; continue; }
    if (s.state != PB_STATE_RESET) { errs[i] = e->state_error(s, PB_STATE_RESET, 1); first = first ? first : PB_STATE; continue; }
    if (!e->prefill_checks(s, tokens + (size_t)i * len, len, reserve, false, &errs[i])) {
      first = first ? first : errs[i].status;
      continue;
    }
    active[i] = 1;
    std::memset(&errs[i], 0, sizeof(pb_error));
  }
  uint32_t st = e->run_prefill(n, seqs, tokens, len, reserve, nullptr, steps, errs, active.data());
  return first ? first : st;
}

uint32_t pb_engine_logits(pb_engine* e, uint32_t row, uint32_t* logits) {
  if (!e || !logits || row >= e->last_rows) return PB_CAPACITY;
  cudaSetDevice(e->device);
  PB_CUDA(cudaMemcpyAsync(logits, e->logits + (size_t)row * 151936, 151936 * 4,
                          cudaMemcpyDeviceToHost, e->stream));
  PB_CUDA(cudaStreamSynchronize(e->stream));
  return PB_OK;
}

uint32_t pb_engine_reset(pb_engine* e, uint32_t seq) {
  if (!seq_ok(e, seq)) return PB_CAPACITY;
  e->reset_state(e->slots[seq]);
  return PB_OK;
}

uint32_t pb_engine_reset_to_prefix(pb_engine* e, uint32_t seq, uint32_t* prefix_out) {
  if (!seq_ok(e, seq)) return PB_CAPACITY;
  Slot& s = e->slots[seq];
  const uint32_t prefix = (uint32_t)s.prefix.size();
  bool valid = false;
  switch (s.state) {
    case PB_STATE_RESET: valid = prefix != 0 && s.position == prefix; break;
    case PB_STATE_READY:
    case PB_STATE_EOS: valid = prefix != 0 && s.position >= prefix && s.position <= PB_CONTEXT_LIMIT; break;
    default: valid = false;
  }
  if (!valid) {
    e->reset_state(s);
    if (prefix_out) *prefix_out = 0;
    return PB_OK;
  }
  s.position = prefix; s.reserve = 0; s.emitted = 0; s.last_selected = 0; s.state = PB_STATE_RESET;
  if (prefix_out) *prefix_out = prefix;
  return PB_OK;
}

uint32_t pb_engine_usage(pb_engine* e, uint32_t seq, pb_usage* out) {
  if (!seq_ok(e, seq) || !out) return PB_CAPACITY;
  const Slot& s = e->slots[seq];
  const uint64_t mb = pb::kModelBytes;
  out->weights = {mb, mb, mb, mb, mb};
  const uint64_t kvb = e->kv_bytes_per_slot();
  out->kv = {kvb, kvb, kvb, (uint64_t)s.position * 24576ull, s.kv_high_water};
  const uint64_t sb = e->scratch_bytes_per_slot();
  out->scratch = {sb, sb, sb, 0, s.scratch_high_water};
  out->position = s.position;
  out->context_limit = e->context_limit;
  out->generation_reserve = s.reserve;
  out->state = s.state;
  return PB_OK;
}

uint32_t pb_engine_position(pb_engine* e, uint32_t seq) {
  return seq_ok(e, seq) ? e->slots[seq].position : 0;
}

void* pb_engine_kv_device(pb_engine* e, uint32_t seq, uint64_t* words) {
  if (!seq_ok(e, seq)) {
    if (words) *words = 0;
    return nullptr;
  }
  const uint64_t per_slot = (uint64_t)e->capacity * 6144ull;
  if (words) *words = per_slot;
  return e->kv + (size_t)seq * per_slot;
}

// A sequence whose KV of positions [0, n) the caller has written into the
// slot's region (pb_engine_kv_device): prefill's prechecks (inference.rs:
// 1109-1191) on the tokens and reserve, then the slot holds `tokens` as its
// history and is READY at position n with no greedy id (decode_selected is the
// next call; decode reports the reference's selected-token state error).
uint32_t pb_engine_restore(pb_engine* e, uint32_t seq, const uint32_t* tokens, uint32_t n,
                           uint32_t reserve, pb_error* err) {
  if (!seq_ok(e, seq)) { if (err) *err = bad_seq(seq, e ? e->max_seqs : 0); return PB_CAPACITY; }
  Slot& s = e->slots[seq];
  pb_error local;
  pb_error* er = err ? err : &local;
  if (s.state == PB_STATE_FAULTED) { *er = e->state_error(s, PB_STATE_RESET, 3); return PB_STATE; }
  if (s.state != PB_STATE_RESET) { *er = e->state_error(s, PB_STATE_RESET, 1); return PB_STATE; }
  if (!tokens && n) { *er = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, 0, NO_TENSOR, 1, 0, K_CONTEXT, 0); return PB_CONTEXT; }
  if (!e->prefill_checks(s, tokens, n, reserve, false, er)) return er->status;
  cudaSetDevice(e->device);
  PB_CUDA(cudaMemcpyAsync(e->history + (size_t)seq * e->capacity, tokens, (size_t)n * 4,
                          cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaStreamSynchronize(e->stream));
  s.position = n;
  s.kv_high_water = std::max<uint64_t>(s.kv_high_water, (uint64_t)n * 24576ull);
  s.scratch_high_water = e->scratch_bytes_per_slot();
  s.reserve = reserve;
  s.emitted = 0;
  s.last_selected = PB_VOCAB;  // no greedy id to continue from
  s.prefix.clear();
  s.state = PB_STATE_READY;
  return PB_OK;
}

static void sampler_error(pb_error* err, const pb::SamplerRow& r, uint64_t count) {
  if (r.status == 7)
    *err = make_error(PB_NONFINITE_OUTPUT, DOM_ARGMAX, NO_LAYER, 0, NO_TENSOR, 0, r.value,
                      K_FINITE, r.index);
  else
    *err = make_error(PB_TOKEN_ID, DOM_ARGMAX, NO_LAYER, 0, NO_TENSOR, count, r.value, K_TOKEN, 0);
}

uint32_t pb_engine_sample(pb_engine* e, uint32_t n, const uint32_t* seqs,
                          pb_sampling_state* states, uint32_t* ids, pb_error* errs) {
  if (!e || n == 0 || n > e->last_rows || !distinct_seqs(e, n, seqs)) return PB_CAPACITY;
  cudaSetDevice(e->device);
  std::vector<uint64_t> off(n);
  std::vector<uint32_t> len(n);
  for (uint32_t i = 0; i < n; ++i) {
    if (!seq_ok(e, seqs[i])) return PB_CAPACITY;
    off[i] = (uint64_t)seqs[i] * e->capacity;
    len[i] = e->slots[seqs[i]].position;
  }
  PB_CUDA(cudaMemcpyAsync(e->d_hist_offset, off.data(), n * 8, cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaMemcpyAsync(e->d_hist_len, len.data(), n * 4, cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaMemcpyAsync(e->d_states, states, n * 16, cudaMemcpyHostToDevice, e->stream));
  e->prof_mark(PB_KC_SAMPLER);
  e->launches += e->sample_rows(n, e->d_hist_len);
  e->prof_mark(PB_KC_SAMPLER);
  PB_CUDA(cudaGetLastError());
  std::vector<pb::SamplerRow> rows(n);
  PB_CUDA(cudaMemcpyAsync(rows.data(), e->d_sampled, n * sizeof(pb::SamplerRow),
                          cudaMemcpyDeviceToHost, e->stream));
  PB_CUDA(cudaMemcpyAsync(states, e->d_states, n * 16, cudaMemcpyDeviceToHost, e->stream));
  PB_CUDA(cudaStreamSynchronize(e->stream));
  e->prof_resolve();
  uint32_t first = PB_OK;
  for (uint32_t i = 0; i < n; ++i) {
    if (rows[i].status) {
      if (errs) sampler_error(&errs[i], rows[i], 151936);
      if (!first) first = rows[i].status;
      ids[i] = 0;
    } else {
      ids[i] = rows[i].selected;
      if (errs) std::memset(&errs[i], 0, sizeof(pb_error));
    }
  }
  return first;
}

uint32_t pb_engine_generate(pb_engine* e, uint32_t n, const uint32_t* seqs,
                            pb_sampling_state* states, uint32_t steps, uint32_t* out_tokens,
                            pb_error* errs) {
  if (!e || n == 0 || n > e->last_rows || !distinct_seqs(e, n, seqs)) return PB_CAPACITY;
  cudaSetDevice(e->device);
  for (uint32_t i = 0; i < n; ++i) {
    if (!seq_ok(e, seqs[i])) return PB_CAPACITY;
    const Slot& s = e->slots[seqs[i]];
    if (s.state != PB_STATE_READY && s.state != PB_STATE_EOS) {
      if (errs) errs[i] = e->state_error(s, PB_STATE_READY, 0);
      return PB_STATE;
    }
    if ((uint64_t)s.emitted + steps > s.reserve || (uint64_t)s.position + steps > e->context_limit) {
      if (errs) errs[i] = make_error(PB_CONTEXT, DOM_PROMPT, NO_LAYER, s.position, NO_TENSOR,
                                     s.reserve, (uint64_t)s.emitted + steps, K_RESERVE, 1);
      return PB_CONTEXT;
    }
  }
  std::vector<uint64_t> off(n);
  for (uint32_t i = 0; i < n; ++i) {
    off[i] = (uint64_t)seqs[i] * e->capacity;
    e->h_slots[i] = (int)seqs[i];
    e->h_positions[i] = (int)e->slots[seqs[i]].position;
  }
  PB_CUDA(cudaMemcpyAsync(e->d_hist_offset, off.data(), n * 8, cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaMemcpyAsync(e->d_slots, e->h_slots, n * 4, cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaMemcpyAsync(e->d_positions, e->h_positions, n * 4, cudaMemcpyHostToDevice, e->stream));
  PB_CUDA(cudaMemcpyAsync(e->d_states, states, n * 16, cudaMemcpyHostToDevice, e->stream));
  uint32_t first = PB_OK;
  std::vector<char> failed(n, 0);
  const int threads = 128, blocks = (int)((n + threads - 1) / threads);
  for (uint32_t done = 0; done < steps;) {
    const uint32_t chunk = std::min<uint32_t>(pb_engine::kErrSteps, steps - done);
    // the logs of this chunk are indexed by position - base on the device
    PB_CUDA(cudaMemcpyAsync(e->d_base, e->d_positions, n * 4, cudaMemcpyDeviceToDevice, e->stream));
    for (uint32_t t = 0; t < chunk; ++t) {
      int span = 4;
      for (uint32_t i = 0; i < n; ++i)
        span = std::max(span, (int)((e->slots[seqs[i]].position + done + t + 4) & ~3u));
      // Only the last step's greedy id is published (InferenceStep::selected).
      const bool greedy = done + t + 1 == steps;
      e->max_span = e->graph_span(span, n);
      auto one_step = [&] {
        // history length == position (every evaluated token is in the history)
        e->prof_mark(PB_KC_SAMPLER);
        e->launches += e->sample_rows(n, reinterpret_cast<const uint32_t*>(e->d_positions)) - 1;
        e->prof_mark(PB_KC_SAMPLER);
        pb::launch_pdl(take_sample_kernel, blocks, threads, 0, e->stream, e->d_sampled,
                       e->d_tokens, e->d_positions, e->d_base, e->d_samp_status, e->d_token_log,
                       (int)n);
        e->enqueue_forward(n, true, e->d_err_cur, false);
        pb::launch_pdl(finish_step_kernel, blocks, threads, 0, e->stream, e->d_positions, e->d_base,
                       e->d_err_cur, e->d_err, (int)n);
        e->launches += 3;
      };
      // The last step's greedy id comes from a launch of its own, so that
      // every step of a generate call replays the same graph.
      if (!e->run_step(pb_engine::GraphKey{n, e->max_span, 1}, one_step))
        PB_CUDA(cudaGetLastError());
      if (greedy) {
        e->prof_mark(PB_KC_ARGMAX);
        pb::launch_argmax(e->logits, pb::kVocab, (int)n, pb::kVocab, e->d_greedy,
                          e->d_greedy_bits, nullptr, e->stream);
        e->prof_mark(PB_KC_ARGMAX);
        ++e->launches;
      }
    }
    PB_CUDA(cudaGetLastError());
    std::vector<unsigned long long> serr((size_t)chunk * n);
    std::vector<uint32_t> toks((size_t)chunk * n);
    PB_CUDA(cudaMemcpyAsync(e->h_err, e->d_err, (size_t)chunk * n * 8, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaMemcpyAsync(serr.data(), e->d_samp_status, (size_t)chunk * n * 8, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaMemcpyAsync(toks.data(), e->d_token_log, (size_t)chunk * n * 4, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaMemcpyAsync(e->h_greedy, e->d_greedy, n * 4, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaMemcpyAsync(e->h_greedy_bits, e->d_greedy_bits, n * 4, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaMemcpyAsync(e->h_tc_status, e->d_tc_status, 4, cudaMemcpyDeviceToHost, e->stream));
    PB_CUDA(cudaStreamSynchronize(e->stream));
    e->prof_resolve();
    if (e->check_tc_status()) return PB_DEVICE;
    for (uint32_t t = 0; t < chunk; ++t)
      for (uint32_t i = 0; i < n; ++i) {
        Slot& s = e->slots[seqs[i]];
        if (failed[i]) continue;
        const unsigned long long se = serr[(size_t)t * n + i];
        const unsigned long long fe = e->h_err[(size_t)t * n + i];
        if (se != pb::kNoError) {
          pb::SamplerRow r{(uint32_t)(se >> 56), (uint32_t)(se >> 32) & 0xffffffu, (uint32_t)se, 0};
          pb_error er;
          sampler_error(&er, r, 151936);
          if (errs) errs[i] = er;
          e->fault(s, er, nullptr);
          failed[i] = 1;
          if (!first) first = er.status;
          continue;
        }
        if (fe != pb::kNoError) {
          pb_error er = stage_error(fe, s.position);
          if (errs) errs[i] = e->fault(s, er, nullptr);
          failed[i] = 1;
          if (!first) first = er.status;
          continue;
        }
        if (out_tokens) out_tokens[(size_t)(done + t) * n + i] = toks[(size_t)t * n + i];
        e->advance(s);
        s.emitted += 1;
      }
    done += chunk;
  }
  PB_CUDA(cudaMemcpyAsync(states, e->d_states, n * 16, cudaMemcpyDeviceToHost, e->stream));
  PB_CUDA(cudaStreamSynchronize(e->stream));
  for (uint32_t i = 0; i < n; ++i)
    if (!failed[i]) e->publish(e->slots[seqs[i]], i);
  e->last_rows = n;
  return first;
}

void* pb_engine_stream(pb_engine* e) { return e ? (void*)e->stream : nullptr; }

uint64_t pb_engine_launch_count(pb_engine* e) { return e ? e->launches : 0; }

uint32_t pb_engine_profile(pb_engine* e, uint32_t class_mask) {
  if (!e) return PB_CAPACITY;
  e->prof_mask = class_mask;
  e->prof_used = 0;
  for (int i = 0; i < 16; ++i) { e->prof_ms[i] = 0.0; e->prof_count[i] = 0; }
  return PB_OK;
}

uint32_t pb_engine_profile_read(pb_engine* e, double* ms_out, uint64_t* launches_out) {
  if (!e) return PB_CAPACITY;
  for (int i = 0; i < 16; ++i) {
    if (ms_out) ms_out[i] = e->prof_ms[i];
    if (launches_out) launches_out[i] = e->prof_count[i];
  }
  return PB_OK;
}

}  // extern "C"
