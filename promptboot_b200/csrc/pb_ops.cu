// Host-buffer sampler entry points (inference.rs:814-965 of sulewicz/promptboot)
// and the device-pointer kernel operators of the C ABI.
#include "pb_common.cuh"
#include "pb_host.h"
#include "pb_kernels.cuh"

#include <algorithm>
#include <vector>

namespace {

constexpr uint32_t NO_LAYER = 0xffffffffu;
constexpr uint32_t NO_TENSOR = 0xffffffffu;
constexpr uint64_t kV = 151936;

void set_err(pb_error* e, uint32_t status, uint32_t domain, uint64_t needed, uint64_t available,
             uint32_t kind, uint32_t sub) {
  if (!e) return;
  e->status = status; e->domain = domain; e->layer = NO_LAYER; e->position = 0;
  e->tensor_id = NO_TENSOR; e->reserved = 0; e->needed = needed; e->available = available;
  e->detail = ((uint64_t)kind << 32) | sub;
}

// inference.rs:737-753 (length) then inference.rs:883-903 (first non-finite word)
uint32_t validate_logits(const uint32_t* logits, uint64_t len, pb_error* err) {
  if (len != kV) { set_err(err, PB_CAPACITY, 18, kV, len, 12, 0); return PB_CAPACITY; }
  for (uint64_t i = 0; i < len; ++i)
    if ((logits[i] & 0x7f800000u) == 0x7f800000u) {
      set_err(err, PB_NONFINITE_OUTPUT, 19, 0, logits[i], 7, (uint32_t)i);
      return PB_NONFINITE_OUTPUT;
    }
  return PB_OK;
}

// Device buffers and stream of the single-row host-API sampler calls, kept per
// host thread and device for the life of the thread: a REPL-style caller
// (src/model_repl.rs:945-967 in the reference calls the sampler once per token)
// pays no device allocation per call.  The history buffer grows to the longest
// history seen so far; everything else has a fixed size.
struct RowScratch {
  int device = -1;
  cudaStream_t stream = nullptr;
  float* logits = nullptr;
  uint32_t* history = nullptr;
  uint64_t history_words = 0;
  uint64_t* offset = nullptr;
  uint32_t* length = nullptr;
  uint8_t* seen = nullptr;
  unsigned long long* state = nullptr;
  pb::SamplerRow* out = nullptr;
  uint32_t* pairs = nullptr;
  unsigned long long* cand = nullptr;  // the split sampler's part lists
  ~RowScratch() {
    if (device < 0) return;
    cudaSetDevice(device);
    void* p[] = {logits, history, offset, length, seen, state, out, pairs, cand};
    for (void* x : p) if (x) cudaFree(x);
    if (stream) cudaStreamDestroy(stream);
  }
  uint32_t setup(int dev) {
    device = dev;
    PB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    PB_CUDA(cudaMalloc(&logits, kV * 4));
    PB_CUDA(cudaMalloc(&offset, 8));
    PB_CUDA(cudaMalloc(&length, 4));
    PB_CUDA(cudaMalloc(&state, 16));
    PB_CUDA(cudaMalloc(&out, sizeof(pb::SamplerRow)));
    PB_CUDA(cudaMalloc(&seen, PB_SEEN_BYTES));
    PB_CUDA(cudaMalloc(&pairs, 16 * 4));
    PB_CUDA(cudaMalloc(&cand, pb::split_sampler_words(1) * 8));
    const uint64_t zero = 0;
    PB_CUDA(cudaMemcpyAsync(offset, &zero, 8, cudaMemcpyHostToDevice, stream));
    PB_CUDA(cudaStreamSynchronize(stream));
    return PB_OK;
  }
  uint32_t reserve_history(uint64_t words) {
    if (words <= history_words) return PB_OK;
    if (history) PB_CUDA(cudaFree(history));
    history = nullptr;
    history_words = 0;
    const uint64_t grown = std::max<uint64_t>(words, 4096);
    PB_CUDA(cudaMalloc(&history, grown * 4));
    history_words = grown;
    return PB_OK;
  }
};

// The calling thread's scratch for the current device (set up on first use).
uint32_t row_scratch(RowScratch** out) {
  static thread_local RowScratch per_device[64];
  int dev = 0;
  PB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    pb::set_last_error("device ordinal out of range");
    return PB_DEVICE;
  }
  RowScratch& s = per_device[dev];
  if (s.device < 0) {
    uint32_t st = s.setup(dev);
    if (st) return st;
  }
  *out = &s;
  return PB_OK;
}

uint32_t run_sampler_row(uint32_t* logits, const uint32_t* tokens, uint64_t count,
                         const uint8_t* seen, pb_sampling_state* state, pb::SamplerRow* row,
                         bool write_back) {
  RowScratch* s = nullptr;
  uint32_t st = row_scratch(&s);
  if (st) return st;
  st = s->reserve_history(count);
  if (st) return st;
  const uint32_t n = (uint32_t)count;
  cudaStream_t stream = s->stream;
  PB_CUDA(cudaMemcpyAsync(s->logits, logits, kV * 4, cudaMemcpyHostToDevice, stream));
  if (count) PB_CUDA(cudaMemcpyAsync(s->history, tokens, count * 4, cudaMemcpyHostToDevice, stream));
  PB_CUDA(cudaMemcpyAsync(s->length, &n, 4, cudaMemcpyHostToDevice, stream));
  PB_CUDA(cudaMemcpyAsync(s->state, state, 16, cudaMemcpyHostToDevice, stream));
  if (seen) PB_CUDA(cudaMemcpyAsync(s->seen, seen, PB_SEEN_BYTES, cudaMemcpyHostToDevice, stream));
  pb::launch_sampler_split(s->logits, kV, 1, (int)kV, s->history, s->offset, s->length,
                           seen ? s->seen : nullptr, s->state, s->out, s->cand, stream);
  PB_CUDA(cudaGetLastError());
  PB_CUDA(cudaMemcpyAsync(row, s->out, sizeof(pb::SamplerRow), cudaMemcpyDeviceToHost, stream));
  PB_CUDA(cudaStreamSynchronize(stream));
  if (row->status == 0) {
    PB_CUDA(cudaMemcpyAsync(state, s->state, 16, cudaMemcpyDeviceToHost, stream));
    if (write_back)
      PB_CUDA(cudaMemcpyAsync(logits, s->logits, kV * 4, cudaMemcpyDeviceToHost, stream));
    PB_CUDA(cudaStreamSynchronize(stream));
  }
  return PB_OK;
}

__global__ void staging_kernel(const int8_t* aq, const float* ad, int rows, int blocks,
                               uint8_t* staging) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * blocks) return;
  int r = i / blocks, b = i % blocks;
  uint8_t* out = staging + (size_t)i * 34;
  uint16_t h = pb::f32_to_half(__float_as_uint(ad[(size_t)r * pb::kActBlocks + b]));
  out[0] = (uint8_t)(h & 0xff);
  out[1] = (uint8_t)(h >> 8);
  for (int e = 0; e < 32; ++e) out[2 + e] = (uint8_t)aq[(size_t)r * pb::kActStride + b * 32 + e];
}

__global__ void expf_kernel(const uint32_t* x, uint64_t n, uint32_t* y) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = pb::bitsf(pb::expf_ref(pb::fbits(x[i])));
}

__global__ void iota_kernel(int* p, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = i;
}

// Tensor-core operands of one operator call: the weight tile image and the
// activation tile layout (zeroed, so padding sequences hold finite values).
struct TcScratch {
  uint8_t* image = nullptr;
  int8_t* aq = nullptr;
  int seqs = 0;
  cudaStream_t s;
  explicit TcScratch(cudaStream_t st) : s(st) {}
  cudaError_t alloc(size_t image_bytes, uint32_t rows, uint32_t cols) {
    seqs = (int)((rows + 63) / 64 * 64);
    const size_t act = pb::tc_act_bytes(seqs, (int)cols);
    cudaError_t e = cudaMallocAsync(&image, image_bytes, s);
    if (!e) e = cudaMallocAsync(&aq, act, s);
    if (!e) e = cudaMemsetAsync(aq, 0, act, s);
    return e;
  }
  ~TcScratch() {
    void* p[] = {image, aq};
    for (void* x : p) if (x) cudaFreeAsync(x, s);
  }
};

// Operator scratch: quantized activations, stage-error words, slot/position maps.
struct OpScratch {
  int8_t* aq = nullptr;
  float* ad = nullptr;
  int* asum = nullptr;
  unsigned long long* err = nullptr;
  int* slots = nullptr;
  int* positions = nullptr;
  unsigned int* tc_status = nullptr;
  cudaStream_t s;
  explicit OpScratch(cudaStream_t st) : s(st) {}
  cudaError_t alloc(uint32_t rows) {
    cudaError_t e = cudaMallocAsync(&aq, (size_t)rows * pb::kActStride, s);
    if (!e) e = cudaMallocAsync(&ad, (size_t)rows * pb::kActBlocks * 4, s);
    if (!e) e = cudaMallocAsync(&asum, (size_t)rows * pb::kActBlocks * 4, s);
    if (!e) e = cudaMallocAsync(&err, (size_t)rows * 8, s);
    if (!e) e = cudaMallocAsync(&slots, (size_t)rows * 4, s);
    if (!e) e = cudaMallocAsync(&positions, (size_t)rows * 4, s);
    if (!e) e = cudaMallocAsync(&tc_status, 4, s);
    if (!e) e = cudaMemsetAsync(tc_status, 0, 4, s);
    if (!e) e = cudaMemsetAsync(err, 0xff, (size_t)rows * 8, s);
    if (!e) iota_kernel<<<(rows + 127) / 128, 128, 0, s>>>(slots, (int)rows);
    return e;
  }
  ~OpScratch() {
    void* p[] = {aq, ad, asum, err, slots, positions, tc_status};
    for (void* x : p) if (x) cudaFreeAsync(x, s);
  }
  pb::Batch batch(uint32_t rows) const {
    pb::Batch b{};
    b.rows = (int)rows; b.slots = slots; b.positions = positions; b.tokens = nullptr;
    b.aq = aq; b.ad = ad; b.asum = asum; b.err = err;
    return b;
  }
};

}  // namespace

extern "C" {

void pb_sampling_state_init(pb_sampling_state* state, uint64_t seed) {
  if (!state) return;
  state->state = seed == 0 ? 0x9e3779b97f4a7c15ull : seed;
  state->draws = 0;
}

uint32_t pb_sample_token(const uint32_t* logits, uint64_t len, pb_sampling_state* state,
                         uint32_t* out, pb_error* err) {
  uint32_t st = validate_logits(logits, len, err);
  if (st) return st;
  std::vector<uint32_t> copy(logits, logits + len);
  pb::SamplerRow row{};
  st = run_sampler_row(copy.data(), nullptr, 0, nullptr, state, &row, false);
  if (st) return st;
  if (out) *out = row.selected;
  return PB_OK;
}

uint32_t pb_sample_token_with_repetition(uint32_t* logits, uint64_t len, const uint32_t* tokens,
                                         uint64_t count, uint8_t* seen, uint64_t seen_len,
                                         pb_sampling_state* state, uint32_t* out, pb_error* err) {
  uint32_t st = validate_logits(logits, len, err);
  if (st) return st;
  const uint64_t need = (len + 7) / 8;
  if (!seen || seen_len < need) {
    set_err(err, PB_CAPACITY, 19, need, seen ? seen_len : 0, 4, 2);
    return PB_CAPACITY;
  }
  for (uint64_t i = 0; i < count; ++i)
    if (tokens[i] >= len) {
      set_err(err, PB_TOKEN_ID, 19, len, tokens[i], 2, 0);
      return PB_TOKEN_ID;
    }
  pb::SamplerRow row{};
  st = run_sampler_row(logits, tokens, count, seen, state, &row, true);
  if (st) return st;
  // fp32_sse2.rs:1871-1875: every history token's bit is cleared afterwards
  for (uint64_t i = 0; i < count; ++i) seen[tokens[i] / 8] &= (uint8_t)~(1u << (tokens[i] & 7));
  if (out) *out = row.selected;
  return PB_OK;
}

uint32_t pb_greedy_token(const uint32_t* logits, uint64_t len, uint32_t* out, pb_error* err) {
  uint32_t st = validate_logits(logits, len, err);
  if (st) return st;
  RowScratch* s = nullptr;
  st = row_scratch(&s);
  if (st) return st;
  PB_CUDA(cudaMemcpyAsync(s->logits, logits, kV * 4, cudaMemcpyHostToDevice, s->stream));
  pb::launch_argmax(s->logits, kV, 1, (int)kV, s->pairs, s->pairs + 1, nullptr, s->stream);
  PB_CUDA(cudaGetLastError());
  uint32_t host[2];
  PB_CUDA(cudaMemcpyAsync(host, s->pairs, 8, cudaMemcpyDeviceToHost, s->stream));
  PB_CUDA(cudaStreamSynchronize(s->stream));
  if (out) *out = host[0];
  return PB_OK;
}

uint32_t pb_top_logits_8(const uint32_t* logits, uint64_t len, pb_top_logit* out8, pb_error* err) {
  uint32_t st = validate_logits(logits, len, err);
  if (st) return st;
  RowScratch* s = nullptr;
  st = row_scratch(&s);
  if (st) return st;
  PB_CUDA(cudaMemcpyAsync(s->logits, logits, kV * 4, cudaMemcpyHostToDevice, s->stream));
  pb::launch_topk8(s->logits, kV, 1, (int)kV, s->pairs, nullptr, s->stream);
  PB_CUDA(cudaGetLastError());
  uint32_t host[16];
  PB_CUDA(cudaMemcpyAsync(host, s->pairs, sizeof host, cudaMemcpyDeviceToHost, s->stream));
  PB_CUDA(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < 8; ++i) out8[i] = pb_top_logit{host[2 * i], host[2 * i + 1]};
  return PB_OK;
}

uint32_t pb_sample_batch_device(uint32_t* logits_device, uint64_t ld, uint32_t rows,
                                const uint32_t* history_device, const uint64_t* offsets_device,
                                const uint32_t* lengths_device, pb_sampling_state* states_device,
                                uint32_t* out_device, void* stream) {
  if (!logits_device || rows == 0 || ld < kV || (ld & 3)) return PB_CAPACITY;
  pb::launch_sampler(reinterpret_cast<float*>(logits_device), ld, (int)rows, (int)kV,
                     history_device, offsets_device, lengths_device, nullptr,
                     reinterpret_cast<unsigned long long*>(states_device),
                     reinterpret_cast<pb::SamplerRow*>(out_device), (cudaStream_t)stream);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_qmatvec_device(uint32_t wtype, const uint8_t* w, uint32_t rows, uint32_t cols,
                           const float* x, uint32_t batch, float* y, void* stream) {
  const uint32_t nb = cols / 32;
  const uint32_t rt = nb > 64 ? 8 : 32;
  if ((wtype != pb::W_Q4_0 && wtype != pb::W_Q8_0) || cols % 32 || cols > (uint32_t)pb::kFfn ||
      rows == 0 || rows % rt || batch == 0)
    return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  pb::init_kernel_attributes();
  OpScratch scr(s);
  PB_CUDA(scr.alloc(batch));
  pb::Batch b = scr.batch(batch);
  const pb::Epilogue ep{pb::EPI_STORE, y, rows, nullptr, scr.err, 0, 0};
  if (batch >= (uint32_t)pb::kTcMinBatch && pb::tc_shape_supported((int)rows, (int)cols)) {
    // Tensor-core path: tile image of w and the activation tile layout, built
    // per call into stream-ordered scratch.
    TcScratch tc(s);
    PB_CUDA(tc.alloc(pb::tc_image_bytes((int)rows, (int)cols), batch, cols));
    b.aq_tc = tc.aq; b.tc_seqs = tc.seqs;
    pb::launch_tc_repack((int)wtype, w, (int)rows, (int)cols, tc.image, s);
    pb::launch_quant(b, x, cols, (int)cols, s);
    pb::TcGemm g{};
    g.wtype = (int)wtype; g.tiles = tc.image; g.rtiles = (int)rows / 128; g.nb = (int)nb;
    g.nseg = 1; g.seg[0].rtile_end = g.rtiles; g.seg[0].ep = ep;
    pb::launch_tc_gemm(g, b, scr.tc_status, s);
    PB_CUDA(cudaGetLastError());
  } else {
    pb::launch_quant(b, x, cols, (int)cols, s);
    pb::launch_qgemv((int)wtype, w, (int)rows, (int)cols, b, ep, s);
    PB_CUDA(cudaGetLastError());
  }
  unsigned int status = 0;
  PB_CUDA(cudaMemcpyAsync(&status, scr.tc_status, 4, cudaMemcpyDeviceToHost, s));
  PB_CUDA(cudaStreamSynchronize(s));
  if (status) {
    pb::set_last_error("tensor-core matvec pipeline timed out waiting for an MMA");
    return PB_DEVICE;
  }
  return PB_OK;
}

namespace {

// The model tensor behind pb_model_matvec_device: weights, shape and, for the
// tensor-core path, its tile image inside the model's stacked images.
struct ModelMatrix {
  int wtype = 0, rows = 0, cols = 0;
  const uint8_t* w = nullptr;
  const uint8_t* image = nullptr;
};

bool model_matrix(const pb_model* m, uint32_t id, ModelMatrix* out) {
  if (id == 0) {  // the Q4_0 token embedding as a 896 -> 151936 head (tied weights)
    *out = {pb::W_Q4_0, pb::kVocab, 896, m->tensor(0), m->tc_embed};
    return true;
  }
  if (id == 290) {
    *out = {pb::W_Q8_0, pb::kVocab, 896, m->tensor(290), m->tc + m->tc_head};
    return true;
  }
  if (id < 1 || id > 288) return false;
  const int layer = (int)(id - 1) / 12;
  const uint32_t role = 10 + (id - 1) % 12;
  const size_t i896 = pb::tc_image_bytes(896, 896), i128 = pb::tc_image_bytes(128, 896);
  const size_t i4864 = pb::tc_image_bytes(4864, 896);
  const uint8_t* tc = m->tc;
  switch (role) {
    case 19: *out = {pb::W_Q4_0, 896, 896, m->tensor(id), tc + m->tc_qkv[layer]}; return true;
    case 16: *out = {pb::W_Q4_0, 128, 896, m->tensor(id), tc + m->tc_qkv[layer] + i896}; return true;
    case 21: *out = {pb::W_Q4_0, 128, 896, m->tensor(id), tc + m->tc_qkv[layer] + i896 + i128}; return true;
    case 17: *out = {pb::W_Q4_0, 896, 896, m->tensor(id), tc + m->tc_o[layer]}; return true;
    case 12: *out = {pb::W_Q4_0, 4864, 896, m->tensor(id), tc + m->tc_gateup[layer]}; return true;
    case 13: *out = {pb::W_Q4_0, 4864, 896, m->tensor(id), tc + m->tc_gateup[layer] + i4864}; return true;
    case 11: *out = {pb::W_Q4_0, 896, 4864, m->tensor(id), tc + m->tc_down[layer]}; return true;
    default: return false;
  }
}

}  // namespace

uint32_t pb_model_matvec_device(pb_model* m, uint32_t id, const float* x, uint32_t batch, float* y,
                                void* stream) {
  ModelMatrix mm;
  if (!m || !x || !y || batch == 0 || batch > 256 || !model_matrix(m, id, &mm)) return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  // scratch: row-major Q8_0 activations, block sums, error words, then the
  // tensor-core layout for 256 rows
  const size_t need = 256 * (size_t)(pb::kActStride + pb::kActBlocks * 8 + 8) +
                      pb::tc_act_bytes(256, pb::kFfn);
  if (m->op_scratch_bytes < need) {
    PB_CUDA(cudaStreamSynchronize(s));
    if (m->op_scratch) PB_CUDA(cudaFree(m->op_scratch));
    m->op_scratch = nullptr;
    PB_CUDA(cudaMalloc(&m->op_scratch, need));
    PB_CUDA(cudaMemset(m->op_scratch, 0, need));
    m->op_scratch_bytes = need;
  }
  if (!m->op_status) {
    PB_CUDA(cudaMalloc(&m->op_status, 4));
    PB_CUDA(cudaMemset(m->op_status, 0, 4));
  }
  if (id == 0 && (int)batch >= pb::kTcMinBatch && !m->tc_embed) {
    PB_CUDA(cudaStreamSynchronize(s));
    PB_CUDA(cudaMalloc(&m->tc_embed, pb::tc_image_bytes(pb::kVocab, 896)));
    pb::launch_tc_repack(pb::W_Q4_0, m->tensor(0), pb::kVocab, 896, m->tc_embed, s);
    PB_CUDA(cudaGetLastError());
    mm.image = m->tc_embed;
  }
  pb::init_kernel_attributes();
  uint8_t* p = m->op_scratch;
  pb::Batch b{};
  b.rows = (int)batch;
  b.aq = reinterpret_cast<int8_t*>(p);            p += 256 * (size_t)pb::kActStride;
  b.ad = reinterpret_cast<float*>(p);             p += 256 * (size_t)pb::kActBlocks * 4;
  b.asum = reinterpret_cast<int*>(p);             p += 256 * (size_t)pb::kActBlocks * 4;
  b.err = reinterpret_cast<unsigned long long*>(p); p += 256 * 8;
  PB_CUDA(cudaMemsetAsync(b.err, 0xff, batch * 8, s));
  const pb::Epilogue ep{pb::EPI_STORE, y, (size_t)mm.rows, nullptr, b.err, 0, 0};
  if ((int)batch >= pb::kTcMinBatch) {
    b.aq_tc = reinterpret_cast<int8_t*>(p);
    b.tc_seqs = 256;
    pb::launch_quant(b, x, mm.cols, mm.cols, s);
    pb::TcGemm g{};
    g.wtype = mm.wtype; g.tiles = mm.image; g.rtiles = mm.rows / 128; g.nb = mm.cols / 32;
    g.nseg = 1; g.seg[0].rtile_end = g.rtiles; g.seg[0].ep = ep;
    pb::launch_tc_gemm(g, b, m->op_status, s);
  } else {
    pb::launch_quant(b, x, mm.cols, mm.cols, s);
    pb::SmallGemv g{};
    g.wtype = mm.wtype; g.cols = mm.cols; g.rt = mm.cols > 896 ? 8 : 32; g.nseg = 1;
    g.seg[0].w = mm.w; g.seg[0].rows_end = mm.rows; g.seg[0].ep = ep;
    if (pb::small_gemv_supported(g, (int)batch))
      pb::launch_small_gemv(g, b, m->op_status, s);
    else
      pb::launch_qgemv(mm.wtype, mm.w, mm.rows, mm.cols, b, ep, s);
  }
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_model_matvec_status(pb_model* m, void* stream) {
  if (!m) return PB_CAPACITY;
  if (!m->op_status) return PB_OK;
  unsigned int st = 0;
  PB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  PB_CUDA(cudaMemcpy(&st, m->op_status, 4, cudaMemcpyDeviceToHost));
  if (st) {
    PB_CUDA(cudaMemset(m->op_status, 0, 4));
    pb::set_last_error("tensor-core matvec pipeline timed out waiting for an MMA");
    return PB_DEVICE;
  }
  return PB_OK;
}

uint32_t pb_quantize_q8_device(const float* x, uint32_t rows, uint32_t cols, uint8_t* staging,
                               void* stream) {
  if (cols % 32 || cols > (uint32_t)pb::kFfn || rows == 0) return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  OpScratch scr(s);
  PB_CUDA(scr.alloc(rows));
  pb::Batch b = scr.batch(rows);
  pb::launch_quant(b, x, cols, (int)cols, s);
  const int total = (int)(rows * (cols / 32));
  staging_kernel<<<(total + 127) / 128, 128, 0, s>>>(scr.aq, scr.ad, (int)rows, (int)(cols / 32), staging);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_rmsnorm_device(const float* x, const float* w, uint32_t rows, float* y, void* stream) {
  // The kernel moves each row as 224 float4 words.
  auto aligned16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  if (rows == 0 || !aligned16(x) || !aligned16(w) || !aligned16(y)) return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  OpScratch scr(s);
  PB_CUDA(scr.alloc(rows));
  pb::Batch b = scr.batch(rows);
  b.hidden = const_cast<float*>(x);
  b.norm_out = y;
  pb::launch_rmsnorm_quant(b, w, 1, pb::D_ATTN_NORM, s);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_swiglu_device(const float* gate, const float* up, uint32_t rows, float* out,
                          void* stream) {
  if (rows == 0) return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  OpScratch scr(s);
  PB_CUDA(scr.alloc(rows));
  pb::Batch b = scr.batch(rows);
  b.gate = const_cast<float*>(gate);
  b.up = const_cast<float*>(up);
  b.product_out = out;
  pb::launch_swiglu_quant(b, 1, s);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_rope_kv_device(float* q, float* k, const float* v, const uint32_t* positions_host,
                           uint32_t rows, float* kv, uint32_t capacity, uint32_t layer,
                           void* stream) {
  if (rows == 0 || capacity == 0 || (capacity & 3) || layer >= 24) return PB_CAPACITY;
  for (uint32_t r = 0; r < rows; ++r) if (positions_host[r] >= capacity) return PB_CAPACITY;
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<float> table;
  pb::build_rope_table(table);
  float* rope = nullptr;
  PB_CUDA(cudaMallocAsync(&rope, table.size() * 4, s));
  PB_CUDA(cudaMemcpyAsync(rope, table.data(), table.size() * 4, cudaMemcpyHostToDevice, s));
  OpScratch scr(s);
  PB_CUDA(scr.alloc(rows));
  PB_CUDA(cudaMemcpyAsync(scr.positions, positions_host, rows * 4, cudaMemcpyHostToDevice, s));
  pb::Batch b = scr.batch(rows);
  b.q = q; b.k = k; b.v = const_cast<float*>(v); b.kv = kv; b.capacity = capacity;
  pb::launch_rope_kv(b, (int)layer, rope, s);
  PB_CUDA(cudaGetLastError());
  PB_CUDA(cudaStreamSynchronize(s));
  PB_CUDA(cudaFree(rope));
  return PB_OK;
}

uint32_t pb_expf_device(const uint32_t* x, uint64_t n, uint32_t* y, void* stream) {
  if (!x || !y || n == 0) return PB_CAPACITY;
  const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, 148ull * 16);
  expf_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, n, y);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}

uint32_t pb_attention_device(const float* q, const float* kv, uint32_t capacity, uint32_t layer,
                             const uint32_t* positions_host, uint32_t rows, uint32_t span,
                             float* out, float* scores, void* stream) {
  if (rows == 0 || capacity == 0 || (capacity & 3) || capacity > PB_CONTEXT_LIMIT || layer >= 24 ||
      (span & 3) || span > PB_CONTEXT_LIMIT)
    return PB_CAPACITY;
  uint32_t span_max = span;
  for (uint32_t r = 0; r < rows; ++r) {
    if (positions_host[r] >= capacity) return PB_CAPACITY;
    span_max = std::max<uint32_t>(span_max, (positions_host[r] + 4) & ~3u);
  }
  cudaStream_t s = (cudaStream_t)stream;
  OpScratch scr(s);
  PB_CUDA(scr.alloc(rows));
  PB_CUDA(cudaMemcpyAsync(scr.positions, positions_host, rows * 4, cudaMemcpyHostToDevice, s));
  float* sc = nullptr;  // raw scores; the probabilities go to `scores`
  PB_CUDA(cudaMallocAsync(&sc, (size_t)rows * 14 * span_max * 4, s));
  pb::Batch b = scr.batch(rows);
  b.q = const_cast<float*>(q); b.kv = const_cast<float*>(kv); b.capacity = capacity;
  b.attn = out; b.scores = sc; b.score_stride = span_max; b.span_min = (int)span;
  b.probs_out = scores;
  pb::launch_attention(b, (int)layer, (int)span_max, false, nullptr, s);
  PB_CUDA(cudaGetLastError());
  PB_CUDA(cudaFreeAsync(sc, s));
  return PB_OK;
}

}  // extern "C"
