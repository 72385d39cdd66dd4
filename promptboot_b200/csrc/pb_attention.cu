// GQA decode attention for sm_100a, one CTA per (sequence, KV head) serving the
// KV head's 7 query heads, so every K/V word is read from HBM once.
//
// Arithmetic of the reference (sulewicz/promptboot fp32_sse2.rs:1430-1672), with
// every order-sensitive f64 sum kept in the reference's order:
//   score[h][p] = fl(f32(sum_c f64(fl(q[h][c] * k[p][c]))) * 0.125)  one thread per (h, p), c in order
//   max over p (exact in any order)
//   e = expf4(score - max), span padded to a multiple of 4 with e = 0
//   sum = sum over 4-groups IN ORDER of f64(fl(fl(e0+e1) + fl(e2+e3)))   one thread per head
//   prob = fl(e * f32(1.0 / sum))
//   out[h][c] = f32(sum_p f64(fl(prob[h][p] * v[p][c])))              one thread per (h, c), p in order
// K arrives in the reference's 4-position tiles and is transposed into shared
// memory ([position][component], row pitch 65 words) so that a warp reading 32
// positions at one component touches 32 banks; V tiles are row-major and are
// streamed with cp.async double buffering.  Scores live in shared memory, so this
// path serves contexts up to kAttnMaxPositions; longer ones use the per-head kernel.
#include "pb_common.cuh"
#include "pb_kernels.cuh"
#include "pb_quant.cuh"

namespace pb {
namespace {

constexpr int kHeadsPerKv = 7;
constexpr int kThreads = kHeadsPerKv * 64;  // 448
constexpr int kTile = 64;                   // positions per K/V tile
constexpr int kKPitch = 65;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

struct AttnSmem {
  static constexpr int kQ = (kHeadsPerKv * kKPitch + 3) & ~3;   // q, padded rows (16-B multiple)
  static constexpr int kKBuf = kTile * kKPitch;                  // transposed K tile
  static constexpr int kVBuf = kTile * 64;                       // V tile
  static constexpr int kBuf = kKBuf > kVBuf ? kKBuf : kVBuf;
  static size_t bytes(int span_cap) {
    return (size_t)(kQ + 2 * kBuf + kHeadsPerKv * span_cap + 64) * 4;
  }
};

__global__ void __launch_bounds__(kThreads)
attention_kv_group_kernel(Batch b, int layer, int span_cap, bool quantize) {
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;
  float* buf0 = sm + AttnSmem::kQ;
  float* buf1 = buf0 + AttnSmem::kBuf;
  float* sc = buf1 + AttnSmem::kBuf;                   // [7][span_cap]
  float* red = sc + kHeadsPerKv * span_cap;            // 64 words of scratch
  float* bufs[2] = {buf0, buf1};

  const int row = blockIdx.x >> 1, kh = blockIdx.x & 1;
  const int tid = threadIdx.x;
  const int h = tid >> 6, lane64 = tid & 63;
  const int positions = b.positions[row] + 1;
  const int span = max((positions + 3) & ~3, b.span_min);
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* kbase = kv + (size_t)layer * 4 * cap * 64 + (size_t)kh * (cap / 4) * 256;
  const float* vbase = kv + (size_t)layer * 4 * cap * 64 + 2 * cap * 64 + (size_t)kh * cap * 64;
  const int ntiles = (positions + kTile - 1) / kTile;

  qs[h * kKPitch + lane64] = b.q[(size_t)row * kHidden + (kh * kHeadsPerKv + h) * 64 + lane64];

  // ---- scores: K tiles transposed into shared memory, one (head, position) per thread
  // Tile t covers positions [64t, 64t + 64): the 16 4-position K tiles starting at
  // word 256 * 16t of this head, i.e. 4096 contiguous words.
  auto load_k = [&](int t, float (&reg)[10]) {
    const int p0 = t * kTile;
    const float* src = kbase + (size_t)p0 * 64;
#pragma unroll
    for (int i = 0; i < 10; ++i) {
      const int wi = tid + i * kThreads;
      const int p = p0 + (wi >> 8) * 4 + (wi & 3);
      reg[i] = (wi < 4096 && p < positions) ? src[wi] : 0.0f;
    }
  };
  auto store_k = [&](float* dst, const float (&reg)[10]) {
#pragma unroll
    for (int i = 0; i < 10; ++i) {
      const int wi = tid + i * kThreads;
      if (wi < 4096) dst[((wi >> 8) * 4 + (wi & 3)) * kKPitch + ((wi >> 2) & 63)] = reg[i];
    }
  };
  float kreg[10];
  load_k(0, kreg);
  store_k(buf0, kreg);
  __syncthreads();
  for (int t = 0; t < ntiles; ++t) {
    float* cur = bufs[t & 1];
    if (t + 1 < ntiles) load_k(t + 1, kreg);  // global loads in flight during the dots
    const int p = t * kTile + lane64;
    if (p < positions) {
      const float* kr = cur + lane64 * kKPitch;
      const float* qr = qs + h * kKPitch;
      double dot = 0.0;
#pragma unroll 16
      for (int c = 0; c < 64; ++c) dot += (double)__fmul_rn(qr[c], kr[c]);
      sc[h * span_cap + p] = __fmul_rn((float)dot, 0.125f);
    }
    if (t + 1 < ntiles) store_k(bufs[(t + 1) & 1], kreg);
    __syncthreads();
  }

  // ---- V tiles start streaming while the softmax runs
  auto load_v = [&](int t, float* dst) {
    const float* src = vbase + (size_t)t * kTile * 64;
    const int rows_here = min(kTile, positions - t * kTile);
    for (int i = tid; i < rows_here * 16; i += kThreads) cp_async16(dst + i * 4, src + i * 4);
    cp_commit();
  };
  load_v(0, buf0);
  if (ntiles > 1) load_v(1, buf1);
  else cp_commit();

  // ---- max per head (exact in any order)
  float m = fbits(0xff800000u);
  for (int p = lane64; p < positions; p += 64) m = fmaxf(m, sc[h * span_cap + p]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  const float maximum = fmaxf(red[2 * h], red[2 * h + 1]);

  // ---- e = expf4(s - max), masked tail e = 0
  for (int p = lane64; p < span; p += 64)
    sc[h * span_cap + p] = p < positions ? expf4_lane(__fsub_rn(sc[h * span_cap + p], maximum)) : 0.0f;
  __syncthreads();
  // ---- f64 sum over 4-groups in order, one thread per head
  if (lane64 == 0) {
    const float* e = sc + h * span_cap;
    double sum = 0.0;
    for (int p = 0; p < span; p += 4)
      sum += (double)__fadd_rn(__fadd_rn(e[p], e[p + 1]), __fadd_rn(e[p + 2], e[p + 3]));
    red[16 + h] = (float)(1.0 / sum);
  }
  __syncthreads();
  const float normalizer = red[16 + h];
  for (int p = lane64; p < positions; p += 64)
    sc[h * span_cap + p] = __fmul_rn(sc[h * span_cap + p], normalizer);
  if (b.probs_out) {
    float* dst = b.probs_out + ((size_t)row * kQHeads + kh * kHeadsPerKv + h) * b.score_stride;
    for (int p = lane64; p < span; p += 64) dst[p] = sc[h * span_cap + p];
  }

  // ---- values: one (head, component) chain per thread, positions in order
  double acc = 0.0;
  const float* prob = sc + h * span_cap;
  for (int t = 0; t < ntiles; ++t) {
    cp_wait1();
    __syncthreads();
    const float* vt = bufs[t & 1];
    const int p0 = t * kTile;
    const int rows_here = min(kTile, positions - p0);
#pragma unroll 8
    for (int i = 0; i < rows_here; ++i)
      acc += (double)__fmul_rn(prob[p0 + i], vt[i * 64 + lane64]);
    __syncthreads();
    if (t + 2 < ntiles) load_v(t + 2, bufs[t & 1]);
    else cp_commit();
  }
  cp_wait0();
  const float o = (float)acc;
  const int qh = kh * kHeadsPerKv + h;
  b.attn[(size_t)row * kHidden + qh * 64 + lane64] = o;
  check_finite(o, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh * 64 + lane64);
  if (quantize) {
    // The group's 448 outputs are Q8_0 blocks 14 kh .. 14 kh + 13 of the
    // o-projection input: stage them (q is no longer read) and quantize one
    // block per warp.
    qs[tid] = o;
    __syncthreads();
    const int w = tid >> 5;
    quantize_row_block(b, qs[w * 32 + (tid & 31)], row, kh * kHeadsPerKv * 2 + w, kHidden / 32);
  }
}

}  // namespace

int attention_smem_positions() { return kAttnMaxPositions; }

void launch_attention_grouped(const Batch& b, int layer, int span_cap, bool quantize, cudaStream_t s) {
  const size_t bytes = AttnSmem::bytes(span_cap);
  static size_t configured = 0;
  if (bytes > configured) {
    cudaFuncSetAttribute(attention_kv_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)AttnSmem::bytes(kAttnMaxPositions));
    configured = AttnSmem::bytes(kAttnMaxPositions);
  }
  attention_kv_group_kernel<<<b.rows * 2, kThreads, bytes, s>>>(b, layer, span_cap, quantize);
}

}  // namespace pb
