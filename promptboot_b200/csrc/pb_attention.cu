// GQA decode attention for sm_100a: every CTA serves the 7 query heads of one
// KV head, so every K/V word is read from HBM once.
//
// Arithmetic of the reference (sulewicz/promptboot fp32_sse2.rs:1430-1672), with
// every order-sensitive f64 sum kept in the reference's order:
//   score[h][p] = fl(f32(sum_c f64(fl(q[h][c] * k[p][c]))) * 0.125)  c in order
//   max over p (exact in any order)
//   e = expf4(score - max), span padded to a multiple of 4 with e = 0
//   sum = sum over 4-groups IN ORDER of f64(fl(fl(e0+e1) + fl(e2+e3)))   one lane per head
//   prob = fl(e * f32(1.0 / sum))
//   out[h][c] = f32(sum_p f64(fl(prob[h][p] * v[p][c])))              p in order
// Two launches, both 224 threads = one warp per query head of a KV head, so q
// and the probabilities are warp broadcasts and the softmax needs no block
// barrier:
//  * attention_scores_kernel: one CTA per (sequence, KV head, 64-position
//    chunk), so thousands of small CTAs keep every SM busy while K streams in.
//    K arrives in the reference's 4-position tiles ([component][4 positions],
//    1 KB) and is copied untransposed by cp.async into tiles padded to 260
//    words: lane (tile, pair) reads positions 4 tile + 2 pair + {0, 1} of one
//    component with one 8-byte load (two independent f64 chains per lane), and
//    a half-warp covers all 32 banks once.  Scores go to the global score
//    scratch (L2-resident).  With the RoPE table given, every CTA rotates q for
//    its 7 heads and the CTA of the last chunk also rotates k and writes this
//    step's K and V (decode steps, where no two rows share a slot).
//  * attention_pv_kernel: one CTA per (sequence, KV head); the softmax of each
//    head runs in its warp from the global scores, then V streams through two
//    64-row buffers while every lane keeps two f64 chains (components 2 lane
//    and 2 lane + 1, one 8-byte load per position, positions in order); the
//    second chain adds integer-built f64 images of its products instead of
//    converting them (scaled_product).
// The probabilities live in shared memory, so this path serves contexts up to
// kAttnMaxPositions; longer ones use the long-context launches below.
#include "pb_common.cuh"
#include "pb_kernels.cuh"
#include "pb_quant.cuh"

#include <cstdlib>

namespace pb {
namespace {

constexpr int kHeadsPerKv = 7;
constexpr int kThreads = kHeadsPerKv * 32;  // 224
constexpr int kChunk = 64;                  // positions per K/V chunk
constexpr int kTilePitch = 260;             // words per padded 4-position K tile

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// f64 bits of fl(a * b) * 2^-896, for a finite product: the sign stays in bit
// 31 of the high word, exponent and fraction move down three bits (the
// arithmetic shift's copies of the sign in bits 30..28 are cleared) and the
// fraction's low three bits open the low word; f32 subnormals land on f64
// subnormals with the same scale.  A chain that adds these images instead of
// f64(fl(a * b)) and multiplies by 2^896 at the end rounds exactly as the
// reference's chain: every term is a multiple of 2^-1045 once scaled, so a
// partial sum below the f64 normal range is exact in both domains, above it
// the roundings coincide, and no partial sum comes near either end of the
// range.  Three integer operations instead of one conversion on the XU pipe.
__device__ __forceinline__ double scaled_product(float a, float b) {
  double d;
  asm("{\n\t.reg .b32 t, hi, lo;\n\t"
      "mul.rn.f32 t, %1, %2;\n\t"
      "shr.s32 hi, t, 3;\n\t"
      "and.b32 hi, hi, 0x8FFFFFFF;\n\t"
      "shl.b32 lo, t, 29;\n\t"
      "mov.b64 %0, {lo, hi};\n\t}"
      : "=d"(d) : "f"(a), "f"(b));
  return d;
}

struct PvSmem {
  static constexpr int kVBuf = kChunk * 64;  // V rows
  static size_t bytes(int span_cap) { return (size_t)(2 * kVBuf + kHeadsPerKv * span_cap) * 4; }
};

__global__ void __launch_bounds__(kThreads, 8)
attention_scores_kernel(Batch b, int layer, const float* rope) {
  pdl_begin();
  __shared__ __align__(16) float qs[kHeadsPerKv * 64];
  __shared__ __align__(16) float ks[(kChunk / 4) * kTilePitch];

  const int t = blockIdx.x, row = blockIdx.y >> 1, kh = blockIdx.y & 1;
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int positions = b.positions[row] + 1;
  if (t * kChunk >= positions) return;
  const bool last = (t + 1) * kChunk >= positions;
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* kbase = kv + (size_t)layer * 4 * cap * 64 + (size_t)kh * (cap / 4) * 256;

  const float* qg = b.q + (size_t)row * kHidden + kh * kHeadsPerKv * 64;
  if (rope) {
    // RoPE and the KV write of this step's position (fp32_sse2.rs:1413-1428,
    // inference.rs:1809-1887), for this CTA's 7 query heads and its KV head:
    // lane `pair` of warp h rotates (pair, pair + 32) of head 7 kh + h; in the
    // last chunk's CTA warp 0 also rotates K head kh and writes it, warps 1-2
    // write V head kh, and the stage checks are recorded once.
    const int position = positions - 1;
    const uint32_t ord = (uint32_t)layer + 1;
    const float* table = rope + (size_t)position * 64;
    const float c = table[lane * 2], sn = table[lane * 2 + 1];
    {
      const float left = qg[h * 64 + lane], right = qg[h * 64 + lane + 32];
      const float l2 = __fsub_rn(__fmul_rn(left, c), __fmul_rn(right, sn));
      const float r2 = __fadd_rn(__fmul_rn(left, sn), __fmul_rn(right, c));
      qs[h * 64 + lane] = l2;
      qs[h * 64 + lane + 32] = r2;
      if (last) {
        const int qi = (kh * kHeadsPerKv + h) * 64 + lane;
        check_finite(l2, &b.err[row], ord, D_ROPE, 0, qi);
        check_finite(r2, &b.err[row], ord, D_ROPE, 0, qi + 32);
      }
    }
    if (last) {
      float* kvs = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
      if (h == 0) {
        const float* kg = b.k + (size_t)row * 128 + kh * 64;
        const float left = kg[lane], right = kg[lane + 32];
        const float l2 = __fsub_rn(__fmul_rn(left, c), __fmul_rn(right, sn));
        const float r2 = __fadd_rn(__fmul_rn(left, sn), __fmul_rn(right, c));
        check_finite(l2, &b.err[row], ord, D_ROPE, 1, kh * 64 + lane);
        check_finite(r2, &b.err[row], ord, D_ROPE, 1, kh * 64 + lane + 32);
        check_finite(l2, &b.err[row], ord, D_KV, 0, kh * 64 + lane);
        check_finite(r2, &b.err[row], ord, D_KV, 0, kh * 64 + lane + 32);
        kvs[kv_key_word(cap, layer, kh, position, lane)] = l2;
        kvs[kv_key_word(cap, layer, kh, position, lane + 32)] = r2;
      } else if (h <= 2) {
        const int cc = (h - 1) * 32 + lane;
        kvs[kv_value_word(cap, layer, kh, position, cc)] = b.v[(size_t)row * 128 + kh * 64 + cc];
      }
      __threadfence();  // the cp.async reads below go through L2
    }
  } else {
    qs[tid] = qg[tid];
    qs[tid + kThreads] = qg[tid + kThreads];
  }
  __syncthreads();

  // Chunk t = K tiles 16t .. 16t + 15, each 1 KB contiguous in the cache.
  {
    const int ntiles = (positions + 3) >> 2;
    const int tiles = min(kChunk / 4, ntiles - t * (kChunk / 4));
    const float* src = kbase + (size_t)t * (kChunk / 4) * 256;
    for (int i = tid; i < tiles * 64; i += kThreads)
      cp_async16(ks + (i >> 6) * kTilePitch + (i & 63) * 4, src + i * 4);
    cp_commit();
    cp_wait0();
  }
  __syncthreads();

  // lane (tile, pair) -> positions 4 tile + 2 pair + {0, 1} of the chunk
  const int tile = lane >> 1, pair = lane & 1;
  const float* qh = qs + h * 64;
  const float* kt = ks + tile * kTilePitch + 2 * pair;
  const int p = t * kChunk + 4 * tile + 2 * pair;
  if (p < positions) {
    double d0 = 0.0, d1 = 0.0;
#pragma unroll 4
    for (int c = 0; c < 64; c += 4) {
      const float4 q4 = *reinterpret_cast<const float4*>(qh + c);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 k2 = *reinterpret_cast<const float2*>(kt + (c + j) * 4);
        d0 += (double)__fmul_rn(qv[j], k2.x);
        d1 += (double)__fmul_rn(qv[j], k2.y);
      }
    }
    float* out = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv + h) * b.score_stride;
    out[p] = __fmul_rn((float)d0, 0.125f);
    if (p + 1 < positions) out[p + 1] = __fmul_rn((float)d1, 0.125f);
  }
}

template <bool kCheckV>
__global__ void __launch_bounds__(kThreads, 4)
attention_pv_kernel(Batch b, int layer, int span_cap, bool quantize) {
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  float* bufs[2] = {sm, sm + PvSmem::kVBuf};
  float* sc = sm + 2 * PvSmem::kVBuf;  // [7][span_cap]

  const int row = blockIdx.x >> 1, kh = blockIdx.x & 1;
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int positions = b.positions[row] + 1;
  const int span = max((positions + 3) & ~3, b.span_min);
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* vbase = kv + (size_t)layer * 4 * cap * 64 + 2 * cap * 64 + (size_t)kh * cap * 64;
  const int nchunks = (positions + kChunk - 1) / kChunk;
  float* score = sc + h * span_cap;
  const float* gs = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv + h) * b.score_stride;

  // ---- this head's scores into shared memory (one copy group), then the V
  // chunks start streaming while the softmax runs
  for (int i = lane; i < ((positions + 3) >> 2); i += 32) cp_async16(score + 4 * i, gs + 4 * i);
  cp_commit();
  auto load_v = [&](int t, float* dst) {
    const float* src = vbase + (size_t)t * kChunk * 64;
    const int rows_here = min(kChunk, positions - t * kChunk);
    for (int i = tid; i < rows_here * 16; i += kThreads) cp_async16(dst + i * 4, src + i * 4);
    cp_commit();
  };
  load_v(0, bufs[0]);
  if (nchunks > 1) load_v(1, bufs[1]);
  else cp_commit();

  // ---- softmax of head h, entirely within warp h
  asm volatile("cp.async.wait_group 2;" ::: "memory");  // the scores group has landed
  __syncwarp();
  float m = fbits(0xff800000u);
  for (int p = lane; p < positions; p += 32) m = fmaxf(m, score[p]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  for (int p = lane; p < span; p += 32)
    score[p] = p < positions ? expf4_lane(__fsub_rn(score[p], m)) : 0.0f;
  __syncwarp();
  float normalizer = 0.0f;
  if (lane == 0) {
    double sum = 0.0;
    for (int p = 0; p < span; p += 4) {
      const float4 e = *reinterpret_cast<const float4*>(score + p);
      sum += (double)__fadd_rn(__fadd_rn(e.x, e.y), __fadd_rn(e.z, e.w));
    }
    normalizer = (float)(1.0 / sum);
  }
  normalizer = __shfl_sync(0xffffffffu, normalizer, 0);
  for (int p = lane; p < positions; p += 32) score[p] = __fmul_rn(score[p], normalizer);
  __syncwarp();
  if (b.probs_out) {
    float* dst = b.probs_out + ((size_t)row * kQHeads + kh * kHeadsPerKv + h) * b.score_stride;
    for (int p = lane; p < span; p += 32) dst[p] = score[p];
  }

  // ---- values: lane owns components 2 lane and 2 lane + 1 of head h (one
  // 8-byte load per position), positions in order.  Component 2 lane + 1 sums
  // scaled images (scaled_product), valid when every product is finite: the
  // probabilities are (a finite normalizer means every e was finite), and
  // V is: by the v-projection stage check (Batch::kv_checked), or here, where
  // fma(v, 0, vchk) stays zero while every V word of the chain is finite;
  // otherwise the lane redoes that chain with conversions below.
  double acc0 = 0.0, acc1 = 0.0;
  float vchk = 0.0f;
  for (int t = 0; t < nchunks; ++t) {
    cp_wait1();
    __syncthreads();
    const float* vt = bufs[t & 1] + 2 * lane;
    const float* pr = score + t * kChunk;
    const int rows_here = min(kChunk, positions - t * kChunk);
    int i = 0;
    for (; i + 4 <= rows_here; i += 4) {
      const float4 p4 = *reinterpret_cast<const float4*>(pr + i);
      const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v2 = *reinterpret_cast<const float2*>(vt + (i + j) * 64);
        acc0 += (double)__fmul_rn(pv[j], v2.x);
        acc1 += scaled_product(pv[j], v2.y);
        if (kCheckV) vchk = __fmaf_rn(v2.y, 0.0f, vchk);
      }
    }
    for (; i < rows_here; ++i) {
      const float2 v2 = *reinterpret_cast<const float2*>(vt + i * 64);
      acc0 += (double)__fmul_rn(pr[i], v2.x);
      acc1 += scaled_product(pr[i], v2.y);
      if (kCheckV) vchk = __fmaf_rn(v2.y, 0.0f, vchk);
    }
    __syncthreads();
    if (t + 2 < nchunks) load_v(t + 2, bufs[t & 1]);
    else cp_commit();
  }
  cp_wait0();
  if (fabsf(normalizer) <= 0x1.fffffep127f && vchk == 0.0f) {
    acc1 *= 0x1p896;
  } else {
    acc1 = 0.0;
    for (int p = 0; p < positions; ++p)
      acc1 += (double)__fmul_rn(score[p], vbase[(size_t)p * 64 + 2 * lane + 1]);
  }
  const float o0 = (float)acc0, o1 = (float)acc1;
  const int qh_index = kh * kHeadsPerKv + h;
  float* out = b.attn + (size_t)row * kHidden + qh_index * 64;
  *reinterpret_cast<float2*>(out + 2 * lane) = make_float2(o0, o1);
  // Stage checks in index order within the lane (the row's atomicMin keeps the
  // lowest index anyway).
  check_finite(o0, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + 2 * lane);
  check_finite(o1, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + 2 * lane + 1);
  if (quantize) {
    // Head qh's 64 outputs are Q8_0 blocks 2 qh and 2 qh + 1 of the
    // o-projection input; element e of a block sits in lane e / 2 (+ 16 for the
    // second block), slot e % 2.
    const int src0 = lane >> 1, src1 = 16 + (lane >> 1);
    const float a0 = __shfl_sync(0xffffffffu, o0, src0), a1 = __shfl_sync(0xffffffffu, o1, src0);
    const float b0 = __shfl_sync(0xffffffffu, o0, src1), b1 = __shfl_sync(0xffffffffu, o1, src1);
    quantize_row_block(b, (lane & 1) ? a1 : a0, row, 2 * qh_index);
    quantize_row_block(b, (lane & 1) ? b1 : b0, row, 2 * qh_index + 1);
  }
}

// ------------------------------------------------------------ long contexts
//
// Beyond kAttnMaxPositions the probabilities no longer fit in shared memory.
// The scores come from attention_scores_kernel as above; then
//  * attention_softmax_long_kernel, one CTA per (sequence, query head): the
//    maximum, e = expf4(s - max) with the span padded by zeros, the 4-lane
//    group terms g = fl(fl(e0+e1) + fl(e2+e3)), their f64 sum, and the
//    probabilities fl(e * f32(1 / sum)) written over the scores.  The sum runs
//    as a tree when that is provably the reference's serial sum: every g is a
//    non-negative multiple of 2^L (L = the lowest bit any nonzero g can carry),
//    so when the total is below 2^(L+53) every partial sum of any grouping is
//    exactly representable and all orders give the exact total; otherwise one
//    thread repeats the serial sum in group order over the terms kept in
//    shared memory.
//  * attention_pv_long_kernel<G>, one CTA per (sequence, KV head, one of G
//    component groups): a thread owns the two f64 chains of components
//    (2 c, 2 c + 1) of one head over all positions in order, V rows of the
//    group and the 7 heads' probabilities streaming through shared memory, so
//    every V word is read once per KV head and the 7 x 64 chains of a KV head
//    run on G SMs.  Each chain is one dependent f64 add per position (8.2
//    cycles measured on B200): at 31k positions that latency, not HBM, bounds
//    the launch.

constexpr int kLongThreads = 256;
constexpr int kLongMaxGroups = kContextLimit / 4;  // spans of at most 32768 positions

__global__ void __launch_bounds__(kLongThreads)
attention_softmax_long_kernel(Batch b) {
  pdl_begin();
  __shared__ float wmax[kLongThreads / 32];
  __shared__ double wsum[kLongThreads / 32];
  __shared__ int wlow[kLongThreads / 32];
  __shared__ float normalizer_s;
  __shared__ float gterm[kLongMaxGroups];  // group terms for the serial fallback
  const int row = blockIdx.x / kQHeads, head = blockIdx.x % kQHeads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int positions = b.positions[row] + 1;
  const int span = max((positions + 3) & ~3, b.span_min);
  float* sc = b.scores + ((size_t)row * kQHeads + head) * b.score_stride;
  float4* sc4 = reinterpret_cast<float4*>(sc);
  const int groups = span >> 2;

  float m = fbits(0xff800000u);
  for (int i = tid; i < groups; i += kLongThreads) {
    const float4 s = sc4[i];
    const int p = 4 * i;
    if (p < positions) m = fmaxf(m, s.x);
    if (p + 1 < positions) m = fmaxf(m, s.y);
    if (p + 2 < positions) m = fmaxf(m, s.z);
    if (p + 3 < positions) m = fmaxf(m, s.w);
  }
  m = warp_max_f32(m);
  if (lane == 0) wmax[warp] = m;
  __syncthreads();
  m = wmax[0];
#pragma unroll
  for (int w = 1; w < kLongThreads / 32; ++w) m = fmaxf(m, wmax[w]);

  // e in place; group terms, their lowest possible bit and a tree partial sum
  double part = 0.0;
  int low = 1 << 20;
  for (int i = tid; i < groups; i += kLongThreads) {
    const float4 s = sc4[i];
    const int p = 4 * i;
    float4 e;
    e.x = p < positions ? expf4_lane(__fsub_rn(s.x, m)) : 0.0f;
    e.y = p + 1 < positions ? expf4_lane(__fsub_rn(s.y, m)) : 0.0f;
    e.z = p + 2 < positions ? expf4_lane(__fsub_rn(s.z, m)) : 0.0f;
    e.w = p + 3 < positions ? expf4_lane(__fsub_rn(s.w, m)) : 0.0f;
    sc4[i] = e;
    const float g = __fadd_rn(__fadd_rn(e.x, e.y), __fadd_rn(e.z, e.w));
    gterm[i] = g;
    part += (double)g;
    const uint32_t gb = bitsf(g) & 0x7fffffffu;
    if (gb != 0) {
      const int ex = (int)(gb >> 23);
      low = min(low, ex == 0 ? -149 : ex - 150);
    }
  }
  part = warp_sum_f64(part);
  for (int o = 16; o > 0; o >>= 1) low = min(low, __shfl_xor_sync(0xffffffffu, low, o));
  if (lane == 0) {
    wsum[warp] = part;
    wlow[warp] = low;
  }
  __syncthreads();
  if (tid == 0) {
    double total = 0.0;
    int lo = 1 << 20;
    for (int w = 0; w < kLongThreads / 32; ++w) {
      total += wsum[w];
      lo = min(lo, wlow[w]);
    }
    // A non-finite or too wide total: the serial sum in group order.  (The
    // tree's relative error is below 2^-40 for these term counts; the bound
    // keeps a margin of 2^-30.)
    const bool exact = lo <= 1000 && total * (1.0 + 0x1p-30) < ldexp(1.0, lo + 53);
    if (!exact) {
      double serial = 0.0;
#pragma unroll 8
      for (int i = 0; i < groups; ++i) serial += (double)gterm[i];
      total = serial;
    }
    normalizer_s = (float)(1.0 / total);
  }
  __syncthreads();
  const float normalizer = normalizer_s;
  float4* probs = b.probs_out ? reinterpret_cast<float4*>(
                                    b.probs_out + ((size_t)row * kQHeads + head) * b.score_stride)
                              : nullptr;
  for (int i = tid; i < groups; i += kLongThreads) {
    float4 e = sc4[i];
    const int p = 4 * i;
    if (p < positions) e.x = __fmul_rn(e.x, normalizer);
    if (p + 1 < positions) e.y = __fmul_rn(e.y, normalizer);
    if (p + 2 < positions) e.z = __fmul_rn(e.z, normalizer);
    if (p + 3 < positions) e.w = __fmul_rn(e.w, normalizer);
    sc4[i] = e;
    if (probs) probs[i] = e;
  }
}

// G component groups of 64 / G components per CTA; a thread owns the two
// chains of components (2 c, 2 c + 1) of one head, the first converting its
// products on the XU pipe, the second summing integer-built images
// (scaled_product), like attention_pv_kernel.  kLongStages chunks of
// kLongChunk positions are in flight (V rows of the group and the 7 heads'
// probabilities, cp.async into shared memory).
constexpr int kLongChunk = 128;
constexpr int kLongStages = 4;

template <int G>
struct PvLong {
  static constexpr int kComps = 64 / G;                           // components per CTA
  static constexpr int kPairs = kComps / 2;                       // threads per head
  static constexpr int kWorkers = kHeadsPerKv * kPairs;
  static constexpr int kThreads = (kWorkers + 31) / 32 * 32;
  static constexpr int kVWords = kLongChunk * kComps;              // V rows of one chunk
  static constexpr int kPWords = kHeadsPerKv * kLongChunk;         // probabilities of one chunk
  static constexpr int kStage = kVWords + kPWords;
  static constexpr size_t kBytes = (size_t)kLongStages * kStage * 4;
};

template <int G, bool kCheckV>
__global__ void __launch_bounds__(PvLong<G>::kThreads)
attention_pv_long_kernel(Batch b, int layer) {
  using C = PvLong<G>;
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  const int row = blockIdx.x >> 1, kh = blockIdx.x & 1, grp = blockIdx.y;
  const int tid = threadIdx.x;
  const int h = tid / C::kPairs, c2 = tid % C::kPairs;
  const bool active = tid < C::kWorkers;
  const int comp = grp * C::kComps + 2 * c2;  // this thread's first component
  const int positions = b.positions[row] + 1;
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* vbase = kv + (size_t)layer * 4 * cap * 64 + 2 * cap * 64 + (size_t)kh * cap * 64;
  const float* probs = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv) * b.score_stride;
  const int nchunks = (positions + kLongChunk - 1) / kLongChunk;

  auto load = [&](int t) {
    if (t < nchunks) {
      float* stage = sm + (t % kLongStages) * C::kStage;
      const int p0 = t * kLongChunk;
      const int rows_here = min(kLongChunk, positions - p0);
      constexpr int kPieces = C::kComps / 4;
      for (int i = tid; i < rows_here * kPieces; i += C::kThreads) {
        const int r = i / kPieces, piece = i % kPieces;
        cp_async16(stage + r * C::kComps + piece * 4,
                   vbase + (size_t)(p0 + r) * 64 + grp * C::kComps + piece * 4);
      }
      // probabilities of the 7 heads, rows_here rounded up to 4 (the scratch
      // holds the padded span)
      const int quads = (rows_here + 3) >> 2;
      float* pst = stage + C::kVWords;
      for (int i = tid; i < kHeadsPerKv * quads; i += C::kThreads) {
        const int hh = i / quads, q = i % quads;
        cp_async16(pst + hh * kLongChunk + 4 * q, probs + (size_t)hh * b.score_stride + p0 + 4 * q);
      }
    }
    cp_commit();  // one group per chunk slot, empty past the end
  };
#pragma unroll
  for (int t = 0; t < kLongStages - 1; ++t) load(t);

  double acc0 = 0.0, acc1 = 0.0;
  float vchk = 0.0f;
  for (int t = 0; t < nchunks; ++t) {
    load(t + kLongStages - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(kLongStages - 1) : "memory");
    __syncthreads();
    const float* stage = sm + (t % kLongStages) * C::kStage;
    const float* vt = stage + 2 * c2;  // this thread's component pair in each V row
    const float* pr = stage + C::kVWords + h * kLongChunk;
    const int rows_here = min(kLongChunk, positions - t * kLongChunk);
    if (active) {
      int i = 0;
      for (; i + 8 <= rows_here; i += 8) {
        const float4 pa = *reinterpret_cast<const float4*>(pr + i);
        const float4 pb = *reinterpret_cast<const float4*>(pr + i + 4);
        const float pv[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
        float2 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const float2*>(vt + (i + j) * C::kComps);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc0 += (double)__fmul_rn(pv[j], v[j].x);
          acc1 += scaled_product(pv[j], v[j].y);
          if (kCheckV) vchk = __fmaf_rn(v[j].y, 0.0f, vchk);
        }
      }
      for (; i < rows_here; ++i) {
        const float2 v = *reinterpret_cast<const float2*>(vt + i * C::kComps);
        acc0 += (double)__fmul_rn(pr[i], v.x);
        acc1 += scaled_product(pr[i], v.y);
        if (kCheckV) vchk = __fmaf_rn(v.y, 0.0f, vchk);
      }
    }
    __syncthreads();  // the slot is refilled by the next iteration's load
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (!active) return;
  const float* hprobs = probs + (size_t)h * b.score_stride;
  // The scaled chain needs finite products: finite probabilities (a finite
  // normalizer; a non-finite one shows in every probability word, position
  // 0's included) and finite V (the v-projection check, or vchk here).
  const float p0 = hprobs[0];
  if (fabsf(p0) <= 0x1.fffffep127f && vchk == 0.0f) {
    acc1 *= 0x1p896;
  } else {
    acc1 = 0.0;
    for (int p = 0; p < positions; ++p)
      acc1 += (double)__fmul_rn(hprobs[p], vbase[(size_t)p * 64 + comp + 1]);
  }
  const float o0 = (float)acc0, o1 = (float)acc1;
  const int qh_index = kh * kHeadsPerKv + h;
  *reinterpret_cast<float2*>(b.attn + (size_t)row * kHidden + qh_index * 64 + comp) =
      make_float2(o0, o1);
  check_finite(o0, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + comp);
  check_finite(o1, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + comp + 1);
}

}  // namespace

int attention_smem_positions() { return kAttnMaxPositions; }

void configure_scores_kernel() {
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    // 8 score CTAs of 18 KB per SM (the default carveout admits 6)
    cudaFuncSetAttribute(attention_scores_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attribute_done(configured);
  }
}

int launch_attention_grouped(const Batch& b, int layer, int span_cap, bool quantize, const float* rope,
                             cudaStream_t s) {
  const size_t bytes = PvSmem::bytes(span_cap);
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(attention_pv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)PvSmem::bytes(kAttnMaxPositions));
    cudaFuncSetAttribute(attention_pv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)PvSmem::bytes(kAttnMaxPositions));
    attribute_done(configured);
  }
  configure_scores_kernel();
  const int chunks = (span_cap + kChunk - 1) / kChunk;
  launch_pdl(attention_scores_kernel, dim3(chunks, b.rows * 2), kThreads, 0, s, b, layer, rope);
  if (b.kv_checked)
    launch_pdl(attention_pv_kernel<false>, b.rows * 2, kThreads, bytes, s, b, layer, span_cap, quantize);
  else
    launch_pdl(attention_pv_kernel<true>, b.rows * 2, kThreads, bytes, s, b, layer, span_cap, quantize);
  return 2;
}

// Component groups of the long-context PV launch (PB_ATTN_LONG_GROUPS=2|4|8
// in the environment selects one for tuning sweeps; tests cover each).
int attention_long_groups() {
  if (const char* f = std::getenv("PB_ATTN_LONG_GROUPS")) {
    const int g = std::atoi(f);
    if (g == 2 || g == 4 || g == 8) return g;
  }
  return 4;
}

template <int G>
static void launch_pv_long(const Batch& b, int layer, cudaStream_t s) {
  using C = PvLong<G>;
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(attention_pv_long_kernel<G, false>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kBytes);
    cudaFuncSetAttribute(attention_pv_long_kernel<G, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kBytes);
    attribute_done(configured);
  }
  const dim3 grid(b.rows * 2, G);
  if (b.kv_checked)
    launch_pdl(attention_pv_long_kernel<G, false>, grid, C::kThreads, C::kBytes, s, b, layer);
  else
    launch_pdl(attention_pv_long_kernel<G, true>, grid, C::kThreads, C::kBytes, s, b, layer);
}

int launch_attention_long(const Batch& b, int layer, int span_cap, bool quantize, const float* rope,
                          cudaStream_t s) {
  configure_scores_kernel();
  const int chunks = (span_cap + kChunk - 1) / kChunk;
  launch_pdl(attention_scores_kernel, dim3(chunks, b.rows * 2), kThreads, 0, s, b, layer, rope);
  launch_pdl(attention_softmax_long_kernel, b.rows * kQHeads, kLongThreads, 0, s, b);
  const int groups = attention_long_groups();
  if (groups == 2) launch_pv_long<2>(b, layer, s);
  else if (groups == 8) launch_pv_long<8>(b, layer, s);
  else launch_pv_long<4>(b, layer, s);
  if (quantize) {
    launch_quant(b, b.attn, kHidden, kHidden, s);
    return 4;
  }
  return 3;
}

}  // namespace pb
