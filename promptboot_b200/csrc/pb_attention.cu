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
// Every launch serves the 7 query heads of one KV head together.
//  * attention_scores4_kernel: one CTA per (sequence, KV head, 128-position
//    chunk), 224 threads = one warp per query head, so thousands of small CTAs
//    keep every SM busy while K streams in.  K arrives in the reference's
//    4-position tiles ([component][4 positions], 1 KB) and is copied
//    untransposed by cp.async into tiles padded to 260 words; lane l of a warp
//    takes tile l, one 16-byte shared load per component serving 4 products,
//    and keeps 4 f64 chains (two converting their products on the XU pipe, two
//    summing integer-built images, scaled_image).  Scores go to the global
//    score scratch (L2-resident).  With the RoPE table given, every CTA
//    rotates q for its 7 heads and the CTA of the last chunk also rotates k and
//    writes this step's K and V (decode steps, where no two rows share a slot).
//  * up to kAttnMaxPositions, attention_pv_kernel: one CTA per (sequence, KV
//    head), one warp per query head; the softmax of each head runs in its warp
//    from the scores copied into shared memory, then V streams through two
//    64-row buffers while every lane keeps two f64 chains (components 2 lane
//    and 2 lane + 1, one 8-byte load per position, positions in order); the
//    second chain adds integer-built f64 images of its products instead of
//    converting them (scaled_product).
//  * beyond that, the probabilities stay in the global scratch: the softmax
//    launch and the one-chain-per-thread PV launch below (up to 8 rows the
//    chains are fed their f64 terms by producer warps, attention_pv_fed_kernel).
#include "pb_common.cuh"
#include "pb_kernels.cuh"
#include "pb_quant.cuh"

#include <cstdlib>
#include <cstring>

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

// f64 image of p * 2^-896 for a finite binary32 p (the conversion-free half
// of scaled_product).
__device__ __forceinline__ double scaled_image(float p) {
  double d;
  asm("{\n\t.reg .b32 hi, lo;\n\t"
      "shr.s32 hi, %1, 3;\n\t"
      "and.b32 hi, hi, 0x8FFFFFFF;\n\t"
      "shl.b32 lo, %1, 29;\n\t"
      "mov.b64 %0, {lo, hi};\n\t}"
      : "=d"(d) : "r"(__float_as_uint(p)));
  return d;
}

struct PvSmem {
  static constexpr int kVBuf = kChunk * 64;  // V rows
  static size_t bytes(int span_cap) { return (size_t)(2 * kVBuf + kHeadsPerKv * span_cap) * 4; }
};

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
      // the products and their f64 images first, then the two dependent add
      // chains
      double t0[4], t1[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v2 = *reinterpret_cast<const float2*>(vt + (i + j) * 64);
        t0[j] = (double)__fmul_rn(pv[j], v2.x);
        t1[j] = scaled_product(pv[j], v2.y);
        if (kCheckV) vchk = __fmaf_rn(v2.y, 0.0f, vchk);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc0 += t0[j];
        acc1 += t1[j];
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
// The scores come from attention_scores4_kernel as above; then
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
//  * attention_pv_chains_kernel<G> (below): one f64 chain per thread over all
//    positions, every V word read once per KV head.

constexpr int kLongThreads = 256;
constexpr int kLongBatch = 4;  // groups loaded per thread before use
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

  // Every pass loads kLongBatch groups per thread before using them, so each
  // CTA keeps 16 KB of L2 reads in flight instead of one round trip per group.
  float m = fbits(0xff800000u);
  for (int i0 = tid; i0 < groups; i0 += kLongBatch * kLongThreads) {
    float4 sb[kLongBatch];
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int i = i0 + k * kLongThreads;
      if (i < groups) sb[k] = sc4[i];
    }
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int p = 4 * (i0 + k * kLongThreads);
      if (p < positions) m = fmaxf(m, sb[k].x);
      if (p + 1 < positions) m = fmaxf(m, sb[k].y);
      if (p + 2 < positions) m = fmaxf(m, sb[k].z);
      if (p + 3 < positions) m = fmaxf(m, sb[k].w);
    }
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
  for (int i0 = tid; i0 < groups; i0 += kLongBatch * kLongThreads) {
    float4 sb[kLongBatch];
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int i = i0 + k * kLongThreads;
      if (i < groups) sb[k] = sc4[i];
    }
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int i = i0 + k * kLongThreads;
      if (i >= groups) break;
      const float4 s = sb[k];
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
  for (int i0 = tid; i0 < groups; i0 += kLongBatch * kLongThreads) {
    float4 eb[kLongBatch];
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int i = i0 + k * kLongThreads;
      if (i < groups) eb[k] = sc4[i];
    }
#pragma unroll
    for (int k = 0; k < kLongBatch; ++k) {
      const int i = i0 + k * kLongThreads;
      if (i >= groups) break;
      float4 e = eb[k];
      const int p = 4 * i;
      if (p < positions) e.x = __fmul_rn(e.x, normalizer);
      if (p + 1 < positions) e.y = __fmul_rn(e.y, normalizer);
      if (p + 2 < positions) e.z = __fmul_rn(e.z, normalizer);
      if (p + 3 < positions) e.w = __fmul_rn(e.w, normalizer);
      sc4[i] = e;
      if (probs) probs[i] = e;
    }
  }
}

// The PV chains over probabilities in the global score scratch.  A CTA serves
// one (sequence, KV head, one of G component groups); thread (head h,
// component c) owns ONE f64 chain over all positions in order.  The chain sums
// integer-built images of its products (scaled_image; converting them on the
// XU pipe measured no faster), with the exact conversion fallback of
// attention_pv_kernel when a probability or a V word is not finite.  V rows of
// the group (transposed in shared memory) and the 7 heads' probabilities
// stream through kStages cp.async buffers.  Each position costs a thread about
// nine instructions, and one warp alone on its scheduler issues them at ~2.5
// cycles each: ~22 cycles per position per chain, against the 8.2-cycle
// latency of the dependent f64 add that bounds any order-preserving chain.
// More CTAs (G 8, 16) do not help: the time is one thread's chain, and the
// 7 x 64 chains of a KV head run in parallel already.
template <int G>
struct PvChains {
  static constexpr int kComps = 64 / G;                            // components per CTA
  static constexpr int kWorkers = kHeadsPerKv * kComps;            // one chain each
  static constexpr int kThreads = (kWorkers + 31) / 32 * 32;
  static constexpr int kChunk = 128;                               // positions per stage
  static constexpr int kStages = 4;
  // V of a stage is component-major, [component][kVPitch positions], so a
  // thread reads four positions of its component with one 16-byte load; the
  // pitch's 4 extra words put the 8 components of a quarter-warp on distinct
  // banks.
  static constexpr int kVPitch = kChunk + 4;
  static constexpr int kVWords = kComps * kVPitch;
  static constexpr int kPWords = kHeadsPerKv * kChunk;
  static constexpr int kStage = kVWords + kPWords;
  static constexpr size_t kBytes = (size_t)kStages * kStage * 4;
};

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

template <int G, bool kScaled, bool kCheckV>
__global__ void __launch_bounds__(PvChains<G>::kThreads)
attention_pv_chains_kernel(Batch b, int layer, bool quantize) {
  using C = PvChains<G>;
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  const int row = blockIdx.x >> 1, kh = blockIdx.x & 1, grp = blockIdx.y;
  const int tid = threadIdx.x;
  const int h = tid / C::kComps, cc = tid % C::kComps;
  const bool active = tid < C::kWorkers;
  const int comp = grp * C::kComps + cc;
  const int positions = b.positions[row] + 1;
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* vbase = kv + (size_t)layer * 4 * cap * 64 + 2 * cap * 64 + (size_t)kh * cap * 64;
  const float* probs = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv) * b.score_stride;
  const int nchunks = (positions + C::kChunk - 1) / C::kChunk;

  auto load = [&](int t) {
    if (t < nchunks) {
      float* stage = sm + (t % C::kStages) * C::kStage;
      const int p0 = t * C::kChunk;
      const int rows_here = min(C::kChunk, positions - p0);
      // V words one by one into the transposed layout (consecutive threads
      // read consecutive components of a position: 32-byte global segments)
      for (int i = tid; i < rows_here * C::kComps; i += C::kThreads) {
        const int r = i / C::kComps, c = i % C::kComps;
        cp_async4(stage + c * C::kVPitch + r, vbase + (size_t)(p0 + r) * 64 + grp * C::kComps + c);
      }
      // probabilities of the 7 heads, rows_here rounded up to 4 (the scratch
      // holds the padded span)
      const int quads = (rows_here + 3) >> 2;
      float* pst = stage + C::kVWords;
      for (int i = tid; i < kHeadsPerKv * quads; i += C::kThreads) {
        const int hh = i / quads, q = i % quads;
        cp_async16(pst + hh * C::kChunk + 4 * q, probs + (size_t)hh * b.score_stride + p0 + 4 * q);
      }
    }
    cp_commit();  // one group per chunk slot, empty past the end
  };
#pragma unroll
  for (int t = 0; t < C::kStages - 1; ++t) load(t);

  double acc = 0.0;
  float vchk = 0.0f;
  for (int t = 0; t < nchunks; ++t) {
    load(t + C::kStages - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(C::kStages - 1) : "memory");
    __syncthreads();
    const float* stage = sm + (t % C::kStages) * C::kStage;
    const float* vt = stage + cc * C::kVPitch;
    const float* pr = stage + C::kVWords + h * C::kChunk;
    const int rows_here = min(C::kChunk, positions - t * C::kChunk);
    if (active) {
      // Software pipeline over batches of 8 positions: the raw probabilities
      // and V words of the next batch are loaded before the current batch, and
      // each dependent add of the current batch is followed by the product and
      // conversion of the matching next-batch position, so the add chain never
      // waits behind a load or a conversion.
      const int full = rows_here & ~7;
      if (full > 0) {
        float pc[8], vc[8];
        auto fetch = [&](int i, float (&pp)[8], float (&vv)[8]) {
          const float4 pa = *reinterpret_cast<const float4*>(pr + i);
          const float4 pb = *reinterpret_cast<const float4*>(pr + i + 4);
          pp[0] = pa.x; pp[1] = pa.y; pp[2] = pa.z; pp[3] = pa.w;
          pp[4] = pb.x; pp[5] = pb.y; pp[6] = pb.z; pp[7] = pb.w;
          const float4 va = *reinterpret_cast<const float4*>(vt + i);
          const float4 vb = *reinterpret_cast<const float4*>(vt + i + 4);
          vv[0] = va.x; vv[1] = va.y; vv[2] = va.z; vv[3] = va.w;
          vv[4] = vb.x; vv[5] = vb.y; vv[6] = vb.z; vv[7] = vb.w;
        };
        auto term = [&](float pk, float vk) {
          if (kCheckV) vchk = __fmaf_rn(vk, 0.0f, vchk);
          const float prod = __fmul_rn(pk, vk);
          return kScaled ? scaled_image(prod) : (double)prod;
        };
        fetch(0, pc, vc);
        double cur[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = term(pc[k], vc[k]);
        for (int i = 8; i < full; i += 8) {
          fetch(i, pc, vc);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            acc += cur[k];
            cur[k] = term(pc[k], vc[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) acc += cur[k];
      }
      for (int i = full; i < rows_here; ++i) {
        const float v = vt[i];
        if (kCheckV) vchk = __fmaf_rn(v, 0.0f, vchk);
        const float prod = __fmul_rn(pr[i], v);
        acc += kScaled ? scaled_image(prod) : (double)prod;
      }
    }
    __syncthreads();  // the slot is refilled by the next iteration's load
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (!active) return;
  if (kScaled) {
    // The scaled images need finite products: finite probabilities (a finite
    // normalizer; a non-finite one shows in every probability word, position
    // 0's included) and finite V (the v-projection check, or vchk here);
    // otherwise the chain is redone with conversions.
    const float* hprobs = probs + (size_t)h * b.score_stride;
    if (fabsf(hprobs[0]) <= 0x1.fffffep127f && vchk == 0.0f) {
      acc *= 0x1p896;
    } else {
      acc = 0.0;
      for (int p = 0; p < positions; ++p)
        acc += (double)__fmul_rn(hprobs[p], vbase[(size_t)p * 64 + comp]);
    }
  }
  const float o = (float)acc;
  const int qh_index = kh * kHeadsPerKv + h;
  b.attn[(size_t)row * kHidden + qh_index * 64 + comp] = o;
  check_finite(o, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + comp);
  // Two groups: warp h holds the 32 outputs of Q8_0 block 2 qh + grp of the
  // o-projection input, element = lane.
  if (G == 2 && quantize) quantize_row_block(b, o, row, 2 * qh_index + grp);
}

// The PV chains for few rows, fed by producer warps.  With at most 8 rows the
// chains of a step fill at most 128 CTAs of two chain warps, one warp per
// scheduler, and a chain thread that also forms its products (multiply, three
// integer operations for the scaled image, the loads) issues ~22 cycles per
// position against the 8.2-cycle dependent add.  Here the CTA of (sequence, KV
// head, one of 8 component groups) holds 2 chain warps (the 56 chains: 7 heads
// x 8 components) and 8 producer warps (four per chain, a quarter of each
// chunk each), one CTA per SM: the producers stream V (transposed) and the
// probabilities through kStages
// cp.async stages and write the scaled f64 images of the products of chunk
// t + 1 into a shared term buffer ([position pair][chain] double2) while the
// chain warps add chunk t's terms in position order, two 16-byte loads per
// four adds.  One barrier per chunk separates the two buffers' roles.
struct PvFed {
  static constexpr int kComps = 8;                          // components per CTA
  static constexpr int kGroups = 64 / kComps;               // grid.y
  static constexpr int kChains = kHeadsPerKv * kComps;      // 56
  static constexpr int kSlots = 64;                         // term row pitch (double2)
  static constexpr int kChainThreads = kSlots;              // warps 0-1
  static constexpr int kParts = 4;                          // producers per chain
  static constexpr int kProducers = kParts * kSlots;        // (slot, quarter chunk)
  static constexpr int kThreads = kChainThreads + kProducers;  // 320
  static constexpr int kChunk = 128;                        // positions per stage
  static constexpr int kPartQuads = kChunk / 4 / kParts;    // 4-position quads per producer
  static constexpr int kPitch = kChunk + 4;                 // words per V / probability row
  static constexpr int kStages = 4;                         // raw cp.async stages
  static constexpr int kRawWords = (kComps + kHeadsPerKv) * kPitch;
  static constexpr int kTermPairs = kChunk / 2;
  static constexpr int kTermStage = kTermPairs * kSlots;    // double2 per term buffer
  static constexpr size_t kBytes = 2 * (size_t)kTermStage * 16 + (size_t)kStages * kRawWords * 4;
};
static_assert(PvFed::kRawWords * 4 % 16 == 0 && PvFed::kComps * PvFed::kPitch * 4 % 16 == 0,
              "16-byte cp.async destinations");

template <bool kCheckV>
__global__ void __launch_bounds__(PvFed::kThreads, 1)
attention_pv_fed_kernel(Batch b, int layer) {
  using C = PvFed;
  pdl_begin();
  extern __shared__ __align__(16) float sm[];
  __shared__ int s_bad;
  double2* terms = reinterpret_cast<double2*>(sm);
  float* raw = sm + 2 * C::kTermStage * 4;
  const int row = blockIdx.x >> 1, kh = blockIdx.x & 1, grp = blockIdx.y;
  const int tid = threadIdx.x;
  const bool producer = tid >= C::kChainThreads;
  const int pt = tid - C::kChainThreads;                      // producer index
  const int slot = producer ? (pt & (C::kSlots - 1)) : tid;   // chain of this thread
  const int part = producer ? pt / C::kSlots : 0;
  const bool active = slot < C::kChains;
  const int h = slot / C::kComps, cc = slot % C::kComps;
  const int comp = grp * C::kComps + cc;
  const int positions = b.positions[row] + 1;
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* vbase = kv + (size_t)layer * 4 * cap * 64 + 2 * cap * 64 + (size_t)kh * cap * 64;
  const float* probs = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv) * b.score_stride;
  const int nchunks = (positions + C::kChunk - 1) / C::kChunk;

  auto load = [&](int t) {  // producers: chunk t into raw stage t % kStages
    if (t < nchunks) {
      float* stage = raw + (t % C::kStages) * C::kRawWords;
      const int p0 = t * C::kChunk;
      const int rows_here = min(C::kChunk, positions - p0);
      const float* vsrc = vbase + (size_t)p0 * 64 + grp * C::kComps;
      for (int i = pt; i < rows_here * C::kComps; i += C::kProducers) {
        const int r = i / C::kComps, c = i % C::kComps;
        cp_async4(stage + c * C::kPitch + r, vsrc + r * 64 + c);
      }
      // probabilities of the 7 heads, rows_here rounded up to 4 (the scratch
      // holds the padded span)
      const int quads = (rows_here + 3) >> 2;
      float* pst = stage + C::kComps * C::kPitch;
      for (int i = pt; i < kHeadsPerKv * (C::kChunk / 4); i += C::kProducers) {
        const int hh = i / (C::kChunk / 4), q = i % (C::kChunk / 4);
        if (q < quads)
          cp_async16(pst + hh * C::kPitch + 4 * q, probs + (size_t)hh * b.score_stride + p0 + 4 * q);
      }
    }
    cp_commit();  // one group per chunk, empty past the end
  };
  float vchk = 0.0f;
  // The low and high words of the scaled f64 image of fl(p * v) (the
  // arithmetic of scaled_image, written out so the words go straight into the
  // registers of a 16-byte store).
  auto image = [](float p, float v, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = __float_as_uint(__fmul_rn(p, v));
    hi = (uint32_t)((int32_t)u >> 3) & 0x8FFFFFFFu;
    lo = u << 29;
  };
  // One quad of positions: the terms of pairs dst[0] and dst[kSlots]; `valid`
  // of its positions are below rows_here (the V check covers only those).
  auto quad = [&](uint4* dst, const float* pq, const float* vq, int valid) {
    const float4 p4 = *reinterpret_cast<const float4*>(pq);
    const float4 v4 = *reinterpret_cast<const float4*>(vq);
    if (kCheckV) {
      vchk = __fmaf_rn(v4.x, 0.0f, vchk);
      if (valid > 1) vchk = __fmaf_rn(v4.y, 0.0f, vchk);
      if (valid > 2) vchk = __fmaf_rn(v4.z, 0.0f, vchk);
      if (valid > 3) vchk = __fmaf_rn(v4.w, 0.0f, vchk);
    }
    uint4 w0, w1;
    image(p4.x, v4.x, w0.x, w0.y);
    image(p4.y, v4.y, w0.z, w0.w);
    image(p4.z, v4.z, w1.x, w1.y);
    image(p4.w, v4.w, w1.z, w1.w);
    dst[0] = w0;
    dst[C::kSlots] = w1;
  };
  auto produce = [&](int t) {  // producers: the images of chunk t's products
    if (!active) return;
    const float* stage = raw + (t % C::kStages) * C::kRawWords;
    const int i0 = part * (4 * C::kPartQuads);
    const float* vt = stage + cc * C::kPitch + i0;
    const float* pr = stage + C::kComps * C::kPitch + h * C::kPitch + i0;
    uint4* term = reinterpret_cast<uint4*>(terms) + (t & 1) * C::kTermStage + slot +
                  (i0 >> 1) * C::kSlots;
    const int rows_here = min(C::kChunk, positions - t * C::kChunk);
    if (rows_here == C::kChunk) {
#pragma unroll
      for (int k = 0; k < C::kPartQuads; ++k)
        quad(term + 2 * k * C::kSlots, pr + 4 * k, vt + 4 * k, 4);
      return;
    }
    // The last chunk: a quad past rows_here reads stale words (the pitch covers
    // it); the chains never add those terms.
    for (int k = 0; k < C::kPartQuads && i0 + 4 * k < rows_here; ++k)
      quad(term + 2 * k * C::kSlots, pr + 4 * k, vt + 4 * k, rows_here - i0 - 4 * k);
  };
  double acc = 0.0;
  auto consume = [&](int t) {  // chain threads: chunk t's terms in position order
    const double2* term = terms + (t & 1) * C::kTermStage + slot;
    const int rows_here = min(C::kChunk, positions - t * C::kChunk);
    if (rows_here == C::kChunk) {
      // the next eight pairs load while the current eight are added
      double2 a[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] = term[k * C::kSlots];
#pragma unroll
      for (int g = 1; g < C::kTermPairs / 8; ++g) {
        double2 n[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) n[k] = term[(8 * g + k) * C::kSlots];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc += a[k].x;
          acc += a[k].y;
          a[k] = n[k];
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc += a[k].x;
        acc += a[k].y;
      }
      return;
    }
    const int pairs = rows_here >> 1;
    for (int j = 0; j < pairs; ++j) {
      const double2 a = term[j * C::kSlots];
      acc += a.x;
      acc += a.y;
    }
    if (rows_here & 1) acc += term[pairs * C::kSlots].x;
  };

  if (tid == 0) s_bad = 0;
  if (producer) {
    load(0);
    load(1);
    load(2);
    asm volatile("cp.async.wait_group 2;" ::: "memory");  // chunk 0 landed (own copies)
  }
  __syncthreads();
  if (producer) {
    produce(0);
    cp_wait1();  // chunk 1
  }
  __syncthreads();
  for (int t = 0; t < nchunks; ++t) {
    if (producer) {
      load(t + 3);  // into the stage chunk t - 1 held (read two barriers ago)
      if (t + 1 < nchunks) produce(t + 1);
      cp_wait1();   // chunk t + 2, for the next iteration
    } else if (active) {
      consume(t);
    }
    __syncthreads();
  }
  if (producer) {
    cp_wait0();
    if (kCheckV && vchk != 0.0f) s_bad = 1;
  }
  __syncthreads();
  if (producer || !active) return;
  // The images need finite products: finite probabilities (position 0's word
  // shows a non-finite normalizer) and finite V; otherwise the chain is redone
  // with conversions.
  const float* hprobs = probs + (size_t)h * b.score_stride;
  if (fabsf(hprobs[0]) <= 0x1.fffffep127f && s_bad == 0) {
    acc *= 0x1p896;
  } else {
    acc = 0.0;
    for (int p = 0; p < positions; ++p)
      acc += (double)__fmul_rn(hprobs[p], vbase[(size_t)p * 64 + comp]);
  }
  const float o = (float)acc;
  const int qh_index = kh * kHeadsPerKv + h;
  b.attn[(size_t)row * kHidden + qh_index * 64 + comp] = o;
  check_finite(o, &b.err[row], (uint32_t)layer + 1, D_ATTENTION, 0, qh_index * 64 + comp);
}

// Scores over chunks of 128 positions: lane l of warp h takes the 4-position K
// tile l, so one 16-byte shared load serves 4 products, and keeps 4 f64
// chains: positions 0-1 of the tile convert their products on the XU pipe,
// positions 2-3 sum integer-built images (scaled_image), redone with
// conversions when a product of theirs is not finite.  RoPE and this step's
// K/V write of this step's position when the RoPE table is given.
constexpr int kChunk4 = 128;

__global__ void __launch_bounds__(kThreads, 6)
attention_scores4_kernel(Batch b, int layer, const float* rope) {
  pdl_begin();
  __shared__ __align__(16) float qs[kHeadsPerKv * 64];
  extern __shared__ __align__(16) float ks[];  // [32 tiles][kTilePitch]

  const int t = blockIdx.x, row = blockIdx.y >> 1, kh = blockIdx.y & 1;
  const int tid = threadIdx.x, h = tid >> 5, lane = tid & 31;
  const int positions = b.positions[row] + 1;
  if (t * kChunk4 >= positions) return;
  const bool last = (t + 1) * kChunk4 >= positions;
  const size_t cap = b.capacity;
  const float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * cap * 64;
  const float* kbase = kv + (size_t)layer * 4 * cap * 64 + (size_t)kh * (cap / 4) * 256;

  const float* qg = b.q + (size_t)row * kHidden + kh * kHeadsPerKv * 64;
  if (rope) {
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

  // Chunk t = K tiles 32t .. 32t + 31, each 1 KB contiguous in the cache.
  {
    const int ntiles = (positions + 3) >> 2;
    const int tiles = min(kChunk4 / 4, ntiles - t * (kChunk4 / 4));
    const float* src = kbase + (size_t)t * (kChunk4 / 4) * 256;
    for (int i = tid; i < tiles * 64; i += kThreads)
      cp_async16(ks + (i >> 6) * kTilePitch + (i & 63) * 4, src + i * 4);
    cp_commit();
    cp_wait0();
  }
  __syncthreads();

  const int p = t * kChunk4 + 4 * lane;  // tile `lane`: positions p .. p + 3
  if (p >= positions) return;
  const float* qh = qs + h * 64;
  const float* kt = ks + lane * kTilePitch;
  double d0 = 0.0, d1 = 0.0, d2 = 0.0, d3 = 0.0;
  float fchk = 0.0f;
#pragma unroll 2
  for (int c = 0; c < 64; c += 4) {
    const float4 q4 = *reinterpret_cast<const float4*>(qh + c);
    const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
    // the 16 products and their f64 images first, then the four add chains
    double t[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = *reinterpret_cast<const float4*>(kt + (c + j) * 4);
      t[j][0] = (double)__fmul_rn(qv[j], k4.x);
      t[j][1] = (double)__fmul_rn(qv[j], k4.y);
      const float p2 = __fmul_rn(qv[j], k4.z), p3 = __fmul_rn(qv[j], k4.w);
      fchk = __fmaf_rn(p2, 0.0f, fchk);
      fchk = __fmaf_rn(p3, 0.0f, fchk);
      t[j][2] = scaled_image(p2);
      t[j][3] = scaled_image(p3);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      d0 += t[j][0];
      d1 += t[j][1];
      d2 += t[j][2];
      d3 += t[j][3];
    }
  }
  if (fchk == 0.0f) {
    d2 *= 0x1p896;
    d3 *= 0x1p896;
  } else {
    d2 = d3 = 0.0;
    for (int c = 0; c < 64; ++c) {
      const float4 k4 = *reinterpret_cast<const float4*>(kt + c * 4);
      d2 += (double)__fmul_rn(qh[c], k4.z);
      d3 += (double)__fmul_rn(qh[c], k4.w);
    }
  }
  float* out = b.scores + ((size_t)row * kQHeads + kh * kHeadsPerKv + h) * b.score_stride;
  *reinterpret_cast<float4*>(out + p) =
      make_float4(__fmul_rn((float)d0, 0.125f), __fmul_rn((float)d1, 0.125f),
                  __fmul_rn((float)d2, 0.125f), __fmul_rn((float)d3, 0.125f));
}

constexpr size_t kScores4Smem = (size_t)(kChunk4 / 4) * kTilePitch * 4;

}  // namespace

int attention_smem_positions() { return kAttnMaxPositions; }

template <int G, bool kScaled, bool kCheckV>
static void launch_pv_chains_as(const Batch& b, int layer, bool quantize, cudaStream_t s) {
  using C = PvChains<G>;
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(attention_pv_chains_kernel<G, kScaled, kCheckV>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kBytes);
    attribute_done(configured);
  }
  launch_pdl(attention_pv_chains_kernel<G, kScaled, kCheckV>, dim3(b.rows * 2, G), C::kThreads,
             C::kBytes, s, b, layer, quantize);
}

template <int G>
static void launch_pv_chains(const Batch& b, int layer, bool quantize, cudaStream_t s) {
  if (b.kv_checked) launch_pv_chains_as<G, true, false>(b, layer, quantize, s);
  else launch_pv_chains_as<G, true, true>(b, layer, quantize, s);
}

static void configure_scores4() {
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(attention_scores4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kScores4Smem);
    cudaFuncSetAttribute(attention_scores4_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
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
  configure_scores4();
  const int chunks = (span_cap + kChunk4 - 1) / kChunk4;
  launch_pdl(attention_scores4_kernel, dim3(chunks, b.rows * 2), kThreads, kScores4Smem, s, b, layer,
             rope);
  if (b.kv_checked)
    launch_pdl(attention_pv_kernel<false>, b.rows * 2, kThreads, bytes, s, b, layer, span_cap, quantize);
  else
    launch_pdl(attention_pv_kernel<true>, b.rows * 2, kThreads, bytes, s, b, layer, span_cap, quantize);
  return 2;
}

template <bool kCheckV>
static void launch_pv_fed_as(const Batch& b, int layer, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(attention_pv_fed_kernel<kCheckV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)PvFed::kBytes);
    attribute_done(configured);
  }
  launch_pdl(attention_pv_fed_kernel<kCheckV>, dim3(b.rows * 2, PvFed::kGroups), PvFed::kThreads,
             PvFed::kBytes, s, b, layer);
}

// Rows up to which the split PV launch is the producer-fed one (one CTA per SM
// at most; more CTAs share the shared-memory bandwidth that the term buffer
// already uses at ~8 bytes a cycle per chain).
constexpr int kPvFedRows = 8;

// The split PV launch: the producer-fed chains (returned as 0) up to
// kPvFedRows rows; from 16 rows two component groups (224 threads, warp =
// query head, the launch then quantizes its own output for the o projection:
// 32 rows 13.3k against 12.6k tok/s per step); four between.
// PB_ATTN_LONG_GROUPS=fed|2|4|8|16 in the environment selects one for tuning
// sweeps; tests cover each.
int attention_long_groups(int rows) {
  if (const char* f = std::getenv("PB_ATTN_LONG_GROUPS")) {
    if (std::strcmp(f, "fed") == 0) return 0;
    const int g = std::atoi(f);
    if (g == 2 || g == 4 || g == 8 || g == 16) return g;
  }
  return rows <= kPvFedRows ? 0 : rows >= 16 ? 2 : 4;
}

int launch_attention_long(const Batch& b, int layer, int span_cap, bool quantize, const float* rope,
                          cudaStream_t s) {
  configure_scores4();
  const int chunks = (span_cap + kChunk4 - 1) / kChunk4;
  launch_pdl(attention_scores4_kernel, dim3(chunks, b.rows * 2), kThreads, kScores4Smem, s, b, layer,
             rope);
  launch_pdl(attention_softmax_long_kernel, b.rows * kQHeads, kLongThreads, 0, s, b);
  const int groups = attention_long_groups(b.rows);
  if (groups == 2) {
    // the PV launch quantizes its own output
    launch_pv_chains<2>(b, layer, quantize, s);
    return 3;
  }
  if (groups == 0) {
    if (b.kv_checked) launch_pv_fed_as<false>(b, layer, s);
    else launch_pv_fed_as<true>(b, layer, s);
  } else if (groups == 4) launch_pv_chains<4>(b, layer, false, s);
  else if (groups == 16) launch_pv_chains<16>(b, layer, false, s);
  else launch_pv_chains<8>(b, layer, false, s);
  if (quantize) {
    launch_quant(b, b.attn, kHidden, kHidden, s);
    return 4;
  }
  return 3;
}

}  // namespace pb
