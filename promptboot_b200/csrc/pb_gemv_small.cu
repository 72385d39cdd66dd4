// Small-batch (B <= 8 rows) block-scaled matvec for sm_100a, with the layer's
// neighbouring elementwise stages fused in:
//   y[s][r] = sum over Q-blocks k, IN ORDER, of the reference's block term
//     Q4_0: fl(fl(f32(i) * dW) * dA)   (fp32_sse2.rs:1217-1248)
//     Q8_0: fl(f32(i) * fl(dW * dA))   (fp32_sse2.rs:1250-1281)
//   with i the exact int32 block dot (dp4a; Q4_0 nibbles enter unsigned and the
//   zero point leaves as -8 * sum(a)).
//
// One CTA owns a slice of rows of up to three stacked matrices (q/k/v) or the
// same rows of a gate/up pair.  Its weight slice is one contiguous run of
// PBTQW25 rows per matrix, fetched into shared memory by cp.async.bulk BEFORE
// the programmatic-dependency wait, so the weight stream of this launch
// overlaps the previous kernel.  After the wait:
//   prologue  the B rows' Q8_0 activations into shared memory: read from the
//             row-major buffers, or computed from the residual stream as
//             RMSNorm (fp32_sse2.rs:1310-1334) + quantizer (fp32_sse2.rs:
//             945-983), every CTA repeating that small exact computation
//             instead of a separate launch;
//   phase 1   every (row, block) item: the B block dots and terms into shared
//             memory;
//   phase 2   every (sequence, row): the binary32 sum in block order, then the
//             epilogue (bias, residual, store) or, for gate/up, SwiGLU
//             (fp32_sse2.rs:1751-1770) and the Q8_0 quantization of the product
//             for the down projection.
// Stage checks (inference.rs:1889-1936) land in the rows' ranked error words.
#include "pb_common.cuh"
#include "pb_kernels.cuh"
#include "pb_quant.cuh"

#include <algorithm>

namespace pb {
namespace {

constexpr int kSgThreads = 256;

__device__ __forceinline__ uint32_t sg_smem(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t sg_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_u32_2aligned_s(const uint8_t* p) {
  const uint32_t lo = *reinterpret_cast<const uint16_t*>(p);
  const uint32_t hi = *reinterpret_cast<const uint16_t*>(p + 2);
  return lo | (hi << 16);
}

// Q8_0 quantization of one 32-element block by one thread (fp32_sse2.rs:945-983):
// the same operations as quantize_lane, serially; y holds the block's values.
__device__ __forceinline__ void quantize_block_serial(const float* y, int8_t* aq, float* ad,
                                                      int* asum) {
  float amax = fabsf(y[0]);
#pragma unroll 8
  for (int j = 1; j < 32; ++j) amax = fmaxf(amax, fabsf(y[j]));
  const float d = __fdiv_rn(amax, 127.0f);
  const float inverse = bitsf(d) == 0 ? 0.0f : __fdiv_rn(1.0f, d);
  int total = 0;
  uint32_t word = 0;
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const float v = __fmul_rn(y[j], inverse);
    const float half = (bitsf(v) >> 31) == 0 ? 0.5f : -0.5f;
    const float t = __fadd_rn(v, half);
    const int q = fabsf(t) < 2147483648.0f ? __float2int_rz(t) : (int)0x80000000u;
    total += (int)(int8_t)q;
    word |= (uint32_t)(uint8_t)q << (8 * (j & 3));
    if ((j & 3) == 3) {
      reinterpret_cast<uint32_t*>(aq)[j >> 2] = word;
      word = 0;
    }
  }
  *ad = __half2float(__float2half_rn(d));
  *asum = total;
}

// RMSNorm (fp32_sse2.rs:1310-1334) of one row x (shared memory) by one warp into
// y (block-major, 33 words per 32-element block): the 896 f64 squares summed as a tree when the
// exponent span proves it equal to the serial sum (rmsnorm_quant_kernel), else
// serially by lane 0.
__device__ void norm_row_warp(const float* __restrict__ x, const float* __restrict__ w, float* y,
                              unsigned long long* err, uint32_t ordinal, uint32_t domain) {
  const int lane = threadIdx.x & 31;
  double sum = 0.0;
  int emin = 255, emax = 0;
  for (int e = lane; e < kHidden; e += 32) {
    const float q = __fmul_rn(x[e], x[e]);
    sum += (double)q;
    const uint32_t qb = bitsf(q) & 0x7fffffffu;
    const int ex = (int)(qb >> 23);
    if (qb != 0) {
      emin = min(emin, max(ex, 1));
      emax = max(emax, max(ex, 1));
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    emin = min(emin, __shfl_xor_sync(0xffffffffu, emin, o));
    emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
  }
  if (emax == 255 || (emax >= emin && emax - emin > 19)) {
    double serial = 0.0;
    if (lane == 0)
      for (int e = 0; e < kHidden; ++e) serial += (double)__fmul_rn(x[e], x[e]);
    sum = __shfl_sync(0xffffffffu, serial, 0);
  }
  const float mean = (float)(sum / 896.0);
  const float inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, fbits(0x358637bdu))));
  for (int e = lane; e < kHidden; e += 32) {
    const float v = __fmul_rn(__fmul_rn(x[e], inverse), w[e]);
    check_finite(v, err, ordinal, domain, 0, e);
    y[(e >> 5) * 33 + (e & 31)] = v;
  }
}

template <int BPB>
__global__ void __launch_bounds__(kSgThreads)
small_gemv_kernel(SmallGemv g, Batch b, unsigned int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = g.cols / 32;
  const size_t row_bytes = (size_t)nb * BPB;
  const int B = b.rows;
  const int mats = g.swiglu ? 2 : 1;
  const int rows_cta = g.rt * mats;          // weight rows held by this CTA
  const int r0 = blockIdx.x * g.rt;          // first launch row (per matrix in SwiGLU mode)

  // shared memory: [barrier 16 B][weights][activations][terms]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint8_t* ws = smem + 16;
  const size_t wbytes = ((size_t)rows_cta * row_bytes + 15) & ~(size_t)15;
  int8_t* aq_s = reinterpret_cast<int8_t*>(ws + wbytes);
  float* ad_s = reinterpret_cast<float*>(aq_s + (size_t)B * g.cols);
  int* asum_s = reinterpret_cast<int*>(ad_s + B * nb);
  float* terms = reinterpret_cast<float*>(asum_s + B * nb);
  const int tstride = nb + 1;

  // ---- weight slice: one bulk copy per matrix piece, before the dependency wait
  int si = 0;
  while (si + 1 < g.nseg && r0 >= g.seg[si].rows_end) ++si;
  const int seg_begin = si ? g.seg[si - 1].rows_end : 0;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sg_smem(bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();  // the barrier is initialized before anyone polls it
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(g.rt * row_bytes);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sg_smem(bar)),
                 "r"(bytes * (uint32_t)mats)
                 : "memory");
    for (int m = 0; m < mats; ++m) {
      const uint8_t* src = g.swiglu ? g.seg[m].w + (size_t)r0 * row_bytes
                                    : g.seg[si].w + (size_t)(r0 - seg_begin) * row_bytes;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              sg_smem(ws + (size_t)m * g.rt * row_bytes)),
          "l"(src), "r"(bytes), "r"(sg_smem(bar))
          : "memory");
    }
  }
  pdl_wait();

  // ---- the B rows' Q8_0 activations into shared memory
  if (g.norm_weight) {
    // The B rows and the norm weight staged into shared memory with every
    // load in flight at once, RMSNorm of each row (a warp per row) into the
    // term buffer, then one thread per (row, block) quantizes.
    float* ys = terms;
    float* xs = ys + B * (kHidden / 32) * 33;
    float* wsm = xs + B * kHidden;
    for (int i = tid; i < B * (kHidden / 4); i += kSgThreads) {
      const int s = i / (kHidden / 4), c = i % (kHidden / 4);
      reinterpret_cast<float4*>(xs + s * kHidden)[c] =
          reinterpret_cast<const float4*>(b.hidden + (size_t)s * kHidden)[c];
    }
    for (int i = tid; i < kHidden / 4; i += kSgThreads)
      reinterpret_cast<float4*>(wsm)[i] = reinterpret_cast<const float4*>(g.norm_weight)[i];
    __syncthreads();
    for (int s = warp; s < B; s += kSgThreads / 32)
      norm_row_warp(xs + s * kHidden, wsm, ys + s * (kHidden / 32) * 33, &b.err[s], g.norm_ordinal,
                    g.norm_domain);
    __syncthreads();
    for (int i = tid; i < B * nb; i += kSgThreads) {
      const int s = i / nb, k = i % nb;
      quantize_block_serial(ys + (s * nb + k) * 33, aq_s + (size_t)s * g.cols + k * 32,
                            ad_s + i, asum_s + i);
    }
  } else {
    const int chunks = g.cols / 16;
    for (int i = tid; i < B * chunks; i += kSgThreads) {
      const int s = i / chunks, c = i % chunks;
      reinterpret_cast<uint4*>(aq_s + (size_t)s * g.cols)[c] =
          reinterpret_cast<const uint4*>(b.aq + (size_t)s * kActStride)[c];
    }
    for (int i = tid; i < B * nb; i += kSgThreads) {
      const int s = i / nb, k = i % nb;
      ad_s[i] = b.ad[(size_t)s * kActBlocks + k];
      asum_s[i] = b.asum[(size_t)s * kActBlocks + k];
    }
  }
  // the weight slice has landed (bounded wait: 200 ms, then report and skip)
  bool landed = true;
  {
    uint32_t ok = 0;
    const uint64_t deadline = sg_ns() + 200000000ull;
    for (;;) {
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0, 20000;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(sg_smem(bar))
          : "memory");
      if (ok) break;
      if (sg_ns() > deadline) {
        landed = false;
        break;
      }
    }
  }
  __syncthreads();
  if (!__syncthreads_and(landed)) {
    if (tid == 0) atomicOr(status, 1u);
    // let the copy finish before the CTA's shared memory goes away
    const uint64_t deadline = sg_ns() + 50000000ull;
    uint32_t ok = 0;
    while (!ok && sg_ns() < deadline)
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(ok)
          : "r"(sg_smem(bar))
          : "memory");
    return;
  }

  // ---- phase 1: block dots and terms of every (row, block)
  for (int item = tid; item < rows_cta * nb; item += kSgThreads) {
    const int r = item / nb, blk = item - r * nb;
    const uint8_t* bp = ws + (size_t)r * row_bytes + (size_t)blk * BPB;
    const float dW = half_to_f32(*reinterpret_cast<const uint16_t*>(bp));
    uint32_t wq[8];
    if (BPB == 18) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t p = ld_u32_2aligned_s(bp + 2 + 4 * j);
        wq[j] = p & 0x0f0f0f0fu;
        wq[4 + j] = (p >> 4) & 0x0f0f0f0fu;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wq[j] = ld_u32_2aligned_s(bp + 2 + 4 * j);
    }
    for (int s = 0; s < B; ++s) {
      const uint4* ap = reinterpret_cast<const uint4*>(aq_s + (size_t)s * g.cols + blk * 32);
      const uint4 a0 = ap[0], a1 = ap[1];
      const int aw[8] = {(int)a0.x, (int)a0.y, (int)a0.z, (int)a0.w,
                         (int)a1.x, (int)a1.y, (int)a1.z, (int)a1.w};
      int dot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) dot = __dp4a((int)wq[j], aw[j], dot);
      const float dA = ad_s[s * nb + blk];
      float term;
      if (BPB == 18) {
        dot -= 8 * asum_s[s * nb + blk];
        term = __fmul_rn(__fmul_rn(__int2float_rn(dot), dW), dA);
      } else {
        term = __fmul_rn(__int2float_rn(dot), __fmul_rn(dW, dA));
      }
      terms[((size_t)s * rows_cta + r) * tstride + blk] = term;
    }
  }
  __syncthreads();

  // ---- phase 2: the ordered sums and the epilogue
  if (g.swiglu) {
    // thread (s, r) = (warp, lane): warp s holds the 32 products of one Q8_0
    // block of row s (rt == 32)
    if (warp < B) {
      const int s = warp, r = lane;
      const float* tg = terms + ((size_t)s * rows_cta + r) * tstride;
      const float* tu = terms + ((size_t)s * rows_cta + g.rt + r) * tstride;
      float gs = 0.0f, us = 0.0f;
      for (int k = 0; k < nb; ++k) {
        gs = __fadd_rn(gs, tg[k]);
        us = __fadd_rn(us, tu[k]);
      }
      const int e = r0 + r;
      const uint32_t ord = g.swiglu_ordinal;
      check_finite(gs, &b.err[s], ord, D_GATE, 0, e);
      check_finite(us, &b.err[s], ord, D_UP, 0, e);
      const float ex = expf4_lane(__fsub_rn(0.0f, gs));
      const float p = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, ex)), us);
      if (b.product_out) b.product_out[(size_t)s * kFfn + e] = p;
      check_finite(p, &b.err[s], ord, D_SWIGLU, 0, e);
      quantize_row_block(b, p, s, r0 / 32);
    }
    return;
  }
  for (int item = tid; item < B * g.rt; item += kSgThreads) {
    const int s = item / g.rt, r = item - s * g.rt;
    const float* t = terms + ((size_t)s * rows_cta + r) * tstride;
    float acc = 0.0f;
    for (int k = 0; k < nb; ++k) acc = __fadd_rn(acc, t[k]);
    const Epilogue& ep = g.seg[si].ep;
    const int orow = r0 - seg_begin + r;
    float* dst = ep.out + (size_t)s * ep.ld + orow;
    float v;
    if (ep.mode == EPI_BIAS) v = __fadd_rn(acc, ep.bias[orow]);
    else if (ep.mode == EPI_RESIDUAL) v = __fadd_rn(*dst, acc);
    else v = acc;
    *dst = v;
    check_finite(v, &ep.err[s], ep.layer_ordinal, ep.domain, 0, orow);
  }
}

size_t small_gemv_smem(const SmallGemv& g, int B) {
  const int nb = g.cols / 32;
  const int bpb = g.wtype == W_Q4_0 ? 18 : 34;
  const int rows_cta = g.rt * (g.swiglu ? 2 : 1);
  const size_t wbytes = ((size_t)rows_cta * nb * bpb + 15) & ~(size_t)15;
  const size_t act = (size_t)B * g.cols + (size_t)B * nb * 8;
  size_t tbytes = (size_t)B * rows_cta * (nb + 1) * 4;
  if (g.norm_weight)
    tbytes = std::max(tbytes, ((size_t)B * ((kHidden / 32) * 33 + kHidden) + kHidden) * 4);
  return 16 + wbytes + act + tbytes;
}

}  // namespace

bool small_gemv_supported(const SmallGemv& g, int B) {
  if (B < 1 || B > 8 || g.rt <= 0 || g.cols % 32) return false;
  if (g.norm_weight && g.cols != kHidden) return false;
  const int bpb = g.wtype == W_Q4_0 ? 18 : 34;
  if (((size_t)g.rt * (g.cols / 32) * bpb) % 16) return false;  // bulk copy size
  if (g.swiglu && (g.rt != 32 || g.nseg != 2 || g.seg[0].rows_end != g.seg[1].rows_end))
    return false;
  // no CTA straddles two stacked matrices
  for (int i = 0; i < g.nseg; ++i) {
    const int begin = (i && !g.swiglu) ? g.seg[i - 1].rows_end : 0;
    if ((g.seg[i].rows_end - begin) % g.rt) return false;
  }
  return small_gemv_smem(g, B) <= 200 * 1024;
}

void launch_small_gemv(const SmallGemv& g, const Batch& b, unsigned int* status, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(small_gemv_kernel<18>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(small_gemv_kernel<34>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attribute_done(configured);
  }
  const int rows = g.swiglu ? g.seg[0].rows_end : g.seg[g.nseg - 1].rows_end;
  const int grid = rows / g.rt;
  const size_t smem = small_gemv_smem(g, b.rows);
  if (g.wtype == W_Q4_0)
    launch_pdl(small_gemv_kernel<18>, grid, kSgThreads, smem, s, g, b, status);
  else
    launch_pdl(small_gemv_kernel<34>, grid, kSgThreads, smem, s, g, b, status);
}

}  // namespace pb
