// Decode-step kernels for sm_100a: embedding, RMSNorm + Q8_0 quantizer, the
// Q4_0 / Q8_0 block-scaled matrix-vector products, RoPE + KV write, GQA decode
// attention, SwiGLU + quantizer and the greedy argmax.
//
// Each kernel follows the operation order of the reference's scalar code
// (sulewicz/promptboot crates/promptboot-core/src/fp32_sse2.rs), cited per
// kernel, so that its binary32 results are the reference's bit for bit.
#include "pb_common.cuh"
#include "pb_kernels.cuh"
#include "pb_quant.cuh"

#include <cstdio>
#include <cstdlib>

namespace pb {

// ---------------------------------------------------------------- reductions

// ------------------------------------------------------------------ embedding

// fp32_sse2.rs:897-922: hidden = fl(d * (q - 8)), low nibbles are elements 0-15.
// The token is also recorded in the slot's history (the sampler's penalty set).
__global__ void embed_kernel(Batch b, const uint8_t* __restrict__ emb) {
  pdl_begin();
  int row = blockIdx.x;
  uint32_t token = b.tokens[row];
  const uint8_t* w = emb + (size_t)token * 28 * 18;
  for (int e = threadIdx.x; e < kHidden; e += blockDim.x) {
    const uint8_t* block = w + (e >> 5) * 18;
    float d = half_to_f32((uint16_t)(block[0] | (block[1] << 8)));
    int i = e & 31;
    uint8_t packed = block[2 + (i & 15)];
    int q = (i < 16 ? (packed & 0x0f) : (packed >> 4)) - 8;
    float h = __fmul_rn(d, __int2float_rn(q));
    b.hidden[(size_t)row * kHidden + e] = h;
    check_finite(h, &b.err[row], 0, D_EMBEDDING, 0, e);
  }
  if (threadIdx.x == 0)
    b.history[(size_t)b.slots[row] * b.capacity + b.positions[row]] = token;
}

void launch_embed(const Batch& b, const uint8_t* embedding, cudaStream_t s) {
  launch_pdl(embed_kernel, b.rows, 128, 0, s, b, embedding);
}

// fp32_sse2.rs:1310-1334 then the quantizer.  The reference sums the 896 f64
// squares serially.  Every square is a binary32 value, a multiple of the
// smallest square's ulp u = 2^(emin - 150) (biased exponents, subnormals as 1);
// all partial sums stay below 896 * 2^(emax - 126) < 2^(emax - 116), so when
// emax - emin <= 19 every partial sum of any grouping is an f64-representable
// multiple of u and the tree sum equals the serial one exactly.  Otherwise (or
// with a non-finite square) one thread repeats the serial sum from shared memory.
constexpr int kNormThreads = kHidden / 4;  // 224: one float4 per thread

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_quant_kernel(Batch b, const float* __restrict__ weight, uint32_t layer_ordinal,
                     uint32_t domain) {
  pdl_begin();
  __shared__ __align__(16) float sq[kHidden];  // squares, then the normalized row
  __shared__ double part[kNormThreads / 32];
  __shared__ int ext[2][kNormThreads / 32];
  __shared__ double total;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int row = blockIdx.x;
  const float4 xv = reinterpret_cast<const float4*>(b.hidden + (size_t)row * kHidden)[t];
  const float4 wv = reinterpret_cast<const float4*>(weight)[t];
  const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
  const float ws[4] = {wv.x, wv.y, wv.z, wv.w};
  double sum = 0.0;
  int emin = 255, emax = 0;  // emax 255 marks a non-finite square
  float q4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float q = __fmul_rn(xs[i], xs[i]);
    q4[i] = q;
    sum += (double)q;
    const uint32_t qb = bitsf(q) & 0x7fffffffu;
    const int e = (int)(qb >> 23);
    if (qb != 0) {
      emin = min(emin, max(e, 1));
      emax = max(emax, max(e, 1));
    }
  }
  *reinterpret_cast<float4*>(&sq[4 * t]) = make_float4(q4[0], q4[1], q4[2], q4[3]);
  sum = warp_sum_f64(sum);
  for (int o = 16; o > 0; o >>= 1) {
    emin = min(emin, __shfl_xor_sync(0xffffffffu, emin, o));
    emax = max(emax, __shfl_xor_sync(0xffffffffu, emax, o));
  }
  if (lane == 0) {
    part[warp] = sum;
    ext[0][warp] = emin;
    ext[1][warp] = emax;
  }
  __syncthreads();
  if (t == 0) {
    double tree = 0.0;
    int lo = 255, hi = 0;
    for (int w = 0; w < kNormThreads / 32; ++w) {
      tree += part[w];
      lo = min(lo, ext[0][w]);
      hi = max(hi, ext[1][w]);
    }
    if (hi == 255 || (hi >= lo && hi - lo > 19)) {
      // index order; the loads and widenings run ahead of the f64 add chain
      double serial = 0.0;
#pragma unroll 8
      for (int e = 0; e < kHidden; e += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(&sq[e]);
        serial += (double)t4.x;
        serial += (double)t4.y;
        serial += (double)t4.z;
        serial += (double)t4.w;
      }
      tree = serial;
    }
    total = tree;
  }
  __syncthreads();
  const float mean = (float)(total / 896.0);
  const float inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, fbits(0x358637bdu))));
  float y4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    y4[i] = __fmul_rn(__fmul_rn(xs[i], inverse), ws[i]);
    check_finite(y4[i], &b.err[row], layer_ordinal, domain, 0, 4 * t + i);
  }
  const float4 yv = make_float4(y4[0], y4[1], y4[2], y4[3]);
  *reinterpret_cast<float4*>(&sq[4 * t]) = yv;
  if (b.norm_out) reinterpret_cast<float4*>(b.norm_out + (size_t)row * kHidden)[t] = yv;
  __syncthreads();
  for (int blk = warp; blk < kHidden / 32; blk += kNormThreads / 32)
    quantize_row_block(b, sq[blk * 32 + lane], row, blk);
}

void launch_rmsnorm_quant(const Batch& b, const float* weight, uint32_t layer_ordinal,
                          uint32_t domain, cudaStream_t s) {
  launch_pdl(rmsnorm_quant_kernel, b.rows, kNormThreads, 0, s, b, weight, layer_ordinal, domain);
}

__global__ void quant_kernel(Batch b, const float* __restrict__ x, size_t ld, int columns) {
  pdl_begin();
  int row = blockIdx.x;
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int blk = warp; blk < columns / 32; blk += blockDim.x >> 5) {
    quantize_row_block(b, x[(size_t)row * ld + blk * 32 + lane], row, blk);
  }
}

void launch_quant(const Batch& b, const float* x, size_t ld, int columns, cudaStream_t s) {
  launch_pdl(quant_kernel, b.rows, 256, 0, s, b, x, ld, columns);
}

// fp32_sse2.rs:1751-1770 then the quantizer: product = fl(fl(g / (1 + e)) * u)
// with e = expf4(0 - g); checked as the SWIGLU stage.  Grid (rows, 4): each CTA
// takes 38 of the 152 blocks, each warp loads all of its blocks before computing.
constexpr int kSwigluSplit = 4;
constexpr int kSwigluPerWarp = (kFfn / 32 / kSwigluSplit + 7) / 8;  // 5

__global__ void __launch_bounds__(256) swiglu_quant_kernel(Batch b, uint32_t layer_ordinal) {
  pdl_begin();
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk0 = blockIdx.y * (kFfn / 32 / kSwigluSplit), blk_end = blk0 + kFfn / 32 / kSwigluSplit;
  const float* g = b.gate + (size_t)row * kFfn;
  const float* u = b.up + (size_t)row * kFfn;
  float gv[kSwigluPerWarp], uv[kSwigluPerWarp];
#pragma unroll
  for (int k = 0; k < kSwigluPerWarp; ++k) {
    const int blk = blk0 + warp + 8 * k;
    if (blk < blk_end) {
      gv[k] = g[blk * 32 + lane];
      uv[k] = u[blk * 32 + lane];
    }
  }
#pragma unroll
  for (int k = 0; k < kSwigluPerWarp; ++k) {
    const int blk = blk0 + warp + 8 * k;
    if (blk < blk_end) {
      const int e = blk * 32 + lane;
      const float ex = expf4_lane(__fsub_rn(0.0f, gv[k]));
      const float silu = __fdiv_rn(gv[k], __fadd_rn(1.0f, ex));
      const float p = __fmul_rn(silu, uv[k]);
      if (b.product_out) b.product_out[(size_t)row * kFfn + e] = p;
      check_finite(p, &b.err[row], layer_ordinal, D_SWIGLU, 0, e);
      quantize_row_block(b, p, row, blk);
    }
  }
}

void launch_swiglu_quant(const Batch& b, uint32_t layer_ordinal, cudaStream_t s) {
  launch_pdl(swiglu_quant_kernel, dim3(b.rows, kSwigluSplit), 256, 0, s, b, layer_ordinal);
}

// ------------------------------------------------ block-scaled matvec (GEMV)
//
// y[b][r] = sum over blocks k, IN ORDER, in binary32 of
//   Q4_0: fl(fl(f32(i32dot) * dW) * dA)   (fp32_sse2.rs:1217-1248)
//   Q8_0: fl(f32(i32dot) * fl(dW * dA))   (fp32_sse2.rs:1250-1281)
// The exact int32 block dots and the per-block terms are computed in parallel
// (phase 1, terms staged in shared memory); the order-sensitive binary32 sum
// runs per (row, sequence) in block order (phase 2).  Q4_0 nibbles enter dp4a
// unsigned (0..15) and the zero point is removed exactly as -8 * sum(a).

constexpr int kGemvThreads = 256;
constexpr int kGemvSeqChunk = 8;

__device__ __forceinline__ uint32_t ld_u32_2aligned(const uint8_t* p) {
  // p is 2-byte aligned in shared memory
  uint32_t lo = *reinterpret_cast<const uint16_t*>(p);
  uint32_t hi = *reinterpret_cast<const uint16_t*>(p + 2);
  return lo | (hi << 16);
}

template <int BPB, int RT>
__global__ void __launch_bounds__(kGemvThreads)
qgemv_kernel(const uint8_t* __restrict__ w, int rows, int nb, Batch b, Epilogue ep) {
  pdl_begin();
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x;
  const int r0 = blockIdx.x * RT;
  const size_t row_bytes = (size_t)nb * BPB;
  const int wbytes = RT * nb * BPB;
  const int wbytes_padded = (wbytes + 15) & ~15;
  const int tstride = nb + 1;
  uint8_t* wt = smem;
  float* terms = reinterpret_cast<float*>(smem + wbytes_padded);

  const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)r0 * row_bytes);
  for (int i = tid; i < wbytes / 16; i += kGemvThreads) reinterpret_cast<uint4*>(wt)[i] = src[i];
  __syncthreads();

  for (int s0 = 0; s0 < b.rows; s0 += kGemvSeqChunk) {
    const int sb = min(kGemvSeqChunk, b.rows - s0);
    for (int item = tid; item < RT * nb; item += kGemvThreads) {
      const int r = item / nb, blk = item - r * nb;
      const uint8_t* bp = wt + (size_t)(r * nb + blk) * BPB;
      const float dW = half_to_f32(*reinterpret_cast<const uint16_t*>(bp));
      uint32_t wq[8];
      if (BPB == 18) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t p = ld_u32_2aligned(bp + 2 + 4 * j);
          wq[j] = p & 0x0f0f0f0fu;
          wq[4 + j] = (p >> 4) & 0x0f0f0f0fu;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) wq[j] = ld_u32_2aligned(bp + 2 + 4 * j);
      }
      for (int s = 0; s < sb; ++s) {
        const int row = s0 + s;
        const uint4* ap = reinterpret_cast<const uint4*>(b.aq + (size_t)row * kActStride + blk * 32);
        const uint4 a0 = ap[0], a1 = ap[1];
        const int aw[8] = {(int)a0.x, (int)a0.y, (int)a0.z, (int)a0.w,
                           (int)a1.x, (int)a1.y, (int)a1.z, (int)a1.w};
        int dot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = __dp4a((int)wq[j], aw[j], dot);
        const float dA = b.ad[(size_t)row * kActBlocks + blk];
        float term;
        if (BPB == 18) {
          dot -= 8 * b.asum[(size_t)row * kActBlocks + blk];
          term = __fmul_rn(__fmul_rn(__int2float_rn(dot), dW), dA);
        } else {
          term = __fmul_rn(__int2float_rn(dot), __fmul_rn(dW, dA));
        }
        terms[(s * RT + r) * tstride + blk] = term;
      }
    }
    __syncthreads();
    for (int item = tid; item < sb * RT; item += kGemvThreads) {
      const int s = item / RT, r = item - s * RT;
      const float* t = terms + (s * RT + r) * tstride;
      float acc = 0.0f;
      for (int blk = 0; blk < nb; ++blk) acc = __fadd_rn(acc, t[blk]);
      const int row = s0 + s, orow = r0 + r;
      float* dst = ep.out + (size_t)row * ep.ld + orow;
      float v;
      if (ep.mode == EPI_BIAS) v = __fadd_rn(acc, ep.bias[orow]);
      else if (ep.mode == EPI_RESIDUAL) v = __fadd_rn(*dst, acc);
      else v = acc;
      *dst = v;
      check_finite(v, &ep.err[row], ep.layer_ordinal, ep.domain, 0, orow);
    }
    __syncthreads();
  }
}

template <int BPB, int RT>
static size_t qgemv_smem(int nb) {
  int wbytes = RT * nb * BPB;
  return (size_t)((wbytes + 15) & ~15) + (size_t)kGemvSeqChunk * RT * (nb + 1) * 4;
}

void launch_qgemv(int wtype, const uint8_t* w, int rows, int columns, const Batch& b,
                  const Epilogue& ep, cudaStream_t s) {
  const int nb = columns / 32;
  if (wtype == W_Q4_0) {
    if (nb > 64) {
      constexpr int RT = 8;
      launch_pdl(qgemv_kernel<18, RT>, rows / RT, kGemvThreads, qgemv_smem<18, RT>(nb), s, w, rows, nb, b, ep);
    } else {
      constexpr int RT = 32;
      launch_pdl(qgemv_kernel<18, RT>, rows / RT, kGemvThreads, qgemv_smem<18, RT>(nb), s, w, rows, nb, b, ep);
    }
  } else {
    if (nb > 64) {
      constexpr int RT = 8;
      launch_pdl(qgemv_kernel<34, RT>, rows / RT, kGemvThreads, qgemv_smem<34, RT>(nb), s, w, rows, nb, b, ep);
    } else {
      constexpr int RT = 32;
      launch_pdl(qgemv_kernel<34, RT>, rows / RT, kGemvThreads, qgemv_smem<34, RT>(nb), s, w, rows, nb, b, ep);
    }
  }
}

// ------------------------------------------------------------- RoPE and KV

// fp32_sse2.rs:1413-1428 on q (14 heads) and k (2 heads), then the KV write of
// inference.rs:1809-1887 (tiled K, row-major V).  Checks: ROPE q, ROPE k, KV k.
__global__ void rope_kv_kernel(Batch b, int layer, const float* __restrict__ rope) {
  pdl_begin();
  int row = blockIdx.x;
  int position = b.positions[row];
  uint32_t ord = (uint32_t)layer + 1;
  const float* table = rope + (size_t)position * 64;
  float* q = b.q + (size_t)row * kHidden;
  float* k = b.k + (size_t)row * 128;
  const float* v = b.v + (size_t)row * 128;
  float* kv = b.kv + (size_t)b.slots[row] * (size_t)kLayers * 4 * b.capacity * 64;
  for (int item = threadIdx.x; item < 16 * 32; item += blockDim.x) {
    int head = item >> 5, pair = item & 31;
    float* x = head < 14 ? q + head * 64 : k + (head - 14) * 64;
    float left = x[pair], right = x[pair + 32];
    float c = table[pair * 2], sn = table[pair * 2 + 1];
    float l2 = __fsub_rn(__fmul_rn(left, c), __fmul_rn(right, sn));
    float r2 = __fadd_rn(__fmul_rn(left, sn), __fmul_rn(right, c));
    x[pair] = l2;
    x[pair + 32] = r2;
    if (head < 14) {
      check_finite(l2, &b.err[row], ord, D_ROPE, 0, head * 64 + pair);
      check_finite(r2, &b.err[row], ord, D_ROPE, 0, head * 64 + pair + 32);
    } else {
      int kh = head - 14;
      check_finite(l2, &b.err[row], ord, D_ROPE, 1, kh * 64 + pair);
      check_finite(r2, &b.err[row], ord, D_ROPE, 1, kh * 64 + pair + 32);
      check_finite(l2, &b.err[row], ord, D_KV, 0, kh * 64 + pair);
      check_finite(r2, &b.err[row], ord, D_KV, 0, kh * 64 + pair + 32);
      kv[kv_key_word(b.capacity, layer, kh, position, pair)] = l2;
      kv[kv_key_word(b.capacity, layer, kh, position, pair + 32)] = r2;
    }
  }
  for (int i = threadIdx.x; i < 128; i += blockDim.x)
    kv[kv_value_word(b.capacity, layer, i >> 6, position, i & 63)] = v[i];
}

void launch_rope_kv(const Batch& b, int layer, const float* rope, cudaStream_t s) {
  launch_pdl(rope_kv_kernel, b.rows, 256, 0, s, b, layer, rope);
}

// --------------------------------------------------------------- attention
//
// fp32_sse2.rs:1430-1672, GQA-shared (pb_attention.cu): the shared-memory path
// up to kAttnMaxPositions, the global-probability path beyond.

int launch_attention(const Batch& b, int layer, int max_span, bool quantize, const float* rope,
                     cudaStream_t s) {
  // The grouped path runs one PV block per (row, KV head): at few rows that
  // leaves most of the 148 SMs idle, and the split path (softmax, then one PV
  // block per group of output components) is faster up to 64 rows at
  // 512-1535 positions.  PB_ATTN_SPLIT=0/1 forces either path.
  const char* f = std::getenv("PB_ATTN_SPLIT");
  const bool split = f && *f ? std::atoi(f) != 0 : b.rows <= kAttnSplitRows && max_span > kAttnSplitMinSpan;
  if (max_span <= kAttnMaxPositions && !split)
    return launch_attention_grouped(b, layer, (max_span + 3) & ~3, quantize, rope, s);
  return launch_attention_long(b, layer, (max_span + 3) & ~3, quantize, rope, s);
}

// -------------------------------------------------------------- argmax/top8

// fp32_sse2.rs:1772-1784: first maximum by strict > (lowest id among equal
// values, +0 and -0 equal).  Also records the first non-finite word.
__global__ void argmax_kernel(const float* __restrict__ logits, size_t ld, int words,
                              uint32_t* ids, uint32_t* bits_out,
                              unsigned long long* first_nonfinite) {
  pdl_begin();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* x = logits + (size_t)blockIdx.x * ld;
  float best = fbits(0xff800000u);
  int besti = 0x7fffffff;
  // Each thread visits its indices in increasing order, so strict > keeps the
  // earliest of equal values; four 16-byte loads in flight per thread.
  auto consider = [&](float v, int i) {
    const uint32_t vb = bitsf(v);
    if (!finite_bits(vb) && first_nonfinite)
      atomicMin(&first_nonfinite[blockIdx.x], ((unsigned long long)i << 32) | vb);
    if (v > best || besti == 0x7fffffff) { best = v; besti = i; }
  };
  const int nvec = (ld % 4 == 0) ? words / 4 : 0;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const int stride = (int)blockDim.x;
  int f = threadIdx.x;
  for (; f + 3 * stride < nvec; f += 4 * stride) {
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = x4[f + u * stride];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i0 = 4 * (f + u * stride);
      consider(a[u].x, i0);
      consider(a[u].y, i0 + 1);
      consider(a[u].z, i0 + 2);
      consider(a[u].w, i0 + 3);
    }
  }
  for (; f < nvec; f += stride) {
    const float4 a = x4[f];
    consider(a.x, 4 * f);
    consider(a.y, 4 * f + 1);
    consider(a.z, 4 * f + 2);
    consider(a.w, 4 * f + 3);
  }
  for (int i = 4 * nvec + threadIdx.x; i < words; i += stride) consider(x[i], i);
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (!(best > ov) && oi < besti)) { best = ov; besti = oi; }
  }
  if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = besti; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (bv[w] > best || (!(best > bv[w]) && bi[w] < besti)) { best = bv[w]; besti = bi[w]; }
    ids[blockIdx.x] = (uint32_t)besti;
    if (bits_out) bits_out[blockIdx.x] = bitsf(x[besti]);
  }
}

void launch_argmax(const float* logits, size_t ld, int rows, int words, uint32_t* ids,
                   uint32_t* bits, unsigned long long* first_nonfinite, cudaStream_t s) {
  launch_pdl(argmax_kernel, rows, 1024, 0, s, logits, ld, words, ids, bits, first_nonfinite);
}

void init_kernel_attributes() {
  cudaFuncSetAttribute(qgemv_kernel<18, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(qgemv_kernel<18, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(qgemv_kernel<34, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(qgemv_kernel<34, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

}  // namespace pb
