// Warp reductions and the Q8_0 activation quantizer shared by the kernels that
// produce matvec inputs (RMSNorm, SwiGLU, attention output, the operator API).
#pragma once

#include <cuda_fp16.h>

#include "pb_common.cuh"
#include "pb_kernels.cuh"

namespace pb {

__device__ __forceinline__ double warp_sum_f64(double v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f32(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i32(int v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------ Q8_0 quantizer

// fp32_sse2.rs:945-983, one warp per 32-element block: d = amax / 127 rounded to
// binary16 for storage, inverse from the unrounded d, q = trunc(x * inv +- 0.5)
// (x86 truncation semantics), stored as its low byte.
// Returns this lane's quant; dstored = the stored scale (binary16 value as f32).
__device__ __forceinline__ int quantize_lane(float x, float& dstored) {
  float amax = warp_max_f32(fbits(bitsf(x) & 0x7fffffffu));
  float d = __fdiv_rn(amax, 127.0f);
  float inverse = bitsf(d) == 0 ? 0.0f : __fdiv_rn(1.0f, d);
  float v = __fmul_rn(x, inverse);
  float half = (bitsf(v) >> 31) == 0 ? 0.5f : -0.5f;
  // binary16 storage of d: the reference's conversion (fp32_sse2.rs:924-943)
  // rounds to nearest even and maps +inf to inf, and d is never NaN (amax, like
  // the reference's strict > scan, skips NaN), so the conversion instruction
  // gives the same bits, and back exactly.
  dstored = __half2float(__float2half_rn(d));
  // fp32_sse2.rs:336-345 truncates with cvttss2si, whose result for a value
  // outside the int32 range, an infinity or a NaN is 0x80000000 (a block whose
  // amax is below ~127 * 2^-128 has an infinite inverse); the conversion
  // instruction here would saturate instead.
  const float t = __fadd_rn(v, half);
  return fabsf(t) < 2147483648.0f ? __float2int_rz(t) : (int)0x80000000u;
}

// Row-major Q8_0 activation (the CUDA-core matvec's input): quants, scale and
// the block's quant sum for the Q4_0 zero-point correction.
__device__ __forceinline__ int quantize_block_warp(float x, int8_t* aq, float* ad, int* asum,
                                                   float& dstored) {
  const int q = quantize_lane(x, dstored);
  const int lane = threadIdx.x & 31;
  aq[lane] = (int8_t)q;
  const int total = warp_sum_i32((int)(int8_t)q);
  if (lane == 0) {
    *ad = dstored;
    *asum = total;
  }
  return q;
}

// Row `row`, block `blk` of an activation: the tensor-core layout when the batch
// carries one (Batch::aq_tc: chunk-major group (blk / 4, row / 8), quants of
// block blk % 4 at 256 (blk % 4), its scales after the 4 blocks), else the
// row-major buffers.
__device__ __forceinline__ void quantize_row_block(const Batch& b, float x, int row, int blk) {
  float d;
  if (b.aq_tc) {
    const int q = quantize_lane(x, d);
    const int lane = threadIdx.x & 31;
    const int j = blk & 3;
    int8_t* grp = b.aq_tc + ((size_t)(blk >> 2) * (b.tc_seqs >> 3) + (row >> 3)) * kTcGroupBytes;
    grp[j * 256 + (lane >> 4) * 128 + (row & 7) * 16 + (lane & 15)] = (int8_t)q;
    if (lane == 0) reinterpret_cast<float*>(grp + 1024)[j * 8 + (row & 7)] = d;
  } else {
    quantize_block_warp(x, b.aq + (size_t)row * kActStride + blk * 32,
                        b.ad + (size_t)row * kActBlocks + blk,
                        b.asum + (size_t)row * kActBlocks + blk, d);
  }
}

}  // namespace pb
