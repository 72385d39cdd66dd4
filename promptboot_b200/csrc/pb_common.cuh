// Device-side building blocks shared by the decode kernels.
//
// Every floating-point helper here reproduces one operation sequence of the
// reference (sulewicz/promptboot, crates/promptboot-core/src/fp32_sse2.rs) with
// IEEE round-to-nearest binary32/binary64 operations.  The library is compiled
// with -fmad=false, so `a * b + c` below is two roundings exactly as the
// reference's scalar SSE2 mulss/addss pair; where a fused multiply-add is
// wanted it is written explicitly as __fmaf_rn and its exactness is argued
// beside it.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace pb {

constexpr int kHidden = 896;
constexpr int kFfn = 4864;
constexpr int kLayers = 24;
constexpr int kQHeads = 14;
constexpr int kKvHeads = 2;
constexpr int kHeadDim = 64;
constexpr int kVocab = 151936;
constexpr int kContextLimit = 32768;
constexpr int kActStride = kFfn;        // int8 activation row stride (largest K)
constexpr int kActBlocks = kFfn / 32;   // per-row activation block count stride
constexpr int kEos = 151645;

// Stage domains of the reference's InferenceDomain (inference.rs:171-195).
enum Domain : uint32_t {
  D_EMBEDDING = 3, D_ATTN_NORM = 4, D_Q = 5, D_K = 6, D_V = 7, D_ROPE = 8, D_KV = 9,
  D_ATTENTION = 10, D_ATTN_OUTPUT = 11, D_FFN_NORM = 12, D_GATE = 13, D_UP = 14,
  D_SWIGLU = 15, D_DOWN = 16, D_OUTPUT_NORM = 17, D_LOGITS = 18,
};

// Programmatic dependent launch: every forward kernel starts with this.  It
// lets the next kernel of the stream be scheduled while this one runs (its
// CTAs then wait here), and waits until the previous kernel has completed and
// its memory is visible, before any global memory is read or written.  A
// no-op for kernels launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.launch_dependents;\n\tgriddepcontrol.wait;" ::: "memory");
}
// The two halves of pdl_begin, for kernels that do dependency-free work (a
// weight prefetch) in between: every thread triggers, and every thread that
// touches global memory written or read by earlier kernels waits first.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float fbits(uint32_t b) { return __uint_as_float(b); }
__device__ __forceinline__ uint32_t bitsf(float f) { return __float_as_uint(f); }
__device__ __forceinline__ bool finite_bits(uint32_t b) {
  return (b & 0x7f800000u) != 0x7f800000u;
}

// A stage failure is ranked so that one 64-bit atomicMin per sequence keeps the
// failure the reference's serial stage order (inference.rs:1454-1765) would have
// reported first: stage rank, then word index; the offending bits ride along.
//   rank = ((layer_ordinal * 32) + domain) * 2 + sub
//   layer_ordinal: 0 embedding, 1..24 decoder layers, 25 output head.
__device__ __forceinline__ unsigned long long error_key(uint32_t layer_ordinal, uint32_t domain,
                                                        uint32_t sub, uint32_t index,
                                                        uint32_t bits) {
  uint64_t rank = ((uint64_t)layer_ordinal * 32u + domain) * 2u + sub;
  return (unsigned long long)((rank << 50) | ((uint64_t)index << 32) | bits);
}
constexpr unsigned long long kNoError = ~0ull;

__device__ __forceinline__ void check_finite(float v, unsigned long long* err,
                                             uint32_t layer_ordinal, uint32_t domain,
                                             uint32_t sub, uint32_t index) {
  uint32_t b = bitsf(v);
  if (!finite_bits(b)) atomicMin(err, error_key(layer_ordinal, domain, sub, index, b));
}

// fp32_sse2.rs:362-376
__device__ __forceinline__ float half_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1fu;
  uint32_t fraction = bits & 0x03ffu;
  uint32_t out;
  if (exponent == 0) {
    if (fraction == 0) {
      out = sign;
    } else {
      uint32_t shift = (uint32_t)__clz(fraction) - 21u;
      uint32_t normalized = fraction << shift;
      out = sign | ((113u - shift) << 23) | ((normalized & 0x03ffu) << 13);
    }
  } else if (exponent == 31) {
    out = sign | 0x7f800000u | (fraction << 13);
  } else {
    out = sign | ((exponent + 112u) << 23) | (fraction << 13);
  }
  return fbits(out);
}

// fp32_sse2.rs:924-943: round-to-nearest-even binary32 -> binary16 built from two
// scaling multiplies and one add.
__device__ __forceinline__ uint16_t f32_to_half(uint32_t bits) {
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  uint32_t magnitude = bits & 0x7fffffffu;
  float base = __fmul_rn(__fmul_rn(fbits(magnitude), fbits(0x77800000u)), fbits(0x08800000u));
  uint32_t doubled = bits + bits;
  uint32_t bias = doubled & 0xff000000u;
  if (bias < 0x71000000u) bias = 0x71000000u;
  uint32_t rounded = bitsf(__fadd_rn(fbits((bias >> 1) + 0x07800000u), base));
  uint32_t exponent = (rounded >> 13) & 0x7c00u;
  uint32_t mantissa = rounded & 0x0fffu;
  if (doubled > 0xff000000u) return (uint16_t)(sign | 0x7e00u);
  return (uint16_t)(sign | (uint16_t)(exponent + mantissa));
}

// fp32_sse2.rs:378-402
__device__ __forceinline__ float scalbn_ref(float value, int exponent) {
  if (exponent > 127) {
    value = __fmul_rn(value, fbits(0x7f000000u));
    exponent -= 127;
    if (exponent > 127) {
      value = __fmul_rn(value, fbits(0x7f000000u));
      exponent -= 127;
      if (exponent > 127) exponent = 127;
    }
  } else if (exponent < -126) {
    float step = __fmul_rn(fbits(0x00800000u), fbits(0x4b800000u));
    value = __fmul_rn(value, step);
    exponent += 126 - 24;
    if (exponent < -126) {
      value = __fmul_rn(value, step);
      exponent += 126 - 24;
      if (exponent < -126) exponent = -126;
    }
  }
  return __fmul_rn(value, fbits((uint32_t)(0x7f + exponent) << 23));
}

// fp32_sse2.rs:404-469: the reference's own binary32 exponential (FreeBSD msun
// e_expf.c as carried by rust libm 0.2.11), used only by the sampler.
__device__ __forceinline__ float expf_ref(float x) {
  uint32_t in = bitsf(x);
  uint32_t magnitude = in & 0x7fffffffu;
  uint32_t sign = in >> 31;
  if (magnitude >= 0x42aeac50u) {
    if (magnitude > 0x7f800000u) return x;
    if (magnitude >= 0x42b17218u && sign == 0) return __fmul_rn(x, fbits(0x7f000000u));
    if (sign != 0 && magnitude >= 0x42cff1b5u) return 0.0f;
  }
  int k;
  float hi, lo;
  if (magnitude > 0x3eb17218u) {
    if (magnitude > 0x3f851592u) {
      float half = sign == 0 ? 0.5f : -0.5f;
      k = __float2int_rz(__fadd_rn(__fmul_rn(fbits(0x3fb8aa3bu), x), half));
    } else {
      k = 1 - (int)sign - (int)sign;
    }
    float kf = __int2float_rn(k);
    hi = __fsub_rn(x, __fmul_rn(kf, fbits(0x3f317200u)));
    lo = __fmul_rn(kf, fbits(0x35bfbe8eu));
    x = __fsub_rn(hi, lo);
  } else if (magnitude > 0x39000000u) {
    k = 0;
    hi = x;
    lo = 0.0f;
  } else {
    return __fadd_rn(1.0f, x);
  }
  float square = __fmul_rn(x, x);
  float c = __fsub_rn(x, __fmul_rn(square, __fadd_rn(fbits(0x3e2aaa8fu),
                                                      __fmul_rn(square, fbits(0xbb355215u)))));
  float fraction = __fdiv_rn(__fmul_rn(x, c), __fsub_rn(2.0f, c));
  float y = __fadd_rn(1.0f, __fadd_rn(__fsub_rn(fraction, lo), hi));
  return k == 0 ? y : scalbn_ref(y, k);
}

// fp32_sse2.rs:1336-1372: one lane of ggml's four-lane vector exponential
// (softmax and SiLU); an input of -inf maps to +0.
__device__ __forceinline__ float expf4_lane(float x) {
  if (bitsf(x) == 0xff800000u) return 0.0f;
  float z = __fadd_rn(__fmul_rn(x, fbits(0x3fb8aa3bu)), fbits(0x4b400000u));
  float n = __fsub_rn(z, fbits(0x4b400000u));
  float b = __fsub_rn(__fsub_rn(x, __fmul_rn(n, fbits(0x3f317200u))),
                      __fmul_rn(n, fbits(0x35bfbe8eu)));
  uint32_t e = bitsf(z) << 23;
  float k = fbits(e + 0x3f800000u);
  float absn = fbits(bitsf(n) & 0x7fffffffu);
  float u = __fmul_rn(b, b);
  float first = __fadd_rn(__fmul_rn(fbits(0x3c072010u), b), fbits(0x3d2b9f17u));
  float second = __fadd_rn(__fmul_rn(fbits(0x3e2aaf33u), b), fbits(0x3efffedbu));
  float poly = __fadd_rn(__fmul_rn(first, u), second);
  float j = __fadd_rn(__fmul_rn(poly, u), __fmul_rn(fbits(0x3f7ffff6u), b));
  if (!(absn > fbits(0x42fc0000u))) return __fadd_rn(__fmul_rn(j, k), k);
  uint32_t g = !(n > 0.0f) ? 0x82000000u : 0u;
  float s1 = fbits(g + 0x7f000000u);
  float s2 = fbits(e - g);
  float exceptional = __fmul_rn(__fadd_rn(__fmul_rn(s2, j), s2), s1);
  return absn > fbits(0x43400000u) ? __fmul_rn(s1, s1) : exceptional;
}

// inference.rs:2035-2052 with the per-sequence context capacity as a parameter
// (the reference fixes it at 32768).  Word offsets inside one sequence's KV.
__device__ __forceinline__ size_t kv_key_word(size_t capacity, int layer, int head, int position,
                                              int component) {
  size_t base = (size_t)layer * 4 * capacity * 64;
  return base + ((((size_t)head * (capacity / 4) + position / 4) * 64 + component) * 4 +
                 position % 4);
}
__device__ __forceinline__ size_t kv_value_word(size_t capacity, int layer, int head,
                                                int position, int component) {
  size_t base = (size_t)layer * 4 * capacity * 64 + 2 * capacity * 64;
  return base + (((size_t)head * capacity + position) * 64 + component);
}

}  // namespace pb
