// Batched block-scaled matvec on the 5th-generation tensor cores (tcgen05,
// kind::i8) for sm_100a: Y[s][r] = sum over Q-blocks k IN ORDER of the
// reference's per-block term (fp32_sse2.rs:1217-1281), for B > 8 sequences.
//
// One tcgen05.mma per 32-element Q-block: M = 128 weight rows (A, K-major int8 in
// shared memory: Q4_0 nibbles as unsigned 0..15, Q8_0 quants signed), N = NT
// sequences (B, the Q8_0 activations, signed), K = 32.  Each MMA writes a fresh
// int32 block dot to one of two TMEM buffers; while the tensor core computes
// block k+1, the four warps drain block k from TMEM (warp w owns TMEM lanes
// 32w..32w+31 = weight rows) and apply the reference's scaling and in-order
// binary32 accumulation in registers:
//   Q4_0: t = fl(fl(f32(i - 8*sum(a)) * dW) * dA)     one IADD (magic-number
//         int->float, exact for |i| < 2^22), one FFMA (x*dW - 1.5*2^23*dW, exact
//         because 1.5*2^23*dW is representable for binary16 dW), one FMUL
//   Q8_0: t = fl(f32(i) * fl(dW * dA))
//   acc = fl(acc + t)
// Shared-memory tiles use the canonical no-swizzle K-major layout: 8-row x
// 16-byte core matrices, the two 16-byte K halves of an 8-row group adjacent
// (leading byte offset 128), groups 256 bytes apart (stride byte offset 256).
// Every mbarrier wait is bounded; a timeout sets *status, stops issuing, waits
// (bounded) for work in flight, frees TMEM and returns.
#include "pb_common.cuh"
#include "pb_kernels.cuh"

namespace pb {
namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after ~2^22 polls (seconds); the caller aborts.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 22); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(zero), "r"(zero)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// K-major, no swizzle: LBO (K direction) 128 B, SBO (M/N direction) 256 B,
// descriptor version 1 (bits 46-47), layout type 0.
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  uint64_t a = (smem_u32(p) >> 4) & 0x3fffu;
  return a | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}

// Byte offset of (row, half) in a canonical K-major tile (32 bytes per row).
__device__ __forceinline__ int tile_off(int row, int half) {
  return (row >> 3) * 256 + half * 128 + (row & 7) * 16;
}

constexpr int kM = 128;
constexpr int kThreads = 128;

constexpr int kStages = 3;  // smem stages (A/B tiles + scales); TMEM has 2 buffers

template <int NT>
struct TcSmem {
  static constexpr int kA = kM * 32;     // A tile bytes per stage
  static constexpr int kB = NT * 32;     // B tile bytes per stage
  static constexpr int kStage = kA + kB;
  static constexpr int kScaleOff = kStages * kStage;                 // dA [kStages][NT] f32
  static constexpr int kCOff = kScaleOff + kStages * NT * 4;         // C  [kStages][NT] i32
  static constexpr int kMiscOff = kCOff + kStages * NT * 4;          // 2 mbarriers + slot
  static constexpr int kBytes = kMiscOff + 64;
};

template <int BPB>
__device__ __forceinline__ void load_weight_block(const uint8_t* __restrict__ w, size_t off,
                                                  uint32_t& scale_bits, uint32_t (&q)[8]) {
  // off is even; read exactly the block's bytes with 2- and 4-byte aligned loads.
  const uint8_t* p = w + off;
  if ((off & 3) == 0) {
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p);
    uint32_t words[BPB == 18 ? 5 : 9];
    constexpr int nfull = BPB == 18 ? 4 : 8;
#pragma unroll
    for (int i = 0; i < nfull; ++i) words[i] = __ldg(p4 + i);
    words[nfull] = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(p + 4 * nfull));
    scale_bits = words[0] & 0xffffu;
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = __funnelshift_r(words[i], words[i + 1], 16);
  } else {
    scale_bits = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(p));
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p + 2);
    constexpr int nfull = BPB == 18 ? 4 : 8;
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = __ldg(p4 + i);
  }
}

template <int BPB, int NT>
__global__ void __launch_bounds__(kThreads)
qgemm_tc_kernel(const uint8_t* __restrict__ w, int rows, int nb, Batch b, Epilogue ep,
                unsigned int* status) {
  using L = TcSmem<NT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  float* dA_s = reinterpret_cast<float*>(smem + L::kScaleOff);
  int* C_s = reinterpret_cast<int*>(smem + L::kCOff);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + L::kMiscOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff + 16);

  constexpr uint32_t kCols = NT * 2 < 32 ? 32 : NT * 2;
  constexpr uint32_t kIdesc = (2u << 4) | ((BPB == 18 ? 0u : 1u) << 7) | (1u << 10) |
                              ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int seq0 = blockIdx.x * NT;
  const int row = blockIdx.y * kM + tid;
  const int nseq = min(NT, b.rows - seq0);
  const size_t row_bytes = (size_t)nb * BPB;

  if (warp == 0) tmem_alloc(tmem_slot, kCols);
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_barrier_init();
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  float acc[NT];
#pragma unroll
  for (int s = 0; s < NT; ++s) acc[s] = 0.0f;

  // Stage one Q-block: A rows (one per thread), B rows (threads < NT), scales.
  auto load_stage = [&](int st, int blk, float& dW, float& negMdW) {
    uint32_t sb, q[8];
    load_weight_block<BPB>(w, (size_t)row * row_bytes + (size_t)blk * BPB, sb, q);
    dW = half_to_f32((uint16_t)sb);
    negMdW = -__fmul_rn(12582912.0f, dW);
    uint8_t* A = smem + st * L::kStage;
    uint4 h0, h1;
    if (BPB == 18) {
      h0 = make_uint4(q[0] & 0x0f0f0f0fu, q[1] & 0x0f0f0f0fu, q[2] & 0x0f0f0f0fu, q[3] & 0x0f0f0f0fu);
      h1 = make_uint4((q[0] >> 4) & 0x0f0f0f0fu, (q[1] >> 4) & 0x0f0f0f0fu,
                      (q[2] >> 4) & 0x0f0f0f0fu, (q[3] >> 4) & 0x0f0f0f0fu);
    } else {
      h0 = make_uint4(q[0], q[1], q[2], q[3]);
      h1 = make_uint4(q[4], q[5], q[6], q[7]);
    }
    *reinterpret_cast<uint4*>(A + tile_off(tid, 0)) = h0;
    *reinterpret_cast<uint4*>(A + tile_off(tid, 1)) = h1;
    if (tid < NT) {
      uint8_t* B = A + L::kA;
      uint4 a0 = make_uint4(0, 0, 0, 0), a1 = a0;
      float da = 0.0f;
      int c = 0x4B400000;
      if (tid < nseq) {
        const size_t srow = (size_t)(seq0 + tid);
        const uint4* ap = reinterpret_cast<const uint4*>(b.aq + srow * kActStride + blk * 32);
        a0 = ap[0];
        a1 = ap[1];
        da = b.ad[srow * kActBlocks + blk];
        c = 0x4B400000 - 8 * b.asum[srow * kActBlocks + blk];
      }
      *reinterpret_cast<uint4*>(B + tile_off(tid, 0)) = a0;
      *reinterpret_cast<uint4*>(B + tile_off(tid, 1)) = a1;
      dA_s[st * NT + tid] = da;
      C_s[st * NT + tid] = c;
    }
    fence_async_shared();  // generic-proxy smem writes -> visible to the tensor core
  };
  auto issue = [&](int blk) {
    uint8_t* A = smem + (blk % kStages) * L::kStage;
    mma_i8(tmem_base + (uint32_t)((blk & 1) * NT), smem_desc(A), smem_desc(A + L::kA), kIdesc);
    mma_commit(&mbar[blk & 1]);
  };

  // Pipeline: in iteration k the CTA stages block k+1 (smem stage (k+1)%3, last
  // read by MMA k-2, already complete), then thread 0 issues MMA k+1 into TMEM
  // buffer (k+1)&1 (drained in iteration k-1), while all warps wait for MMA k
  // and drain buffer k&1.  Barrier votes keep every exit block-uniform.
  float dW_cur, negMdW_cur, dW_next = 0.0f, negMdW_next = 0.0f;
  uint32_t phase[2] = {0, 0};
  int pending[2] = {0, 0};  // MMAs committed and not yet waited for, per buffer (thread 0)
  load_stage(0, 0, dW_cur, negMdW_cur);
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (tid == 0) { issue(0); pending[0] = 1; }
  int timed_out = 0;
  for (int blk = 0; blk < nb; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nb) load_stage((blk + 1) % kStages, blk + 1, dW_next, negMdW_next);
    tc_before_sync();
    const int stop = __syncthreads_or(timed_out);
    tc_after_sync();
    if (stop) break;
    if (tid == 0 && blk + 1 < nb) { issue(blk + 1); pending[buf ^ 1] = 1; }
    if (!mbar_wait_bounded(&mbar[buf], phase[buf])) {
      timed_out = 1;
      continue;  // the vote at the top of the next iteration stops everyone
    }
    if (tid == 0) pending[buf] = 0;
    phase[buf] ^= 1u;
    const int st = blk % kStages;
    const float* dA = dA_s + st * NT;
    const int* C = C_s + st * NT;
    const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * NT);
#pragma unroll
    for (int c0 = 0; c0 < NT; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + c0, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int s = c0 + j;
        float t;
        if (BPB == 18) {
          const float x = __int_as_float((int)v[j] + C[s]);
          t = __fmul_rn(__fmaf_rn(x, dW_cur, negMdW_cur), dA[s]);
        } else {
          const float f = __fsub_rn(__int_as_float((int)v[j] + 0x4B400000), 12582912.0f);
          t = __fmul_rn(f, __fmul_rn(dW_cur, dA[s]));
        }
        acc[s] = __fadd_rn(acc[s], t);
      }
    }
    dW_cur = dW_next;
    negMdW_cur = negMdW_next;
  }
  tc_before_sync();
  const int aborted = __syncthreads_or(timed_out);
  tc_after_sync();
  if (aborted && tid == 0) {
    atomicOr(status, 1u);
    // Wait (bounded) for MMAs still in flight before their TMEM is released.
    for (int k = 0; k < 2; ++k)
      if (pending[k]) mbar_wait_bounded(&mbar[k], phase[k]);
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (warp == 0) tmem_dealloc(tmem_base, kCols);
  if (aborted) return;

#pragma unroll
  for (int s = 0; s < NT; ++s) {
    if (s < nseq) {
      const int seq = seq0 + s;
      float* dst = ep.out + (size_t)seq * ep.ld + row;
      float v;
      if (ep.mode == EPI_BIAS) v = __fadd_rn(acc[s], ep.bias[row]);
      else if (ep.mode == EPI_RESIDUAL) v = __fadd_rn(*dst, acc[s]);
      else v = acc[s];
      *dst = v;
      check_finite(v, &ep.err[seq], ep.layer_ordinal, ep.domain, 0, row);
    }
  }
}

template <int BPB, int NT>
void launch_tc(const uint8_t* w, int rows, int nb, const Batch& b, const Epilogue& ep,
               unsigned int* status, cudaStream_t s) {
  dim3 grid((b.rows + NT - 1) / NT, rows / kM);
  qgemm_tc_kernel<BPB, NT><<<grid, kThreads, TcSmem<NT>::kBytes, s>>>(w, rows, nb, b, ep, status);
}

}  // namespace

bool qgemm_tc_supported(int rows, int batch) { return rows % kM == 0 && batch > 8; }

// Picks the sequence tile so that the grid covers the 148 SMs; the weight tile
// is the slow grid dimension so the CTAs sharing it run together (one HBM read).
void launch_qgemm_tc(int wtype, const uint8_t* w, int rows, int columns, const Batch& b,
                     const Epilogue& ep, unsigned int* status, cudaStream_t s) {
  const int nb = columns / 32;
  const int rtiles = rows / kM;
  auto ctas = [&](int nt) { return rtiles * ((b.rows + nt - 1) / nt); };
  const int nt = ctas(64) >= 296 ? 64 : ctas(32) >= 148 ? 32 : 16;
  if (wtype == W_Q4_0) {
    if (nt == 64) launch_tc<18, 64>(w, rows, nb, b, ep, status, s);
    else if (nt == 32) launch_tc<18, 32>(w, rows, nb, b, ep, status, s);
    else launch_tc<18, 16>(w, rows, nb, b, ep, status, s);
  } else {
    if (nt == 64) launch_tc<34, 64>(w, rows, nb, b, ep, status, s);
    else if (nt == 32) launch_tc<34, 32>(w, rows, nb, b, ep, status, s);
    else launch_tc<34, 16>(w, rows, nb, b, ep, status, s);
  }
}

}  // namespace pb
