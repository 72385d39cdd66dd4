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
// Warp-specialised pipeline over 4-block chunks, chained by mbarriers only: a
// loader warp streams raw weight bytes (8-byte cp.async granules; 18- and
// 34-byte blocks are only 2-byte aligned) and scatters activation rows by 16-byte
// cp.async straight into the canonical B layout, four unpack warps turn the raw
// weights into the canonical A tile, one thread issues the four MMAs of a chunk
// with one commit, and eight epilogue warps drain the TMEM group.  Every wait is
// bounded (200 ms on %globaltimer, or another role's abort); an abort sets
// *status, lets committed MMAs finish (bounded), frees TMEM and returns.
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

constexpr int kKC = 4;  // Q-blocks per chunk = MMAs per commit
constexpr int kRS = 4;  // ring stages
// Warp roles: one cp.async loader, one MMA issuer, four unpackers (one weight
// row each), eight epilogue warps (two per TMEM lane quarter, half the columns each).
constexpr int kLoaderWarp = 0, kMmaWarp = 1, kUnpackWarp0 = 2, kEpiWarp0 = 6;
constexpr int kUnpackWarps = 4, kEpiWarps = 8;
constexpr int kWsThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 448

template <int BPB, int NT>
struct TcLayout {
  static constexpr int kRowRaw = ((kKC * BPB + 15) / 16) * 16;  // 80 (Q4_0) / 144 (Q8_0)
  static constexpr int kARaw = kM * kRowRaw;
  static constexpr int kBTile = NT * 32;
  static constexpr int kBRaw = kKC * kBTile;
  static constexpr int kScale = NT * kKC * 4;
  static constexpr int kDaOff = kARaw + kBRaw;
  static constexpr int kSumOff = kDaOff + kScale;
  static constexpr int kStage = kSumOff + kScale;
  static constexpr int kAcanOff = kRS * kStage;               // [2][kKC] canonical A tiles
  static constexpr int kBarOff = kAcanOff + 2 * kKC * kM * 32;
  static constexpr int kSlotOff = kBarOff + (2 * kRS + 8) * 8;
  static constexpr int kBytes = kSlotOff + 16;
  static constexpr uint32_t kCols = 2 * kKC * NT;             // two TMEM groups of kKC blocks
};

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
// Arrives on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase of `bar` with the given parity.  Gives up when another
// role has aborted, or after 200 ms (then aborts every role); false = give up.
__device__ __noinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = global_ns() + 200000000ull;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() > deadline) {
      *abort_flag = 1;
      return false;
    }
  }
}

// wait_phase for a whole warp: every lane gets the same answer, so the warp
// never splits around the .sync.aligned instructions that follow.
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return __all_sync(0xffffffffu, wait_phase(bar, parity, abort_flag));
}

template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[NC]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                 "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&v)[16]) {
  tmem_ld16(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&v)[32]) {
  uint32_t (&lo)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[0]);
  uint32_t (&hi)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16]);
  tmem_ld16(taddr, lo);
  tmem_ld16(taddr + 16, hi);
}

// One 18- or 34-byte block at a 2-byte aligned shared address: the 16 / 32
// quant bytes as little-endian words, reading only the block's bytes.
template <int BPB>
__device__ __forceinline__ void read_quants(const uint8_t* p, uint32_t (&q)[8]) {
  constexpr int nfull = BPB == 18 ? 4 : 8;
  if ((smem_u32(p) & 3) == 0) {
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p);
    uint32_t words[nfull + 1];
#pragma unroll
    for (int i = 0; i < nfull; ++i) words[i] = p4[i];
    words[nfull] = *reinterpret_cast<const uint16_t*>(p + 4 * nfull);
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = __funnelshift_r(words[i], words[i + 1], 16);
  } else {
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p + 2);
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = p4[i];
  }
}

template <int BPB, int NT>
__global__ void __launch_bounds__(kWsThreads, NT <= 16 ? 2 : 1)
qgemm_tc_kernel(const uint8_t* __restrict__ w, int rows, int nb, Batch b, Epilogue ep,
                unsigned int* status) {
  using L = TcLayout<BPB, NT>;
  constexpr int kHalf = NT / 2;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);  // raw chunk landed
  uint64_t* empty = full + kRS;                                        // ring stage free
  uint64_t* afull = empty + kRS;                                       // canonical A ready [2]
  uint64_t* aempty = afull + 2;                                        // canonical A free [2]
  uint64_t* tfull = aempty + 2;                                        // TMEM group ready [2]
  uint64_t* tempty = tfull + 2;                                        // TMEM group drained [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kSlotOff + 4);

  constexpr uint32_t kIdesc = (2u << 4) | ((BPB == 18 ? 0u : 1u) << 7) | (1u << 10) |
                              ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq0 = blockIdx.x * NT;
  const int row0 = blockIdx.y * kM;
  const int nseq = min(NT, b.rows - seq0);
  const size_t row_bytes = (size_t)nb * BPB;
  const int nchunks = nb / kKC;

  if (warp == kLoaderWarp) tmem_alloc(tmem_slot, L::kCols);
  if (tid == kMmaWarp * 32) {
    for (int st = 0; st < kRS; ++st) {
      mbar_init(&full[st], 32);
      mbar_init(&empty[st], kUnpackWarps + kEpiWarps);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&afull[g], kUnpackWarps);
      mbar_init(&aempty[g], 1);
      mbar_init(&tfull[g], 1);
      mbar_init(&tempty[g], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  float acc[kHalf];
#pragma unroll
  for (int s = 0; s < kHalf; ++s) acc[s] = 0.0f;
  int mma_last = -1;  // MMA lane: last chunk committed

  if (warp == kLoaderWarp) {
    for (int c = 0; c < nchunks; ++c) {
      const int st = c % kRS;
      if (!wait_warp(&empty[st], ((c / kRS) & 1) ^ 1, abort_flag)) break;
      uint8_t* sp = smem + st * L::kStage;
      const int blk0 = c * kKC;
#pragma unroll
      for (int rr = 0; rr < kM / 32; ++rr) {
        const int r = lane + 32 * rr;
        const uint8_t* src = w + (size_t)(row0 + r) * row_bytes + (size_t)blk0 * BPB;
        uint8_t* dst = sp + r * L::kRowRaw;
#pragma unroll
        for (int gch = 0; gch < kKC * BPB / 8; ++gch) cp_async8(dst + 8 * gch, src + 8 * gch);
      }
      for (int s = lane; s < NT; s += 32) {
        const bool valid = s < nseq;
        const size_t srow = valid ? (size_t)(seq0 + s) : 0;
        const int8_t* a = b.aq + srow * kActStride + (size_t)blk0 * 32;
#pragma unroll
        for (int j = 0; j < kKC; ++j) {
          cp_async16(sp + L::kARaw + j * L::kBTile + tile_off(s, 0), a + j * 32, valid);
          cp_async16(sp + L::kARaw + j * L::kBTile + tile_off(s, 1), a + j * 32 + 16, valid);
        }
        cp_async16(sp + L::kDaOff + s * kKC * 4, b.ad + srow * kActBlocks + blk0, valid);
        cp_async16(sp + L::kSumOff + s * kKC * 4, b.asum + srow * kActBlocks + blk0, valid);
      }
      cp_async_arrive(&full[st]);
    }
    cp_async_wait_all();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      for (int c = 0; c < nchunks; ++c) {
        const int g = c & 1, st = c % kRS, k2 = c >> 1;
        if (!wait_phase(&afull[g], k2 & 1, abort_flag)) break;
        if (!wait_phase(&tempty[g], (k2 & 1) ^ 1, abort_flag)) break;
        if (!wait_phase(&full[st], (c / kRS) & 1, abort_flag)) break;
        fence_async_shared();
        tc_after_sync();
        const uint8_t* bst = smem + st * L::kStage + L::kARaw;
#pragma unroll
        for (int j = 0; j < kKC; ++j) {
          const uint8_t* A = smem + L::kAcanOff + (g * kKC + j) * (kM * 32);
          mma_i8(tmem_base + (uint32_t)((g * kKC + j) * NT), smem_desc(A),
                 smem_desc(bst + j * L::kBTile), kIdesc);
        }
        mma_commit(&aempty[g]);
        mma_commit(&tfull[g]);
        mma_last = c;
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    const int u = tid - kUnpackWarp0 * 32;  // weight row of this thread
    for (int c = 0; c < nchunks; ++c) {
      const int g = c & 1, st = c % kRS, k2 = c >> 1;
      if (!wait_warp(&full[st], (c / kRS) & 1, abort_flag)) break;
      if (!wait_warp(&aempty[g], (k2 & 1) ^ 1, abort_flag)) break;
      const uint8_t* raw = smem + st * L::kStage + u * L::kRowRaw;
#pragma unroll
      for (int j = 0; j < kKC; ++j) {
        uint32_t q[8];
        read_quants<BPB>(raw + j * BPB, q);
        uint8_t* A = smem + L::kAcanOff + (g * kKC + j) * (kM * 32);
        if (BPB == 18) {
          *reinterpret_cast<uint4*>(A + tile_off(u, 0)) =
              make_uint4(q[0] & 0x0f0f0f0fu, q[1] & 0x0f0f0f0fu, q[2] & 0x0f0f0f0fu, q[3] & 0x0f0f0f0fu);
          *reinterpret_cast<uint4*>(A + tile_off(u, 1)) =
              make_uint4((q[0] >> 4) & 0x0f0f0f0fu, (q[1] >> 4) & 0x0f0f0f0fu,
                         (q[2] >> 4) & 0x0f0f0f0fu, (q[3] >> 4) & 0x0f0f0f0fu);
        } else {
          *reinterpret_cast<uint4*>(A + tile_off(u, 0)) = make_uint4(q[0], q[1], q[2], q[3]);
          *reinterpret_cast<uint4*>(A + tile_off(u, 1)) = make_uint4(q[4], q[5], q[6], q[7]);
        }
      }
      fence_async_shared();  // generic-proxy tile writes -> tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[g]);
        mbar_arrive(&empty[st]);
      }
    }
  } else {
    // Epilogue warp: TMEM lanes of its quarter (warp % 4 by the tcgen05.ld rule),
    // half of the chunk's columns, 16 columns x 4 blocks per TMEM batch.
    static_assert(kKC == 4, "float4 scale loads assume 4 blocks per chunk");
    constexpr int kSub = kHalf < 16 ? kHalf : 16;
    const int quarter = warp & 3, colhalf = (warp - kEpiWarp0) >> 2;
    const int lrow = quarter * 32 + lane;
    for (int c = 0; c < nchunks; ++c) {
      const int g = c & 1, st = c % kRS, k2 = c >> 1;
      if (!wait_warp(&tfull[g], k2 & 1, abort_flag)) break;
      if (!wait_warp(&full[st], (c / kRS) & 1, abort_flag)) break;
      tc_after_sync();
      const uint8_t* sp = smem + st * L::kStage;
      const float4* dA4 = reinterpret_cast<const float4*>(sp + L::kDaOff);
      const int4* asum4 = reinterpret_cast<const int4*>(sp + L::kSumOff);
      float dW[kKC], negMdW[kKC];
#pragma unroll
      for (int j = 0; j < kKC; ++j) {
        dW[j] = half_to_f32(*reinterpret_cast<const uint16_t*>(sp + lrow * L::kRowRaw + j * BPB));
        negMdW[j] = -__fmul_rn(12582912.0f, dW[j]);
      }
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(g * kKC * NT);
#pragma unroll
      for (int sb = 0; sb < kHalf; sb += kSub) {
        uint32_t v[kKC][kSub];
#pragma unroll
        for (int j = 0; j < kKC; ++j) tmem_ld<kSub>(tbase + (uint32_t)(j * NT + colhalf * kHalf + sb), v[j]);
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < kSub; ++jj) {
          const int s = colhalf * kHalf + sb + jj;
          const float4 da = dA4[s];
          const float dav[4] = {da.x, da.y, da.z, da.w};
          float a = acc[sb + jj];
          if (BPB == 18) {
            const int4 sm = asum4[s];
            const int smv[4] = {sm.x, sm.y, sm.z, sm.w};
#pragma unroll
            for (int j = 0; j < kKC; ++j) {
              const float x = __int_as_float((int)v[j][jj] + 0x4B400000 - 8 * smv[j]);
              a = __fadd_rn(a, __fmul_rn(__fmaf_rn(x, dW[j], negMdW[j]), dav[j]));
            }
          } else {
#pragma unroll
            for (int j = 0; j < kKC; ++j) {
              const float f = __fsub_rn(__int_as_float((int)v[j][jj] + 0x4B400000), 12582912.0f);
              a = __fadd_rn(a, __fmul_rn(f, __fmul_rn(dW[j], dav[j])));
            }
          }
          acc[sb + jj] = a;  // blocks in order per column
        }
      }
      tc_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[g]);
        mbar_arrive(&empty[st]);
      }
    }
  }

  __syncthreads();
  const bool aborted = *abort_flag != 0;
  if (aborted && warp == kMmaWarp && lane == 0 && mma_last >= 0) {
    // MMAs already committed must finish before their TMEM is released.
    const uint64_t deadline = global_ns() + 50000000ull;
    while (!mbar_try_wait(&tfull[mma_last & 1], (mma_last >> 1) & 1) && global_ns() < deadline) {
    }
  }
  if (aborted && tid == 0) atomicOr(status, 1u);
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (warp == kLoaderWarp) tmem_dealloc(tmem_base, L::kCols);
  if (aborted || warp < kEpiWarp0) return;

  const int row = row0 + (warp & 3) * 32 + lane;
  const int colhalf = (warp - kEpiWarp0) >> 2;
#pragma unroll
  for (int jj = 0; jj < kHalf; ++jj) {
    const int s = colhalf * kHalf + jj;
    if (s < nseq) {
      const int seq = seq0 + s;
      float* dst = ep.out + (size_t)seq * ep.ld + row;
      float v;
      if (ep.mode == EPI_BIAS) v = __fadd_rn(acc[jj], ep.bias[row]);
      else if (ep.mode == EPI_RESIDUAL) v = __fadd_rn(*dst, acc[jj]);
      else v = acc[jj];
      *dst = v;
      check_finite(v, &ep.err[seq], ep.layer_ordinal, ep.domain, 0, row);
    }
  }
}

template <int BPB, int NT>
void launch_tc(const uint8_t* w, int rows, int nb, const Batch& b, const Epilogue& ep,
               unsigned int* status, cudaStream_t s) {
  static bool configured = false;  // one device per process
  if (!configured) {
    cudaFuncSetAttribute(qgemm_tc_kernel<BPB, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         TcLayout<BPB, NT>::kBytes);
    configured = true;
  }
  dim3 grid((b.rows + NT - 1) / NT, rows / kM);
  qgemm_tc_kernel<BPB, NT><<<grid, kWsThreads, TcLayout<BPB, NT>::kBytes, s>>>(w, rows, nb, b, ep,
                                                                              status);
}

}  // namespace

bool qgemm_tc_supported(int rows, int batch, int columns) {
  return rows % kM == 0 && batch > 8 && (columns / 32) % kKC == 0;
}

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
