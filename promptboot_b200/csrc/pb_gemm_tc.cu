// Batched block-scaled matvec on the 5th-generation tensor cores (tcgen05,
// kind::i8) for sm_100a: Y[s][r] = sum over Q-blocks k IN ORDER of the
// reference's per-block term (fp32_sse2.rs:1217-1281), for B > 8 sequences.
//
// Operands come from two device images built for this kernel:
//  * the weight TILE IMAGE (built once per model by tc_repack_kernel): for each
//    128-row tile and each chunk of 4 Q-blocks, 18432 contiguous bytes = four
//    canonical K-major int8 tiles (Q4_0 nibbles already shifted to q - 8, Q8_0
//    quants as stored) followed by the 128 x 4 binary32 block scales;
//  * the activation TILE LAYOUT written by the Q8_0 quantizers beside the
//    row-major one: quants as [seq / 8][block][256 B] (two 8 x 16-byte core
//    matrices per block) and scales as [block][seq].
// So every chunk arrives with 1 + NT/8 + 4 bulk copies (cp.async.bulk, no
// multicast) on one transaction-count mbarrier, issued by one thread.
//
// One tcgen05.mma per Q-block: M = 128 weight rows, N = NT sequences, K = 32,
// both operands signed.  TMEM columns are preloaded with 0x4B400000 and the MMA
// accumulates into them, so each column reads back as the binary32 bit pattern
// of 1.5 * 2^23 + i (exact for |i| < 2^22; |i| <= 2^19 here); the epilogue
// writes the constant back after reading.  Epilogue per (row, sequence, block),
// on packed f32x2 operations (two sequences per instruction, IEEE RN per lane;
// the assembler fuses a packed multiply into a following packed add even with
// explicit rounding, so each rounded product is an fma with a run-time -0.0
// addend):
//   Q4_0: t = fl(fl(i * dW) * dA), with fl(i * dW) = fma(x, dW, -1.5*2^23*dW)
//         exact because 1.5 * 2^23 * dW is representable for binary16 dW
//   Q8_0: t = fl(f32(i) * fl(dW * dA)), f32(i) = x - 1.5*2^23 exactly
//   acc = fl(acc + t), blocks in order per (row, sequence).
//
// Warp roles, chained by mbarriers only: warp 0 allocates TMEM and its lane 0
// issues the bulk copies into a ring of stages; warp 1 lane 0 issues the four
// MMAs of a chunk into one of two TMEM groups and commits; NT/4 epilogue warps
// (TMEM lane quarter = warp % 4, 16 columns each) drain a group and release its
// stage.  Every wait is bounded (200 ms on %globaltimer, or another role's
// abort); an abort sets *status, lets copies and MMAs in flight finish
// (bounded), frees TMEM and returns.
#include "pb_common.cuh"
#include "pb_kernels.cuh"

#include <cstdlib>

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
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Global -> shared bulk copy completing `bytes` transactions on `bar`.  Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
// D[tmem] += A * B (accumulates into the preloaded columns).
__device__ __forceinline__ void mma_i8_acc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc) {
  const uint32_t one = 1, zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(one), "r"(zero)
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
// Writes one 32-bit value to 16 consecutive columns of the warp's 32 lanes.
__device__ __forceinline__ void tmem_st16_same(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
          taddr),
      "r"(x)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// K-major, no swizzle: leading byte offset (between the two 16-byte K halves)
// 128 B, stride byte offset (between 8-row groups) `sbo`, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t sbo) {
  uint64_t a = (smem_u32(p) >> 4) & 0x3fffu;
  return a | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) | (1ull << 46);
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
// Drain wait used on the way out: bounded by `ns`, ignores the abort flag.
__device__ __noinline__ void wait_drain(uint64_t* bar, uint32_t parity, uint64_t ns) {
  const uint64_t deadline = global_ns() + ns;
  while (!mbar_try_wait(bar, parity) && global_ns() < deadline) {
  }
}

// Packed binary32 pairs (sm_100 f32x2 instructions, round to nearest even per lane).
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t pk_u(uint32_t lo, uint32_t hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ void unpk(uint64_t x, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(x));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

constexpr int kM = 128;            // weight rows per tile (MMA M)
constexpr int kKC = 4;             // Q-blocks per chunk = MMAs per commit
constexpr int kATile = kM * 32;    // one canonical 128 x 32 int8 tile
constexpr int kDwOff = kKC * kATile;
constexpr uint32_t kMagic = 0x4B400000u;  // binary32 1.5 * 2^23
static_assert(kDwOff + kM * kKC * 4 == kTcChunkBytes, "tile image chunk size");

template <int NT>
struct TcCfg {
  static constexpr int kEpiWarps = NT / 4;  // 4 lane quarters x NT/16 column groups
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kStages = NT == 64 ? 6 : 4;
  static constexpr int kBOff = kTcChunkBytes;          // [NT/8][4 blocks][256 B]
  static constexpr int kDaOff = kBOff + NT * 128;      // [4 blocks][NT] f32
  static constexpr int kStage = kDaOff + NT * 16;
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kBytes = kBarOff + (2 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kCols = 2 * kKC * NT;      // two TMEM groups of 4 blocks
  static_assert(kStage % 128 == 0, "stage alignment");
};

template <bool Q4, int NT>
__global__ void __launch_bounds__(TcCfg<NT>::kThreads, NT == 64 ? 1 : 2)
qgemm_tc_kernel(TcGemm g, Batch b, unsigned int* status) {
  using C = TcCfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // stage landed
  uint64_t* empty = full + S;                                         // stage drained
  uint64_t* tfull = empty + S;                                        // TMEM group ready [2]
  uint64_t* tempty = tfull + 2;                                       // TMEM group drained [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // kind::i8 instruction descriptor: s32 accumulator, A and B signed, K-major,
  // N = NT, M = 128.
  constexpr uint32_t kIdesc =
      (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq0 = blockIdx.x * NT;
  const int rt = blockIdx.y;
  const int nseq = min(NT, b.rows - seq0);
  const int nchunks = g.nb / kKC;
  const int quarter = warp & 3, cg = (warp - 2) >> 2;  // epilogue warps only

  if (warp == 0) tmem_alloc(tmem_slot, C::kCols);
  if (tid == 32) {
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], C::kEpiWarps);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(&tfull[k], 1);
      mbar_init(&tempty[k], C::kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tlane = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(cg * 16);
  if (warp >= 2) {
#pragma unroll
    for (int k = 0; k < 2 * kKC; ++k) tmem_st16_same(tlane + (uint32_t)(k * NT), kMagic);
    tmem_wait_st();
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();

  uint64_t acc[8];  // epilogue: 16 columns as 8 packed pairs
#pragma unroll
  for (int p = 0; p < 8; ++p) acc[p] = 0;
  int mma_last = -1;

  if (warp == 0) {
    if (lane == 0) {
      const uint8_t* wt = g.tiles + (size_t)rt * nchunks * kTcChunkBytes;
      const int8_t* bq = b.aq_tc + (size_t)(seq0 >> 3) * g.nb * 256;
      const float* da = b.ad_tc + seq0;
      int load_last = -1;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % S;
        if (!wait_phase(&empty[st], ((c / S) & 1) ^ 1, abort_flag)) break;
        uint8_t* sp = smem + st * C::kStage;
        mbar_expect_tx(&full[st], C::kStage);
        bulk_g2s(sp, wt + (size_t)c * kTcChunkBytes, kTcChunkBytes, &full[st]);
#pragma unroll
        for (int rg = 0; rg < NT / 8; ++rg)
          bulk_g2s(sp + C::kBOff + rg * 1024, bq + ((size_t)rg * g.nb + c * kKC) * 256, 1024, &full[st]);
#pragma unroll
        for (int j = 0; j < kKC; ++j)
          bulk_g2s(sp + C::kDaOff + j * NT * 4, da + (size_t)(c * kKC + j) * b.tc_seqs, NT * 4,
                   &full[st]);
        load_last = c;
      }
      // Every issued copy lands before the CTA may exit.
      for (int c = max(0, load_last - S + 1); c <= load_last; ++c)
        wait_drain(&full[c % S], (c / S) & 1, 50000000ull);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      for (int c = 0; c < nchunks; ++c) {
        const int gr = c & 1, st = c % S, k2 = c >> 1;
        if (!wait_phase(&tempty[gr], (k2 & 1) ^ 1, abort_flag)) break;
        if (!wait_phase(&full[st], (c / S) & 1, abort_flag)) break;
        tc_after_sync();
        const uint8_t* sp = smem + st * C::kStage;
#pragma unroll
        for (int j = 0; j < kKC; ++j)
          mma_i8_acc(tmem_base + (uint32_t)((gr * kKC + j) * NT), smem_desc(sp + j * kATile, 256),
                     smem_desc(sp + C::kBOff + j * 256, 1024), kIdesc);
        mma_commit(&tfull[gr]);
        mma_last = c;
      }
    }
    __syncwarp();
  } else {
    const int lrow = quarter * 32 + lane;
    const uint64_t neg_magic2 = pk(-12582912.0f, -12582912.0f);
    const float nz = __uint_as_float(g.neg_zero_bits);
    const uint64_t z2 = pk(nz, nz);
    for (int c = 0; c < nchunks; ++c) {
      const int gr = c & 1, st = c % S, k2 = c >> 1;
      if (!wait_warp(&tfull[gr], k2 & 1, abort_flag)) break;
      if (!wait_warp(&full[st], (c / S) & 1, abort_flag)) break;
      tc_after_sync();
      const uint8_t* sp = smem + st * C::kStage;
      const float4 dw4 = *reinterpret_cast<const float4*>(sp + kDwOff + lrow * 16);
      const float dw[kKC] = {dw4.x, dw4.y, dw4.z, dw4.w};
      const uint32_t tg = tlane + (uint32_t)(gr * kKC * NT);
      const float* dA = reinterpret_cast<const float*>(sp + C::kDaOff) + cg * 16;
      // Two blocks per TMEM batch keeps the live registers low; every
      // (row, sequence) still adds its blocks in order j = 0, 1, 2, 3.
#pragma unroll
      for (int jb = 0; jb < kKC; jb += 2) {
        uint32_t v[2][16];
        tmem_ld16(tg + (uint32_t)(jb * NT), v[0]);
        tmem_ld16(tg + (uint32_t)((jb + 1) * NT), v[1]);
        tmem_wait_ld();
        tmem_st16_same(tg + (uint32_t)(jb * NT), kMagic);
        tmem_st16_same(tg + (uint32_t)((jb + 1) * NT), kMagic);
        uint64_t w2[2], n2[2];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          w2[jj] = pk(dw[jb + jj], dw[jb + jj]);
          const float nm = -__fmul_rn(12582912.0f, dw[jb + jj]);
          n2[jj] = pk(nm, nm);
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          uint64_t a = acc[p];
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const uint64_t da2 = *reinterpret_cast<const uint64_t*>(dA + (jb + jj) * NT + 2 * p);
            const uint64_t x2 = pk_u(v[jj][2 * p], v[jj][2 * p + 1]);
            uint64_t t;
            if (Q4) {
              t = fma2(fma2(x2, w2[jj], n2[jj]), da2, z2);
            } else {
              t = fma2(add2(x2, neg_magic2), mul2(w2[jj], da2), z2);
            }
            a = add2(a, t);
          }
          acc[p] = a;
        }
      }
      tmem_wait_st();
      tc_before_sync();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[gr]);
        mbar_arrive(&empty[st]);
      }
    }
  }

  __syncthreads();
  const bool aborted = *abort_flag != 0;
  if (aborted && warp == 1 && lane == 0 && mma_last >= 0)
    wait_drain(&tfull[mma_last & 1], (mma_last >> 1) & 1, 50000000ull);  // committed MMAs finish
  if (aborted && tid == 0) atomicOr(status, 1u);
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (warp == 0) tmem_dealloc(tmem_base, C::kCols);
  if (aborted || warp < 2) return;

  int si = 0;
  while (si + 1 < g.nseg && rt >= g.seg[si].rtile_end) ++si;
  const Epilogue& ep = g.seg[si].ep;
  const int row = (rt - (si ? g.seg[si - 1].rtile_end : 0)) * kM + quarter * 32 + lane;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    float pair[2];
    unpk(acc[p], pair[0], pair[1]);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = cg * 16 + 2 * p + h;
      if (s < nseq) {
        const int seq = seq0 + s;
        float* dst = ep.out + (size_t)seq * ep.ld + row;
        float y;
        if (ep.mode == EPI_BIAS) y = __fadd_rn(pair[h], ep.bias[row]);
        else if (ep.mode == EPI_RESIDUAL) y = __fadd_rn(*dst, pair[h]);
        else y = pair[h];
        *dst = y;
        check_finite(y, &ep.err[seq], ep.layer_ordinal, ep.domain, 0, row);
      }
    }
  }
}

template <bool Q4, int NT>
void launch_tc(const TcGemm& g, const Batch& b, unsigned int* status, cudaStream_t s) {
  using C = TcCfg<NT>;
  static bool configured = false;  // one device per process
  if (!configured) {
    cudaFuncSetAttribute(qgemm_tc_kernel<Q4, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
    configured = true;
  }
  dim3 grid((b.rows + NT - 1) / NT, g.rtiles);
  qgemm_tc_kernel<Q4, NT><<<grid, C::kThreads, C::kBytes, s>>>(g, b, status);
}

// Tile image of one matrix: grid (chunks, row tiles), thread = row of the tile.
template <int BPB>
__global__ void tc_repack_kernel(const uint8_t* __restrict__ w, int nb, uint8_t* __restrict__ out) {
  const int c = blockIdx.x, rt = blockIdx.y, r = threadIdx.x;
  const int nchunks = nb / kKC;
  const uint8_t* src = w + ((size_t)rt * kM + r) * nb * BPB + (size_t)c * kKC * BPB;
  uint8_t* tile = out + ((size_t)rt * nchunks + c) * kTcChunkBytes;
  float* scales = reinterpret_cast<float*>(tile + kDwOff);
#pragma unroll
  for (int j = 0; j < kKC; ++j) {
    const uint8_t* blk = src + j * BPB;
    scales[r * kKC + j] = half_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    uint8_t* a = tile + j * kATile + (r >> 3) * 256 + (r & 7) * 16;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      int q;
      if (BPB == 18) q = (e < 16 ? (blk[2 + e] & 15) : (blk[2 + e - 16] >> 4)) - 8;
      else q = (int)(int8_t)blk[2 + e];
      a[(e >> 4) * 128 + (e & 15)] = (uint8_t)(int8_t)q;
    }
  }
}

}  // namespace

bool tc_shape_supported(int rows, int columns) {
  return rows % kM == 0 && columns % (32 * kKC) == 0;
}

size_t tc_image_bytes(int rows, int columns) {
  return (size_t)(rows / kM) * (size_t)(columns / (32 * kKC)) * kTcChunkBytes;
}

void launch_tc_repack(int wtype, const uint8_t* w, int rows, int columns, uint8_t* out,
                      cudaStream_t s) {
  const int nb = columns / 32;
  dim3 grid(nb / kKC, rows / kM);
  if (wtype == W_Q4_0) tc_repack_kernel<18><<<grid, kM, 0, s>>>(w, nb, out);
  else tc_repack_kernel<34><<<grid, kM, 0, s>>>(w, nb, out);
}

// Picks the sequence tile NT (16, 32 or 64 sequences) with the smallest
// estimated time: tile waves over the SM slots the tile's TMEM and shared
// memory allow, times the per-tile epilogue work (grows with NT) plus a fixed
// per-tile cost.  The weight row tile is the slow grid dimension so the CTAs
// sharing it run together (one HBM read).  PB_TC_TILE=16|32|64 in the
// environment forces a width (tests cover every width; tuning sweeps).
int tc_pick_tile(int rtiles, int batch) {
  if (const char* f = std::getenv("PB_TC_TILE")) {
    const int nt = std::atoi(f);
    if (nt == 16 || nt == 32 || nt == 64) return nt;
  }
  static const int kSms = [] {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
  }();
  const int nts[3] = {64, 32, 16};
  const int per_sm[3] = {1, 2, 2};
  int best = 16;
  double best_cost = 1e30;
  for (int i = 0; i < 3; ++i) {
    const int nt = nts[i];
    const long tiles = (long)rtiles * ((batch + nt - 1) / nt);
    const long slots = (long)kSms * per_sm[i];
    const long waves = (tiles + slots - 1) / slots;
    const double cost = (double)waves * (nt + 16) / per_sm[i];
    if (cost < best_cost) {
      best_cost = cost;
      best = nt;
    }
  }
  return best;
}

void launch_tc_gemm(const TcGemm& g, const Batch& b, unsigned int* status, cudaStream_t s) {
  const int nt = tc_pick_tile(g.rtiles, b.rows);
  if (g.wtype == W_Q4_0) {
    if (nt == 64) launch_tc<true, 64>(g, b, status, s);
    else if (nt == 32) launch_tc<true, 32>(g, b, status, s);
    else launch_tc<true, 16>(g, b, status, s);
  } else {
    if (nt == 64) launch_tc<false, 64>(g, b, status, s);
    else if (nt == 32) launch_tc<false, 32>(g, b, status, s);
    else launch_tc<false, 16>(g, b, status, s);
  }
}

}  // namespace pb
