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
//    row-major one, chunk-major: per chunk and 8 sequences, 4 blocks x 256 B
//    of quants (two 8 x 16-byte core matrices per block) then their
//    [4 blocks][8 sequences] binary32 scales (1152 B, the B operand's 8-row
//    group stride).
// So every chunk arrives with two bulk copies (cp.async.bulk, no multicast) on
// one transaction-count mbarrier, issued by one thread.
//
// One tcgen05.mma per Q-block: M = 128 weight rows, N = NT sequences, K = 32,
// both operands signed, without accumulation: each block's int32 dot i lands on
// its own TMEM columns, and the epilogue adds 0x4B400000 to the word as an
// integer, giving the binary32 bit pattern of 1.5 * 2^23 + i (exact for
// |i| < 2^22; |i| <= 2^19 here).  Epilogue per (row, sequence, block),
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

#include <algorithm>
#include <cstdlib>
#include <type_traits>

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
// D[tmem] = A * B (enable-input-d false: each block's dot lands on its own
// columns, no accumulation).
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%4, %4, %4, %4}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(zero)
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
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Slow path of wait_phase: polls with a 20 us suspend hint; gives up when
// another role has aborted, or after 200 ms (then aborts every role).
__device__ __noinline__ bool wait_phase_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint64_t deadline = global_ns() + 200000000ull;
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() > deadline) {
      *abort_flag = 1;
      return false;
    }
  }
}
// Waits for the phase of `bar` with the given parity; false = give up.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_phase_slow(bar, parity, abort_flag);
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

// Kernel configurations: NT = MMA N, SEQ <= NT sequences per tile (a half-filled
// N=16 MMA doubles the tiles of matrices with few row tiles), CPW TMEM columns
// per epilogue warp (4 lane quarters x SEQ / CPW column groups), PER_SM resident CTAs per SM
// (shared memory, TMEM columns and registers sized for that count), STAGES ring
// depth.  Wide tiles for many tiles per SM, narrow tiles with many epilogue
// warps when there are about as many tiles as SMs (latency-bound).
template <int NT_, int CPW_, int PER_SM_, int STAGES_, int GROUPS_, int SEQ_ = NT_>
struct TcCfg {
  static constexpr int NT = NT_;    // MMA N (TMEM columns per block)
  static constexpr int SEQ = SEQ_;  // sequences per tile (<= NT; rows SEQ..NT-1 of B unused)
  static constexpr int kCpw = CPW_;
  static constexpr int kEpiWarps = 4 * SEQ / kCpw;
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kPerSm = PER_SM_;
  static constexpr int kStages = STAGES_;
  // TMEM groups of 4 block dots: the MMA runs up to kGroups - 1 chunks ahead of
  // the epilogue, hiding the MMA issue-to-commit latency.
  static constexpr int kGroups = GROUPS_;
  // Q-blocks per TMEM load batch (up to 32 registers of block dots per thread:
  // the whole chunk, one load wait, for 8-column epilogue warps).
  static constexpr int kBatch = kCpw * kKC <= 32 ? kKC : 2;
  static constexpr int kBOff = kTcChunkBytes;  // [NT/8] groups of kTcGroupBytes
  static constexpr int kStage = kBOff + (NT / 8) * kTcGroupBytes;
  static constexpr uint32_t kTxBytes = kTcChunkBytes + (SEQ / 8) * kTcGroupBytes;  // per chunk
  static constexpr int kBarOff = kStages * kStage;
  static constexpr int kBytes = kBarOff + (2 * kStages + 2 * kGroups) * 8 + 16;
  static constexpr uint32_t kCols = kGroups * kKC * NT;
  static_assert(kStage % 128 == 0, "stage alignment");
  static_assert(kCpw == 4 || kCpw == 8 || kCpw == 16, "epilogue column batch");
  static_assert(kThreads <= 1024, "block size");
  static_assert(SEQ % 8 == 0 && SEQ <= NT && SEQ % kCpw == 0, "sequence tile");
  static_assert(kPerSm * kCols <= 512, "TMEM columns per SM");
  static_assert((kCols & (kCols - 1)) == 0 && kCols >= 32, "TMEM allocation size");
  static_assert(kPerSm * (kBytes + 1024) <= 233472, "shared memory per SM");
};
using Cfg8 = TcCfg<16, 8, 2, 5, 2, 8>;
using Cfg16 = TcCfg<16, 8, 2, 4, 4>;
using Cfg32 = TcCfg<32, 16, 2, 4, 2>;
using Cfg64 = TcCfg<64, 16, 1, 6, 2>;

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, uint32_t (&v)[16]) {
  tmem_ld16(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld_cols<8>(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                 "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cols<4>(uint32_t taddr, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr)
               : "memory");
}
// Persistent: CTA i serves tiles i, i + G, i + 2G, ... (G = gridDim.x) of the
// (row tile, sequence tile) grid, sequence tile fastest, so CTAs running at the
// same time share weight tiles in L2; the ring, the MMA issue and the TMEM
// groups run on one chunk counter across tile boundaries.
template <bool Q4, class C>
__global__ void __launch_bounds__(C::kThreads, C::kPerSm)
qgemm_tc_kernel(TcGemm g, Batch b, unsigned int* status) {
  // Programmatic dependent launch: the loader prefetches the first stages' weight
  // tiles (written once at model open) before waiting for the previous kernel;
  // the epilogue warps wait before touching activations and outputs; the MMA
  // warp touches no global memory.
  pdl_trigger();
  constexpr int NT = C::NT;
  constexpr int SEQ = C::SEQ;
  constexpr int S = C::kStages;
  constexpr int CPW = C::kCpw;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // stage landed
  uint64_t* empty = full + S;                                         // stage drained
  constexpr int G = C::kGroups;
  uint64_t* tfull = empty + S;                                        // TMEM group ready [G]
  uint64_t* tempty = tfull + G;                                       // TMEM group drained [G]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + G);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // kind::i8 instruction descriptor: s32 accumulator, A and B signed, K-major,
  // N = NT, M = 128.
  constexpr uint32_t kIdesc =
      (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nchunks = g.nb / kKC;
  const int nst = (b.rows + SEQ - 1) / SEQ;  // sequence tiles
  const int ntiles = g.rtiles * nst;
  const int quarter = warp & 3, cg = (warp - 2) >> 2;  // epilogue warps only

  if (warp == 0) tmem_alloc(tmem_slot, C::kCols);
  if (tid == 32) {
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], C::kEpiWarps);
    }
    for (int k = 0; k < G; ++k) {
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
  const uint32_t tlane = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(cg * CPW);
  tc_before_sync();
  __syncthreads();
  tc_after_sync();

  int mma_last = -1;

  if (warp == 0) {
    if (lane == 0) {
      int q = 0, load_last = -1;
      bool stop = false;
      // Weight tiles of the first stages of this CTA's first tile.
      const int pre = blockIdx.x < ntiles ? min(S, nchunks) : 0;
      if (pre > 0) {
        const uint8_t* wt0 = g.tiles + (size_t)(blockIdx.x / nst) * nchunks * kTcChunkBytes;
        for (int c = 0; c < pre; ++c) {
          mbar_expect_tx(&full[c], C::kTxBytes);
          bulk_g2s(smem + c * C::kStage, wt0 + (size_t)c * kTcChunkBytes, kTcChunkBytes, &full[c]);
        }
      }
      pdl_wait();
      for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x) {
        const int rt = tile / nst, seq0 = (tile % nst) * SEQ;
        const uint8_t* wt = g.tiles + (size_t)rt * nchunks * kTcChunkBytes;
        for (int c = 0; c < nchunks; ++c, ++q) {
          const int st = q % S;
          uint8_t* sp = smem + st * C::kStage;
          if (q >= pre) {
            if (!wait_phase(&empty[st], ((q / S) & 1) ^ 1, abort_flag)) {
              stop = true;
              break;
            }
            mbar_expect_tx(&full[st], C::kTxBytes);
            bulk_g2s(sp, wt + (size_t)c * kTcChunkBytes, kTcChunkBytes, &full[st]);
          }
          bulk_g2s(sp + C::kBOff,
                   b.aq_tc + ((size_t)c * (b.tc_seqs >> 3) + (seq0 >> 3)) * kTcGroupBytes,
                   (SEQ / 8) * kTcGroupBytes, &full[st]);
          load_last = q;
        }
      }
      if (pre > load_last + 1) load_last = pre - 1;  // prefetched stages still land
      // Every issued copy lands before the CTA may exit.
      for (int k = max(0, load_last - S + 1); k <= load_last; ++k)
        wait_drain(&full[k % S], (k / S) & 1, 50000000ull);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int q = 0;
      bool stop = false;
      for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x) {
        for (int c = 0; c < nchunks; ++c, ++q) {
          const int gr = q % G, st = q % S, k2 = q / G;
          if (!wait_phase(&tempty[gr], (k2 & 1) ^ 1, abort_flag) ||
              !wait_phase(&full[st], (q / S) & 1, abort_flag)) {
            stop = true;
            break;
          }
          tc_after_sync();
          const uint8_t* sp = smem + st * C::kStage;
#pragma unroll
          for (int j = 0; j < kKC; ++j)
            mma_i8(tmem_base + (uint32_t)((gr * kKC + j) * NT), smem_desc(sp + j * kATile, 256),
                   smem_desc(sp + C::kBOff + j * 256, kTcGroupBytes), kIdesc);
          mma_commit(&tfull[gr]);
          mma_last = q;
        }
      }
    }
    __syncwarp();
  } else {
    pdl_wait();
    const int lrow = quarter * 32 + lane;
    const uint64_t neg_magic2 = pk(-12582912.0f, -12582912.0f);
    const float nz = __uint_as_float(g.neg_zero_bits);
    const uint64_t z2 = pk(nz, nz);
    int q = 0;
    bool stop = false;
    for (int tile = blockIdx.x; tile < ntiles && !stop; tile += gridDim.x) {
      uint64_t acc[CPW / 2];
#pragma unroll
      for (int p = 0; p < CPW / 2; ++p) acc[p] = 0;
      for (int c = 0; c < nchunks; ++c, ++q) {
        const int gr = q % G, st = q % S, k2 = q / G;
        if (!wait_warp(&tfull[gr], k2 & 1, abort_flag) || !wait_warp(&full[st], (q / S) & 1, abort_flag)) {
          stop = true;
          break;
        }
        tc_after_sync();
        const uint8_t* sp = smem + st * C::kStage;
        const float4 dw4 = *reinterpret_cast<const float4*>(sp + kDwOff + lrow * 16);
        const float dw[kKC] = {dw4.x, dw4.y, dw4.z, dw4.w};
        const uint32_t tg = tlane + (uint32_t)(gr * kKC * NT);
        // dA of (block j, column s): group s / 8, float 256 + 8 j + s % 8.
        const int s0 = cg * CPW;
        // kBatch blocks per TMEM load batch; every (row, sequence) still adds
        // its blocks in order j = 0, 1, 2, 3.
        constexpr int BT = C::kBatch;
#pragma unroll
        for (int jb = 0; jb < kKC; jb += BT) {
          uint32_t v[BT][CPW];
#pragma unroll
          for (int jj = 0; jj < BT; ++jj) tmem_ld_cols<CPW>(tg + (uint32_t)((jb + jj) * NT), v[jj]);
          tmem_wait_ld();
          uint64_t w2[BT], n2[BT];
          bool exact_fma = true;  // Q4_0: fma(x, dW, -1.5*2^23*dW) needs a finite dW
#pragma unroll
          for (int jj = 0; jj < BT; ++jj) {
            w2[jj] = pk(dw[jb + jj], dw[jb + jj]);
            const float nm = -__fmul_rn(12582912.0f, dw[jb + jj]);
            n2[jj] = pk(nm, nm);
            exact_fma = exact_fma && finite_bits(__float_as_uint(dw[jb + jj]));
          }
          exact_fma = __all_sync(0xffffffffu, exact_fma);
          // Warp-uniform choice of the Q4_0 product form (two unrolled copies).
          auto accumulate = [&](auto fast) {
#pragma unroll
            for (int p = 0; p < CPW / 2; ++p) {
              uint64_t a = acc[p];
#pragma unroll
              for (int jj = 0; jj < BT; ++jj) {
                const int s = s0 + 2 * p;
                const uint64_t da2 = *reinterpret_cast<const uint64_t*>(
                    sp + C::kBOff + (s >> 3) * kTcGroupBytes + 1024 + ((jb + jj) * 8 + (s & 7)) * 4);
                // bits of 1.5 * 2^23 + i, exactly, for the block dot i (|i| < 2^22)
                const uint64_t x2 = pk_u(v[jj][2 * p] + kMagic, v[jj][2 * p + 1] + kMagic);
                uint64_t t;
                if (Q4) {
                  // Non-finite dW (never in a sane image): fl(f32(i) * dW) with
                  // f32(i) = x - 1.5*2^23 exactly, as the reference computes it.
                  const uint64_t idw = decltype(fast)::value ? fma2(x2, w2[jj], n2[jj])
                                                             : fma2(add2(x2, neg_magic2), w2[jj], z2);
                  t = fma2(idw, da2, z2);
                } else {
                  t = fma2(add2(x2, neg_magic2), mul2(w2[jj], da2), z2);
                }
                a = add2(a, t);
              }
              acc[p] = a;
            }
          };
          if (!Q4 || exact_fma) accumulate(std::true_type{});
          else accumulate(std::false_type{});
        }
        tc_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[gr]);
          mbar_arrive(&empty[st]);
        }
      }
      if (stop) break;
      // Tile done: epilogue stores for rows of this warp's lane quarter.
      const int rt = tile / nst, seq0 = (tile % nst) * SEQ;
      const int nseq = min(SEQ, b.rows - seq0);
      int si = 0;
      while (si + 1 < g.nseg && rt >= g.seg[si].rtile_end) ++si;
      const Epilogue& ep = g.seg[si].ep;
      const int row = (rt - (si ? g.seg[si - 1].rtile_end : 0)) * kM + lrow;
#pragma unroll
      for (int p = 0; p < CPW / 2; ++p) {
        float pair[2];
        unpk(acc[p], pair[0], pair[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int s = cg * CPW + 2 * p + h;
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
  }

  __syncthreads();
  const bool aborted = *abort_flag != 0;
  if (aborted && warp == 1 && lane == 0 && mma_last >= 0)
    wait_drain(&tfull[mma_last % G], (mma_last / G) & 1, 50000000ull);  // committed MMAs finish
  if (aborted && tid == 0) atomicOr(status, 1u);
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (warp == 0) tmem_dealloc(tmem_base, C::kCols);
}

template <bool Q4, class C>
void launch_tc(const TcGemm& g, const Batch& b, unsigned int* status, cudaStream_t s, int sms) {
  static std::atomic<uint64_t> configured{0};
  if (attribute_needed(configured)) {
    cudaFuncSetAttribute(qgemm_tc_kernel<Q4, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
    attribute_done(configured);
  }
  const int tiles = g.rtiles * ((b.rows + C::SEQ - 1) / C::SEQ);
  const int grid = std::min(tiles, sms * C::kPerSm);
  launch_pdl(qgemm_tc_kernel<Q4, C>, grid, C::kThreads, C::kBytes, s, g, b, status);
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

namespace {
int sm_count() {
  static const int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}
}  // namespace

// Configuration choice (0 Cfg8, 1 Cfg16, 2 Cfg32, 3 Cfg64), from measurements
// at 256 sequences: wide tiles re-read each weight tile fewer times, which pays
// once there are several tiles per SM slot (the output head); narrow tiles
// spread matrices with few row tiles (q/k/v, o, down) over more SMs.
// PB_TC_TILE=8|16|32|64 in the environment forces one (tests cover every
// configuration; tuning sweeps).
int tc_pick_config(int rtiles, int batch) {
  if (const char* f = std::getenv("PB_TC_TILE")) {
    const int nt = std::atoi(f);
    if (nt == 8) return 0;
    if (nt == 16) return 1;
    if (nt == 32) return 2;
    if (nt == 64) return 3;
  }
  const long sms = sm_count();
  if ((long)rtiles * ((batch + 15) / 16) <= sms) return 0;
  if ((long)rtiles * ((batch + 63) / 64) >= 4 * sms) return 3;
  if ((long)rtiles * ((batch + 31) / 32) >= Cfg32::kPerSm * sms) return 2;
  return 1;
}

void launch_tc_gemm(const TcGemm& g, const Batch& b, unsigned int* status, cudaStream_t s) {
  const int cfg = tc_pick_config(g.rtiles, b.rows);
  const int sms = sm_count();
  if (g.wtype == W_Q4_0) {
    if (cfg == 0) launch_tc<true, Cfg8>(g, b, status, s, sms);
    else if (cfg == 1) launch_tc<true, Cfg16>(g, b, status, s, sms);
    else if (cfg == 2) launch_tc<true, Cfg32>(g, b, status, s, sms);
    else launch_tc<true, Cfg64>(g, b, status, s, sms);
  } else {
    if (cfg == 0) launch_tc<false, Cfg8>(g, b, status, s, sms);
    else if (cfg == 1) launch_tc<false, Cfg16>(g, b, status, s, sms);
    else if (cfg == 2) launch_tc<false, Cfg32>(g, b, status, s, sms);
    else launch_tc<false, Cfg64>(g, b, status, s, sms);
  }
}

}  // namespace pb
