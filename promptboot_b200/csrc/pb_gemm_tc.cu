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
// Operands stream in through a 4-stage cp.async ring of 4-block chunks: raw
// weight bytes (8-byte granules; 18- and 34-byte blocks are only 2-byte
// aligned) are unpacked by the threads into the canonical A tile, while the
// activation rows are scattered by 16-byte cp.async straight into the canonical
// B layout.  Every mbarrier wait is bounded; a timeout sets *status, stops
// issuing, waits (bounded) for work in flight, frees TMEM and returns.
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

constexpr int kKC = 4;     // Q-blocks per cp.async chunk = MMAs per commit group
constexpr int kRS = 4;     // chunk ring stages
constexpr int kWarps = 16;     // four warps per TMEM lane quarter ...
constexpr int kColGroups = 4;  // ... each draining a quarter of the columns

template <int BPB, int NT>
struct TcLayout {
  static constexpr int kRowRaw = ((kKC * BPB + 15) / 16) * 16;  // 80 (Q4_0) / 144 (Q8_0)
  static constexpr int kARaw = kM * kRowRaw;
  static constexpr int kBTile = NT * 32;
  static constexpr int kBRaw = kKC * kBTile;
  static constexpr int kScale = NT * kKC * 4;
  static constexpr int kDaOff = kARaw + kBRaw;
  static constexpr int kCOff = kDaOff + kScale;
  static constexpr int kStage = kCOff + kScale;
  static constexpr int kAcanOff = kRS * kStage;                  // [2][kKC] canonical A tiles
  static constexpr int kDwOff = kAcanOff + 2 * kKC * kM * 32;    // [2][kKC][128] dW, -1.5*2^23*dW
  static constexpr int kMiscOff = kDwOff + 2 * 2 * kKC * kM * 4;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr uint32_t kCols = 2 * kKC * NT;                // two TMEM groups of kKC blocks
};

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[NC]);
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr)
               : "memory");
}
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

// One 18- or 34-byte block at a 2-byte aligned shared address: binary16 scale
// bits and the 16 / 32 quant bytes as little-endian words, reading only its bytes.
template <int BPB>
__device__ __forceinline__ void read_block(const uint8_t* p, uint32_t& scale_bits, uint32_t (&q)[8]) {
  constexpr int nfull = BPB == 18 ? 4 : 8;
  if ((smem_u32(p) & 3) == 0) {
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p);
    uint32_t words[nfull + 1];
#pragma unroll
    for (int i = 0; i < nfull; ++i) words[i] = p4[i];
    words[nfull] = *reinterpret_cast<const uint16_t*>(p + 4 * nfull);
    scale_bits = words[0] & 0xffffu;
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = __funnelshift_r(words[i], words[i + 1], 16);
  } else {
    scale_bits = *reinterpret_cast<const uint16_t*>(p);
    const uint32_t* p4 = reinterpret_cast<const uint32_t*>(p + 2);
#pragma unroll
    for (int i = 0; i < nfull; ++i) q[i] = p4[i];
  }
}

template <int BPB, int NT>
__global__ void __launch_bounds__(kWarps * 32)
qgemm_tc_kernel(const uint8_t* __restrict__ w, int rows, int nb, Batch b, Epilogue ep,
                unsigned int* status) {
  using L = TcLayout<BPB, NT>;
  constexpr int kHalf = NT / kColGroups;  // columns drained per warp
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + L::kMiscOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff + 16);
  float* dWs = reinterpret_cast<float*>(smem + L::kDwOff);  // [2][kKC][2][128]

  constexpr uint32_t kIdesc = (2u << 4) | ((BPB == 18 ? 0u : 1u) << 7) | (1u << 10) |
                              ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int quarter = warp & 3, colhalf = warp >> 2;
  const int erow = blockIdx.y * kM + quarter * 32 + (tid & 31);  // epilogue row of this thread
  const int urow = tid & (kM - 1);                               // unpack row of this thread
  const int ublk = tid >> 7;                                     // its block within the chunk
  const int seq0 = blockIdx.x * NT;
  const int nseq = min(NT, b.rows - seq0);
  const size_t row_bytes = (size_t)nb * BPB;
  const int nchunks = nb / kKC;
  const uint8_t* wrow = w + (size_t)(blockIdx.y * kM + urow) * row_bytes;

  if (warp == 0) tmem_alloc(tmem_slot, L::kCols);
  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_barrier_init();
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  // Chunk c = blocks 4c..4c+3 into ring stage c % kRS; always one commit group.
  auto issue_chunk = [&](int c) {
    if (c < nchunks) {
      uint8_t* st = smem + (c % kRS) * L::kStage;
      const int blk0 = c * kKC;
      if (tid < kM) {
        const uint8_t* src = wrow + (size_t)blk0 * BPB;
        uint8_t* dst = st + tid * L::kRowRaw;
#pragma unroll
        for (int g = 0; g < kKC * BPB / 8; ++g) cp_async8(dst + 8 * g, src + 8 * g);
      } else if (tid - kM < NT) {
        const int s = tid - kM;
        const bool valid = s < nseq;
        const size_t srow = valid ? (size_t)(seq0 + s) : 0;
        const int8_t* a = b.aq + srow * kActStride + (size_t)blk0 * 32;
#pragma unroll
        for (int j = 0; j < kKC; ++j) {
          cp_async16(st + L::kARaw + j * L::kBTile + tile_off(s, 0), a + j * 32, valid);
          cp_async16(st + L::kARaw + j * L::kBTile + tile_off(s, 1), a + j * 32 + 16, valid);
        }
        cp_async16(st + L::kDaOff + s * kKC * 4, b.ad + srow * kActBlocks + blk0, valid);
        cp_async16(st + L::kCOff + s * kKC * 4, b.asum + srow * kActBlocks + blk0, valid);
      }
    }
    cp_async_commit();
  };

  float acc[kHalf];
#pragma unroll
  for (int s = 0; s < kHalf; ++s) acc[s] = 0.0f;
  uint32_t phase[2] = {0, 0};
  int pending[2] = {0, 0};  // thread 0: committed MMA groups not yet waited for

  // Drains chunk c's kKC blocks, in block order, into the accumulators.
  auto epilogue = [&](int c) {
    const uint8_t* st = smem + (c % kRS) * L::kStage;
    const float4* dA4 = reinterpret_cast<const float4*>(st + L::kDaOff);
    const int4* C4 = reinterpret_cast<const int4*>(st + L::kCOff);
    const float* dw = dWs + (c & 1) * (kKC * 2 * kM);
    const int lrow = quarter * 32 + (tid & 31);
    uint32_t v[kKC][kHalf];
#pragma unroll
    for (int j = 0; j < kKC; ++j)
      tmem_ld<kHalf>(tmem_base + ((uint32_t)(quarter * 32) << 16) +
                         (uint32_t)(((c & 1) * kKC + j) * NT + colhalf * kHalf),
                     v[j]);
    tmem_wait_ld();
    float dW[kKC], negMdW[kKC];
#pragma unroll
    for (int j = 0; j < kKC; ++j) {
      dW[j] = dw[(j * 2) * kM + lrow];
      negMdW[j] = dw[(j * 2 + 1) * kM + lrow];
    }
#pragma unroll
    for (int jj = 0; jj < kHalf; ++jj) {
      const int s = colhalf * kHalf + jj;
      const float4 da4 = dA4[s];  // the column's scales for the chunk's 4 blocks
      const float da[4] = {da4.x, da4.y, da4.z, da4.w};
      int cc[4] = {0, 0, 0, 0};
      if (BPB == 18) {
        const int4 c4 = C4[s];
        cc[0] = c4.x; cc[1] = c4.y; cc[2] = c4.z; cc[3] = c4.w;
      }
#pragma unroll
      for (int j = 0; j < kKC; ++j) {
        float t;
        if (BPB == 18) {
          const float x = __int_as_float((int)v[j][jj] + cc[j]);
          t = __fmul_rn(__fmaf_rn(x, dW[j], negMdW[j]), da[j]);
        } else {
          const float f = __fsub_rn(__int_as_float((int)v[j][jj] + 0x4B400000), 12582912.0f);
          t = __fmul_rn(f, __fmul_rn(dW[j], da[j]));
        }
        acc[jj] = __fadd_rn(acc[jj], t);  // blocks in order per column
      }
    }
  };

  for (int c = 0; c < kRS; ++c) issue_chunk(c);
  int timed_out = 0;
  int c = 0;
  for (; c < nchunks; ++c) {
    uint8_t* st = smem + (c % kRS) * L::kStage;
    // Chunk c has landed: groups issued so far end at chunk max(kRS-1, c+1).
    cp_async_wait<kRS - 3>();
    __syncthreads();
    if (BPB == 18 && tid >= kM && tid - kM < NT) {
      int* C = reinterpret_cast<int*>(st + L::kCOff) + (tid - kM) * kKC;
#pragma unroll
      for (int k = 0; k < kKC; ++k) C[k] = 0x4B400000 - 8 * C[k];
    }
    // unpack one block of one row into the canonical A tiles of group c & 1
    {
      const int j = ublk;
      uint32_t sb, q[8];
      read_block<BPB>(st + urow * L::kRowRaw + j * BPB, sb, q);
      const float dW = half_to_f32((uint16_t)sb);
      float* dw = dWs + (c & 1) * (kKC * 2 * kM);
      dw[(j * 2) * kM + urow] = dW;
      dw[(j * 2 + 1) * kM + urow] = -__fmul_rn(12582912.0f, dW);
      uint8_t* A = smem + L::kAcanOff + ((c & 1) * kKC + j) * (kM * 32);
      if (BPB == 18) {
        *reinterpret_cast<uint4*>(A + tile_off(urow, 0)) =
            make_uint4(q[0] & 0x0f0f0f0fu, q[1] & 0x0f0f0f0fu, q[2] & 0x0f0f0f0fu, q[3] & 0x0f0f0f0fu);
        *reinterpret_cast<uint4*>(A + tile_off(urow, 1)) =
            make_uint4((q[0] >> 4) & 0x0f0f0f0fu, (q[1] >> 4) & 0x0f0f0f0fu,
                       (q[2] >> 4) & 0x0f0f0f0fu, (q[3] >> 4) & 0x0f0f0f0fu);
      } else {
        *reinterpret_cast<uint4*>(A + tile_off(urow, 0)) = make_uint4(q[0], q[1], q[2], q[3]);
        *reinterpret_cast<uint4*>(A + tile_off(urow, 1)) = make_uint4(q[4], q[5], q[6], q[7]);
      }
    }
    fence_async_shared();
    tc_before_sync();
    const int stop = __syncthreads_or(timed_out);
    tc_after_sync();
    if (stop) break;
    // Chunk c-2 was drained in iteration c-1 by every thread: refill its stage.
    if (c >= 2) issue_chunk(c - 2 + kRS);
    if (tid == 0) {
#pragma unroll
      for (int j = 0; j < kKC; ++j) {
        const uint8_t* A = smem + L::kAcanOff + ((c & 1) * kKC + j) * (kM * 32);
        const uint8_t* B = st + L::kARaw + j * L::kBTile;
        mma_i8(tmem_base + (uint32_t)(((c & 1) * kKC + j) * NT), smem_desc(A), smem_desc(B), kIdesc);
      }
      mma_commit(&mbar[c & 1]);
      pending[c & 1] = 1;
    }
    if (c >= 1) {
      const int pc = c - 1;
      if (!mbar_wait_bounded(&mbar[pc & 1], phase[pc & 1])) {
        timed_out = 1;
      } else {
        phase[pc & 1] ^= 1u;
        if (tid == 0) pending[pc & 1] = 0;
        epilogue(pc);
      }
    }
  }
  if (!timed_out && c == nchunks) {
    const int pc = nchunks - 1;
    if (!mbar_wait_bounded(&mbar[pc & 1], phase[pc & 1])) {
      timed_out = 1;
    } else {
      phase[pc & 1] ^= 1u;
      if (tid == 0) pending[pc & 1] = 0;
      epilogue(pc);
    }
  }
  cp_async_wait_all();
  tc_before_sync();
  const int aborted = __syncthreads_or(timed_out);
  tc_after_sync();
  if (aborted && tid == 0) {
    atomicOr(status, 1u);
    for (int k = 0; k < 2; ++k)
      if (pending[k]) mbar_wait_bounded(&mbar[k], phase[k]);
  }
  tc_before_sync();
  __syncthreads();
  tc_after_sync();
  if (warp == 0) tmem_dealloc(tmem_base, L::kCols);
  if (aborted) return;

#pragma unroll
  for (int jj = 0; jj < kHalf; ++jj) {
    const int s = colhalf * kHalf + jj;
    if (s < nseq) {
      const int seq = seq0 + s;
      float* dst = ep.out + (size_t)seq * ep.ld + erow;
      float v;
      if (ep.mode == EPI_BIAS) v = __fadd_rn(acc[jj], ep.bias[erow]);
      else if (ep.mode == EPI_RESIDUAL) v = __fadd_rn(*dst, acc[jj]);
      else v = acc[jj];
      *dst = v;
      check_finite(v, &ep.err[seq], ep.layer_ordinal, ep.domain, 0, erow);
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
  qgemm_tc_kernel<BPB, NT><<<grid, kWarps * 32, TcLayout<BPB, NT>::kBytes, s>>>(w, rows, nb, b, ep,
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
  const int nt = ctas(32) >= 148 ? 32 : 16;
  if (wtype == W_Q4_0) {
    if (nt == 32) launch_tc<18, 32>(w, rows, nb, b, ep, status, s);
    else launch_tc<18, 16>(w, rows, nb, b, ep, status, s);
  } else {
    if (nt == 32) launch_tc<34, 32>(w, rows, nb, b, ep, status, s);
    else launch_tc<34, 16>(w, rows, nb, b, ep, status, s);
  }
}

}  // namespace pb
