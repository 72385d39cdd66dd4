// Fused sampler for sm_100a: one CTA per logits row.
//
// Reference semantics (sulewicz/promptboot):
//   inference.rs:919-965       sample_token_with_repetition (validate, penalty, one draw)
//   fp32_sse2.rs:1848-1876     repetition penalty once per distinct history token
//   fp32_sse2.rs:1786-1846     top-20 (strict >, earlier id first), expf((v-v0)/0.7),
//                              f64 totals, top-p 0.8 cutoff, 24-bit draw
//   inference.rs:801-809       xorshift64 draw generator
//
// The row is streamed from HBM once.  A shared-memory bitmap of the history
// marks the logits the penalty changes; the penalised value feeds a warp-level
// top-k kept in registers, ordered by a 64-bit key (order-preserving value with
// -0 folded onto +0, then inverted id) so ties keep the lowest id exactly as
// the reference's insertion scan does.  Sixteen per-warp lists are merged by
// one warp; the twenty-term f64 sums then run sequentially in one thread.
#include "pb_common.cuh"
#include "pb_kernels.cuh"

namespace pb {

constexpr int kSampThreads = 512;
constexpr int kSampWarps = kSampThreads / 32;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t order_key(float v) {
  uint32_t u = bitsf(v);
  if (u == 0x80000000u) u = 0;  // ucomiss: -0 == +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Inverse of order_key on the key's high word.
__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t k = (uint32_t)(key >> 32);
  return fbits((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ float penalize(float v) {
  uint32_t s = bitsf(v);
  return ((s & 0x80000000u) && (s & 0x7fffffffu)) ? __fmul_rn(v, fbits(0x3f8ccccdu))
                                                   : __fdiv_rn(v, fbits(0x3f8ccccdu));
}

// Lanes 0..K-1 hold the warp's current best keys in descending order (0 = empty,
// smaller than every real key); lanes >= K keep 0.
template <int K>
__device__ __forceinline__ void list_insert(unsigned long long& entry, unsigned long long cand,
                                            int lane) {
  int pos = __popc(__ballot_sync(kFull, entry > cand));
  unsigned long long up = __shfl_up_sync(kFull, entry, 1);
  if (lane < K) {
    if (lane == pos) entry = cand;
    else if (lane > pos) entry = up;
  }
}

template <int K>
__device__ __forceinline__ void list_offer(unsigned long long& entry, unsigned long long& thr,
                                           unsigned long long key, int lane) {
  unsigned m = __ballot_sync(kFull, key > thr);
  while (m) {
    int src = __ffs(m) - 1;
    unsigned long long cand = __shfl_sync(kFull, key, src);
    list_insert<K>(entry, cand, lane);
    thr = __shfl_sync(kFull, entry, K - 1);
    m &= ~(1u << src);
    m &= __ballot_sync(kFull, key > thr);
  }
}

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t id) {
  return ((unsigned long long)order_key(v) << 32) | (unsigned long long)(~id);
}

// The K largest of n keys (nonzero keys distinct: every id is in one list
// only; 0 marks an empty entry) into out_keys in descending order, by rank:
// each nonzero key counts the keys above it, the whole CTA at once.  Ends with
// a CTA barrier.
template <int K>
__device__ void merge_ranked(const unsigned long long* keys, int n, unsigned long long* out_keys) {
  if (threadIdx.x < K) out_keys[threadIdx.x] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long k = keys[i];
    if (k == 0) continue;
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += keys[j] > k ? 1 : 0;
    if (rank < K) out_keys[rank] = k;
  }
  __syncthreads();
}

// Streams [0, words) of one row (or of a slice of it whose first id is
// id_base), folding every element into the CTA's top-K.  penal (may be null)
// marks the slice's ids whose value is penalised before ranking.
// Leaves the final list sorted in `out_keys[0..K)` (shared) and the first
// non-finite index/bits in *bad (shared, ~0 when none).
template <int K, int NW = kSampWarps>
__device__ void row_topk(const float* __restrict__ x, int words, const uint32_t* penal,
                         unsigned long long* warp_keys, unsigned long long* out_keys,
                         unsigned long long* bad, int id_base = 0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = ((words + NW * 128 - 1) / (NW * 128)) * 128;
  const int start = warp * seg;
  const int end = min(words, start + seg);
  unsigned long long entry = 0, thr = 0;
  // Float image of the list's K-th key: a penalty only lowers a value (x/1.1
  // for x >= 0, 1.1x for x < 0, zeros unchanged), so a raw value below it can
  // never enter the list and skips the key work; equal values go on to the
  // exact (value, id) key comparison.  One compare per value and one warp vote
  // per four values; non-finite values are not ranked here but leave
  // fma(v, 0, fin) NaN, and the row is then rescanned for its first one.
  float thr_f = fbits(0xff800000u);
  float fin = 0.0f;
  auto offer = [&](float val, int i) {
    unsigned long long key = 0;
    if (i < end && val >= thr_f) {
      if (penal && (penal[i >> 5] >> (i & 31) & 1u)) val = penalize(val);
      key = make_key(val, (uint32_t)(id_base + i));
    }
    list_offer<K>(entry, thr, key, lane);
    thr_f = thr == 0 ? fbits(0xff800000u) : key_value(thr);
  };
  auto offer4 = [&](float v0, float v1, float v2, float v3, int i0) {
    fin = __fmaf_rn(v0, 0.0f, fin);
    fin = __fmaf_rn(v1, 0.0f, fin);
    fin = __fmaf_rn(v2, 0.0f, fin);
    fin = __fmaf_rn(v3, 0.0f, fin);
    const bool any = v0 >= thr_f || v1 >= thr_f || v2 >= thr_f || v3 >= thr_f;
    if (__ballot_sync(kFull, any) == 0) return;
    offer(v0, i0);
    offer(v1, i0 + 1);
    offer(v2, i0 + 2);
    offer(v3, i0 + 3);
  };
  // Software pipeline: the next four 512-byte loads of the warp are in flight
  // while the current four are ranked.
  constexpr int kBatch = 4;
  int base = start;
  if (base + kBatch * 128 <= end) {
    float4 cur[kBatch], nxt[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      cur[u] = *reinterpret_cast<const float4*>(x + base + u * 128 + lane * 4);
    for (;;) {
      const int next = base + kBatch * 128;
      const bool more = next + kBatch * 128 <= end;
      if (more) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          nxt[u] = *reinterpret_cast<const float4*>(x + next + u * 128 + lane * 4);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        offer4(cur[u].x, cur[u].y, cur[u].z, cur[u].w, base + u * 128 + lane * 4);
      base = next;
      if (!more) break;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) cur[u] = nxt[u];
    }
  }
  for (; base < end; base += 128) {
    const int i0 = base + lane * 4;
    float v[4];
    if (i0 + 3 < end) {
      float4 f = *reinterpret_cast<const float4*>(x + i0);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (i0 + j < end) ? x[i0 + j] : 0.0f;
    }
    offer4(v[0], v[1], v[2], v[3], i0);
  }
  if (lane < K) warp_keys[warp * K + lane] = entry;
  if (__syncthreads_or(fin != 0.0f)) {
    // some value is not finite: the first one, in index order
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const uint32_t vb = bitsf(x[i]);
      if (!finite_bits(vb)) atomicMin(bad, ((unsigned long long)(id_base + i) << 32) | vb);
    }
    __syncthreads();
  }
  if (warp == 0) {
    // the warps' sorted lists folded by insertion (after the first list few
    // keys pass the threshold)
    entry = 0;
    thr = 0;
    for (int base = 0; base < NW * K; base += 32) {
      unsigned long long key = (base + lane < NW * K) ? warp_keys[base + lane] : 0ull;
      list_offer<K>(entry, thr, key, lane);
    }
    if (lane < K) out_keys[lane] = entry;
  }
  __syncthreads();
}

// The draw and top-k/top-p of one row (fp32_sse2.rs:1818-1845, inference.rs:
// 801-809) from its final sorted top-20 keys, or its rejection: the first
// non-finite logit (status 7) before the first history id out of range (3).
__device__ void sample_tail(const unsigned long long* top, unsigned long long bad,
                            unsigned long long bad_token, unsigned long long* states,
                            SamplerRow* out, int row) {
  SamplerRow r;
  r.selected = 0;
  if (bad != kNoError) {
    r.status = 7;
    r.index = (uint32_t)(bad >> 32);
    r.value = (uint32_t)bad;
    out[row] = r;
    return;
  }
  if (bad_token != kNoError) {
    r.status = 3;
    r.index = (uint32_t)(bad_token >> 32);
    r.value = (uint32_t)bad_token;
    out[row] = r;
    return;
  }
  // inference.rs:801-809
  unsigned long long state = states[2 * row];
  state ^= state >> 12;
  state ^= state << 25;
  state ^= state >> 27;
  states[2 * row] = state;
  states[2 * row + 1] += 1;
  const uint32_t random24 = (uint32_t)((state * 0x2545f4914f6cdd1dull) >> 40);

  // fp32_sse2.rs:1818-1845
  // The ranked (penalised) values come back from the keys (order_key is
  // invertible up to -0 -> +0, which no result below can distinguish).
  uint32_t ids[20];
  float weights[20];
  const float maximum = key_value(top[0]);
  double total = 0.0;
  for (int at = 0; at < 20; ++at) {
    ids[at] = ~(uint32_t)top[at];
    float v = key_value(top[at]);
    weights[at] = expf_ref(__fdiv_rn(__fsub_rn(v, maximum), fbits(0x3f333333u)));
    total += (double)weights[at];
  }
  const float cutoff = __fmul_rn((float)total, fbits(0x3f4ccccdu));
  int kept = 20;
  double kept_total = 0.0;
  for (int at = 0; at < 20; ++at) {
    kept_total += (double)weights[at];
    if (!(cutoff > (float)kept_total)) { kept = at + 1; break; }
  }
  const float unit = __fdiv_rn((float)(random24 & 0x00ffffffu), fbits(0x4b800000u));
  const float target = __fmul_rn((float)kept_total, unit);
  uint32_t selected = ids[kept - 1];
  double cumulative = 0.0;
  for (int at = 0; at < kept; ++at) {
    cumulative += (double)weights[at];
    if ((float)cumulative > target) { selected = ids[at]; break; }
  }
  r.status = 0;
  r.index = 0;
  r.value = random24;
  r.selected = selected;
  out[row] = r;
}

__global__ void __launch_bounds__(kSampThreads)
sampler_kernel(float* logits, size_t ld, int words, const uint32_t* __restrict__ history,
               const uint64_t* __restrict__ hist_offset, const uint32_t* __restrict__ hist_len,
               const uint8_t* __restrict__ initial_seen, unsigned long long* states,
               SamplerRow* out) {
  pdl_begin();
  __shared__ uint32_t penal[(kVocab + 31) / 32];
  __shared__ unsigned long long warp_keys[kSampWarps * 20];
  __shared__ unsigned long long top[20];
  __shared__ unsigned long long bad;
  __shared__ unsigned long long bad_token;
  const int row = blockIdx.x;
  float* x = logits + (size_t)row * ld;
  const uint32_t* hist = history + hist_offset[row];
  const uint32_t n = hist_len[row];
  const int map_words = (words + 31) / 32;

  for (int i = threadIdx.x; i < map_words; i += blockDim.x) penal[i] = 0;
  if (threadIdx.x == 0) { bad = kNoError; bad_token = kNoError; }
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    uint32_t t = hist[j];
    if (t < (uint32_t)words) atomicOr(&penal[t >> 5], 1u << (t & 31));
    else atomicMin(&bad_token, ((unsigned long long)j << 32) | t);
  }
  __syncthreads();
  if (initial_seen) {
    // Tokens already marked in the caller's bitmap are skipped by the reference.
    for (int i = threadIdx.x; i < map_words; i += blockDim.x) {
      uint32_t m = 0;
      for (int byte = 0; byte < 4; ++byte) {
        int at = i * 4 + byte;
        if (at < (words + 7) / 8) m |= (uint32_t)initial_seen[at] << (8 * byte);
      }
      penal[i] &= ~m;
    }
    __syncthreads();
  }

  row_topk<20>(x, words, penal, warp_keys, top, &bad);

  const bool ok = bad == kNoError && bad_token == kNoError;
  if (ok) {
    // Write the penalised logits back in place, once per distinct token.
    for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
      uint32_t t = hist[j];
      uint32_t bit = 1u << (t & 31);
      uint32_t old = atomicAnd(&penal[t >> 5], ~bit);
      if (old & bit) x[t] = penalize(x[t]);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) sample_tail(top, bad, bad_token, states, out, row);
}

void launch_sampler(float* logits, size_t ld, int rows, int words, const uint32_t* history,
                    const uint64_t* hist_offset, const uint32_t* hist_len,
                    const uint8_t* initial_seen, unsigned long long* states, SamplerRow* out,
                    cudaStream_t s) {
  launch_pdl(sampler_kernel, rows, kSampThreads, 0, s, logits, ld, words, history, hist_offset,
                                               hist_len, initial_seen, states, out);
}

// ------------------------------------------------------ split rows
//
// Few rows leave most SMs idle with one CTA per row, so a row's vocabulary
// is split over kSplitParts CTAs: each ranks its slice (penalised by the
// history tokens that fall in it) into a top-20 of global ids; a merge CTA per
// row then folds the parts' lists (the same keys, so the same order and ties
// as one scan), writes the penalised logits back once per distinct history
// token and draws, exactly as sampler_kernel does.
constexpr int kSplitSlice = ((kVocab + kSplitParts - 1) / kSplitParts + 127) / 128 * 128;

constexpr int kPartWarps = 4;

__global__ void __launch_bounds__(kPartWarps * 32)
sampler_part_kernel(const float* logits, size_t ld, int words, const uint32_t* __restrict__ history,
                    const uint64_t* __restrict__ hist_offset, const uint32_t* __restrict__ hist_len,
                    const uint8_t* __restrict__ initial_seen, unsigned long long* cand) {
  pdl_begin();
  __shared__ uint32_t penal[kSplitSlice / 32];
  __shared__ unsigned long long warp_keys[kPartWarps * 20];
  __shared__ unsigned long long top[20];
  __shared__ unsigned long long bad;
  const int row = blockIdx.x, part = blockIdx.y;
  const int lo = part * kSplitSlice, hi = min(words, lo + kSplitSlice);
  unsigned long long* mine = cand + ((size_t)row * kSplitParts + part) * 21;
  if (lo >= hi) {  // an empty tail part
    if (threadIdx.x < 20) mine[threadIdx.x] = 0;
    if (threadIdx.x == 0) mine[20] = kNoError;
    return;
  }
  const float* x = logits + (size_t)row * ld;
  const uint32_t* hist = history + hist_offset[row];
  const uint32_t n = hist_len[row];
  const int map_words = (hi - lo + 31) / 32;
  for (int i = threadIdx.x; i < map_words; i += blockDim.x) penal[i] = 0;
  if (threadIdx.x == 0) bad = kNoError;
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    const uint32_t t = hist[j];
    if (t >= (uint32_t)lo && t < (uint32_t)hi) atomicOr(&penal[(t - lo) >> 5], 1u << ((t - lo) & 31));
  }
  __syncthreads();
  if (initial_seen) {
    // tokens already marked in the caller's bitmap are skipped (lo is a
    // multiple of 32, so slice word i is seen bytes 4 (lo / 32 + i) ..)
    for (int i = threadIdx.x; i < map_words; i += blockDim.x) {
      uint32_t m = 0;
      for (int byte = 0; byte < 4; ++byte) {
        const int at = (lo >> 3) + i * 4 + byte;
        if (at < (words + 7) / 8) m |= (uint32_t)initial_seen[at] << (8 * byte);
      }
      penal[i] &= ~m;
    }
    __syncthreads();
  }
  row_topk<20, kPartWarps>(x + lo, hi - lo, penal, warp_keys, top, &bad, lo);
  if (threadIdx.x < 20) mine[threadIdx.x] = top[threadIdx.x];
  if (threadIdx.x == 0) mine[20] = bad;
}

__global__ void __launch_bounds__(kSampThreads)
sampler_merge_kernel(float* logits, size_t ld, int words, const uint32_t* __restrict__ history,
                     const uint64_t* __restrict__ hist_offset, const uint32_t* __restrict__ hist_len,
                     const uint8_t* __restrict__ initial_seen, const unsigned long long* cand,
                     unsigned long long* states, SamplerRow* out) {
  pdl_begin();
  __shared__ uint32_t penal[(kVocab + 31) / 32];
  __shared__ unsigned long long part_keys[kSplitParts * 20];
  __shared__ unsigned long long top[20];
  __shared__ unsigned long long bad;
  __shared__ unsigned long long bad_token;
  const int row = blockIdx.x;
  float* x = logits + (size_t)row * ld;
  const uint32_t* hist = history + hist_offset[row];
  const uint32_t n = hist_len[row];
  const int map_words = (words + 31) / 32;
  const unsigned long long* rc = cand + (size_t)row * kSplitParts * 21;
  for (int i = threadIdx.x; i < map_words; i += blockDim.x) penal[i] = 0;
  if (threadIdx.x == 0) {
    unsigned long long b0 = kNoError;
    for (int part = 0; part < kSplitParts; ++part) b0 = min(b0, rc[part * 21 + 20]);
    bad = b0;
    bad_token = kNoError;
  }
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
    const uint32_t t = hist[j];
    if (t < (uint32_t)words) atomicOr(&penal[t >> 5], 1u << (t & 31));
    else atomicMin(&bad_token, ((unsigned long long)j << 32) | t);
  }
  for (int i = threadIdx.x; i < kSplitParts * 20; i += blockDim.x)
    part_keys[i] = rc[(i / 20) * 21 + i % 20];
  __syncthreads();
  merge_ranked<20>(part_keys, kSplitParts * 20, top);
  if (initial_seen) {
    for (int i = threadIdx.x; i < map_words; i += blockDim.x) {
      uint32_t m = 0;
      for (int byte = 0; byte < 4; ++byte) {
        const int at = i * 4 + byte;
        if (at < (words + 7) / 8) m |= (uint32_t)initial_seen[at] << (8 * byte);
      }
      penal[i] &= ~m;
    }
    __syncthreads();
  }
  if (bad == kNoError && bad_token == kNoError) {
    // the penalised logits back in place, once per distinct token
    for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
      const uint32_t t = hist[j];
      const uint32_t bit = 1u << (t & 31);
      const uint32_t old = atomicAnd(&penal[t >> 5], ~bit);
      if (old & bit) x[t] = penalize(x[t]);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) sample_tail(top, bad, bad_token, states, out, row);
}

void launch_sampler_split(float* logits, size_t ld, int rows, int words, const uint32_t* history,
                          const uint64_t* hist_offset, const uint32_t* hist_len,
                          const uint8_t* initial_seen, unsigned long long* states, SamplerRow* out,
                          unsigned long long* cand, cudaStream_t s) {
  launch_pdl(sampler_part_kernel, dim3(rows, kSplitParts), kPartWarps * 32, 0, s, logits, ld, words,
             history, hist_offset, hist_len, initial_seen, cand);
  launch_pdl(sampler_merge_kernel, rows, kSampThreads, 0, s, logits, ld, words, history, hist_offset,
             hist_len, initial_seen, cand, states, out);
}

// inference.rs:814-859 top_logits_8: descending, equal values (and signed zeros)
// in ascending token order; also the first non-finite word.
__global__ void __launch_bounds__(kSampThreads)
topk8_kernel(const float* logits, size_t ld, int words, uint32_t* out_pairs,
             unsigned long long* first_nonfinite) {
  __shared__ unsigned long long warp_keys[kSampWarps * 8];
  __shared__ unsigned long long top[8];
  __shared__ unsigned long long bad;
  const int row = blockIdx.x;
  const float* x = logits + (size_t)row * ld;
  if (threadIdx.x == 0) bad = kNoError;
  __syncthreads();
  row_topk<8>(x, words, nullptr, warp_keys, top, &bad);
  if (threadIdx.x < 8) {
    uint32_t id = ~(uint32_t)top[threadIdx.x];
    out_pairs[(size_t)row * 16 + 2 * threadIdx.x] = id;
    out_pairs[(size_t)row * 16 + 2 * threadIdx.x + 1] = bitsf(x[id]);
  }
  if (threadIdx.x == 0 && first_nonfinite) first_nonfinite[row] = bad;
}

void launch_topk8(const float* logits, size_t ld, int rows, int words, uint32_t* out_pairs,
                  unsigned long long* first_nonfinite, cudaStream_t s) {
  topk8_kernel<<<rows, kSampThreads, 0, s>>>(logits, ld, words, out_pairs, first_nonfinite);
}

}  // namespace pb
