// GQA decode attention over an HBM-resident bf16 KV cache (sm_100a).
//
// Computes, for every sequence b and query head h = kvh * G + g,
//   o[b,h,:] = softmax(q[b,h,:] . K[b,kvh,:len,:]^T * scale) . V[b,kvh,:len,:]
// with exact bf16 x bf16 products, fp32 accumulation, an fp32 online softmax
// (running max m, running sum l, accumulator rescale) and a bf16
// round-to-nearest-even store.  This is the arithmetic of the reference's
// datapath (hw/rtl/attn_top.sv:301-625: QK^T over depth, scale by 1/sqrt(D),
// online softmax per block, P.V, O = O*corr + dO, normalise by l) with true
// fp32 exp instead of the 1024-entry LUT, and P kept in fp32.
//
// Design (one CTA per (split, kv head, sequence)):
//  * the split's K and V rows are streamed with bulk TMA copies
//    (cp.async.bulk, no multicast, L2 evict-first) into a kStages-deep
//    shared-memory ring; an mbarrier per stage counts the transaction bytes.
//    There is no producer warp: the consumer warp whose arrival completes a
//    stage's release (a shared-memory counter) issues that stage's refill, so
//    no thread waits on the release side.  Every mbarrier wait is bounded by
//    %globaltimer.
//  * 8 warps split each tile by tokens.  A lane owns VEC contiguous head
//    dims (a 16-byte vector, 8-byte for G = 8) of one token row, so a warp
//    covers 32*VEC/D token rows per pass with conflict-free shared loads.
//    The G query heads of the group are packed into the same pass, so every
//    K/V byte read from HBM is used by all G heads.
//  * QK partial sums (ITER tokens x G heads per lane) are finished with a
//    reduce-scatter over the D/8 lanes of a row: after log2(D/8) exchange
//    steps each lane holds one complete score, instead of every lane
//    butterfly-reducing every score.
//  * each warp runs its own online softmax over its token slice (no CTA-wide
//    barrier per tile); warps and splits are merged at the end with the
//    log-sum-exp rule in log2 domain.  The last CTA of a (sequence, kv head)
//    to finish (an atomic arrival counter, no waiting) merges the split
//    partials and writes the bf16 output.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "decode_merge.cuh"
#include "lara_internal.h"

namespace lara {

namespace {

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }
constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int kPageCacheEntries = 256;  // block-table entries of a CTA's chunk kept in shared memory

template <int D, int G>
struct Traits {
  static constexpr int kVec = (G >= 8) ? 4 : 8;             // bf16 per lane per row
  static constexpr int kLPT = D / kVec;                      // lanes per token row
  static constexpr int kTPI = 32 / kLPT;                     // token rows per warp pass
  static constexpr int kIter = cmax(1, cmin(4, kLPT / G));   // passes per tile per warp
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kTokPerWarp = kIter * kTPI;
  static constexpr int kTile = kWarps * kTokPerWarp;         // tokens per stage
  static constexpr int kRowBytes = D * 2;
  static constexpr int kHalfStage = kTile * kRowBytes;       // K (or V) bytes per stage
  static constexpr int kStageBytes = 2 * kHalfStage;
  static constexpr int kStages = cmax(2, cmin(8, 98304 / kStageBytes));
  static constexpr int kNV = kIter * G;                      // partial sums per lane
  static constexpr int kLogLPT = ilog2(kLPT);
  static constexpr int kH = cmin(kLogLPT, ilog2(kNV));       // reduce-scatter steps
  static constexpr int kR = kLogLPT - kH;                    // duplicate-lane butterfly steps
  static constexpr int kLogG = ilog2(G);
  static constexpr int kLogIter = ilog2(kIter);
  static constexpr int kHP = cmin(kH, kLogIter);             // steps split on a pass bit (the rest on a head bit)
  static constexpr int kMinBlocks = 2;
  // shared memory layout
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kMergeBytes = kWarps * G * (D + 2) * 4;
  static constexpr int kBigBytes = cmax(kRingBytes, kMergeBytes);
  static constexpr int kPbufFloats = 2 * kWarps * kTokPerWarp * G;
  static constexpr int kCbufFloats = 2 * kWarps * G;
  static constexpr int kPbufOff = kBigBytes;
  static constexpr int kCbufOff = kPbufOff + kPbufFloats * 4;
  static constexpr int kBarOff = (kCbufOff + kCbufFloats * 4 + 15) / 16 * 16;  // full[], empty[]
  static constexpr int kCntOff = kBarOff + 2 * kStages * 8;                      // refill round per stage
  static constexpr int kFlagOff = kCntOff + kStages * 4;
  static constexpr int kPageCache = kPageCacheEntries;
  static constexpr int kPageOff = (kFlagOff + 16 + 15) / 16 * 16;                // page offsets (int64)
  static constexpr int kSmemBytes = kPageOff + kPageCache * 8;
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  static_assert(kLPT <= 32 && 32 % kLPT == 0, "a token row must fit one warp");
  static_assert(G >= 1 && G <= kLPT && (G & (G - 1)) == 0, "group size must be a power of two <= lanes per row");
  static_assert((kNV >> kH) == 1, "one finished score per lane");
};

__device__ __forceinline__ int seq_len_of(const DecodeParams& p, int seq, int row_in_seq) {
  long long len = (long long)p.len_c0 + (long long)p.len_c1 * row_in_seq;
  if (p.lens) {
    const int l = p.lens[seq];
    if (l < 0 || l > p.max_seq_len) atomicOr(p.status, kDevBadLength);
    len += l;
  }
  return len < 0 ? 0 : (len > p.max_seq_len ? p.max_seq_len : (int)len);
}

// Paged caches: element offset of the (page, kv head) block that holds token
// `tok` of `seq` in the pool [pages][Hkv][page][D].  An out-of-range
// block-table entry flags the status word and reads page 0 instead, so every
// issued copy stays in bounds and completes.
__device__ __forceinline__ long long page_block(const int32_t* block_table, int pages_per_seq, int page_log2,
                                                int num_pages, int n_kv_heads, int* status, int seq, int kvh,
                                                int tok, int d) {
  int page = __ldg(block_table + (long long)seq * pages_per_seq + (tok >> page_log2));
  if (page < 0 || page >= num_pages) {
    atomicOr(status, kDevBadPage);
    page = 0;
  }
  return (((long long)page * n_kv_heads + kvh) << page_log2) * d;
}

// The same, for a page past the CTA's shared-memory cache (chunks of more than
// kPageCacheEntries pages), kept out of line so the refill path stays short.
__device__ __noinline__ long long page_block_uncached(const int32_t* block_table, int pages_per_seq, int page_log2,
                                                      int num_pages, int n_kv_heads, int* status, int seq, int kvh,
                                                      int tok, int d) {
  return page_block(block_table, pages_per_seq, page_log2, num_pages, n_kv_heads, status, seq, kvh, tok, d);
}

// Offset of the block holding `tok`: from the CTA's validated cache of the
// chunk's pages, or from the block table past it.
template <int D>
__device__ __forceinline__ long long page_base(const DecodeParams& p, const long long* pbase, int seq, int kvh,
                                               int tok, int tok_begin) {
  const int idx = (tok >> p.page_log2) - (tok_begin >> p.page_log2);
  if (idx < kPageCacheEntries) return pbase[idx];
  return page_block_uncached(p.block_table, p.pages_per_seq, p.page_log2, p.num_pages, p.n_kv_heads, p.status, seq,
                             kvh, tok, D);
}

// Issue the bulk copies of tile `t` (K rows then V rows) into stage `st`.
template <int D, int G, bool kPaged>
__device__ __forceinline__ void issue_tile(uint8_t* smem, uint64_t* full, int t, int ntok, const DecodeParams& p,
                                           int seq, int kvh, int tok_begin, const long long* pbase, uint64_t pol,
                                           long long pre_base = -1) {
  using T = Traits<D, G>;
  const int st = t % T::kStages;
  const int n = min(T::kTile, ntok - t * T::kTile);
  const uint32_t bytes = (uint32_t)n * T::kRowBytes;
  uint8_t* stage = smem + st * T::kStageBytes;
  mbar_arrive_expect_tx(&full[st], 2u * bytes);
  const int tok0 = tok_begin + t * T::kTile;
  if constexpr (!kPaged) {
    const long long off = (long long)seq * p.kv_sb + (long long)kvh * p.kv_sh + (long long)tok0 * D;
    bulk_g2s(stage, p.k + off, bytes, &full[st], pol);
    bulk_g2s(stage + T::kHalfStage, p.v + off, bytes, &full[st], pol);
    return;
  }
  // A tile lies inside one page when pages are at least a tile long (tiles
  // start on tile boundaries): one copy each for K and V, as for a contiguous
  // cache.  Smaller pages take one copy per page piece.
  const int ps = 1 << p.page_log2;
  const int in_page0 = tok0 & (ps - 1);
  if (n <= ps - in_page0) {
    const long long base = pre_base >= 0 ? pre_base : page_base<D>(p, pbase, seq, kvh, tok0, tok_begin);
    const long long off = base + (long long)in_page0 * D;
    bulk_g2s(stage, p.k + off, bytes, &full[st], pol);
    bulk_g2s(stage + T::kHalfStage, p.v + off, bytes, &full[st], pol);
    return;
  }
  // Pages shorter than a tile divide it, so the tile starts on a page boundary:
  // piece i is the first cnt rows of cached page idx0 + i.
  const int idx0 = (tok0 >> p.page_log2) - (tok_begin >> p.page_log2);
  for (int i = 0, r = 0; r < n; ++i, r += ps) {
    const int cnt = min(n - r, ps);
    const int idx = idx0 + i;
    const long long off = idx < kPageCacheEntries
                              ? pbase[idx]
                              : page_block_uncached(p.block_table, p.pages_per_seq, p.page_log2, p.num_pages,
                                                    p.n_kv_heads, p.status, seq, kvh, tok0 + r, D);
    bulk_g2s(stage + r * T::kRowBytes, p.k + off, (uint32_t)cnt * T::kRowBytes, &full[st], pol);
    bulk_g2s(stage + T::kHalfStage + r * T::kRowBytes, p.v + off, (uint32_t)cnt * T::kRowBytes, &full[st], pol);
  }
}

// Paged caches, issued by a whole warp (every lane calls this): a tile inside
// one page takes lane 0's two copies; a tile split over pages shorter than a
// tile gives each (page piece, K or V) copy to its own lane, so the refill
// costs one copy's issue latency instead of 2 x pieces in a row.
template <int D, int G>
__device__ __forceinline__ void issue_tile_paged_warp(uint8_t* smem, uint64_t* full, int t, int ntok,
                                                      const DecodeParams& p, int seq, int kvh, int tok_begin,
                                                      const long long* pbase, uint64_t pol, int lane,
                                                      long long pre_base = -1) {
  using T = Traits<D, G>;
  const int n = min(T::kTile, ntok - t * T::kTile);
  const int ps = 1 << p.page_log2;
  const int tok0 = tok_begin + t * T::kTile;
  if (n <= ps - (tok0 & (ps - 1))) {
    if (lane == 0) issue_tile<D, G, true>(smem, full, t, ntok, p, seq, kvh, tok_begin, pbase, pol, pre_base);
    return;
  }
  const int st = t % T::kStages;
  uint8_t* stage = smem + st * T::kStageBytes;
  if (lane == 0) mbar_arrive_expect_tx(&full[st], 2u * (uint32_t)n * T::kRowBytes);
  __syncwarp();
  // the tile starts on a page boundary; piece i is the first cnt rows of cached page idx0 + i
  const int pieces = (n + ps - 1) >> p.page_log2;
  const int i = lane >> 1;
  if (i < pieces) {
    const int r = i << p.page_log2;
    const int cnt = min(n - r, ps);
    const int idx = (tok0 >> p.page_log2) - (tok_begin >> p.page_log2) + i;
    const long long off = idx < kPageCacheEntries
                              ? pbase[idx]
                              : page_block_uncached(p.block_table, p.pages_per_seq, p.page_log2, p.num_pages,
                                                    p.n_kv_heads, p.status, seq, kvh, tok0 + r, D);
    const int half = lane & 1;
    bulk_g2s(stage + half * T::kHalfStage + r * T::kRowBytes, (half ? p.v : p.k) + off,
             (uint32_t)cnt * T::kRowBytes, &full[st], pol);
  }
}

// VEC bf16 words from shared memory -> VEC/2 fp32 pairs (element 2i in .x,
// 2i+1 in .y), the low element by a byte permute and the high one by a mask,
// both on the integer ALU, so the FMA pipe keeps to the dot products.
template <int VEC>
__device__ __forceinline__ void load_bf16_pairs_alu(const uint16_t* p, float2 f[VEC / 2]) {
  uint32_t w[VEC / 2];
  if constexpr (VEC == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
  } else {
    static_assert(VEC == 4, "VEC must be 4 or 8");
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x; w[1] = u.y;
  }
#pragma unroll
  for (int i = 0; i < VEC / 2; ++i) {
    uint32_t lo, hi;
    asm("prmt.b32 %0, %1, 0, 0x1044;" : "=r"(lo) : "r"(w[i]));
    asm("and.b32 %0, %1, 0xFFFF0000;" : "=r"(hi) : "r"(w[i]));
    f[i] = make_float2(__uint_as_float(lo), __uint_as_float(hi));
  }
}

// kPaged: K/V in a page pool addressed through the block table; each cache
// layout gets its own instantiation, so a kernel holds only the copy code it runs.
template <int D, int G, bool kPaged>
__global__ void __launch_bounds__(Traits<D, G>::kThreads, Traits<D, G>::kMinBlocks)
    gqa_decode_kernel(const DecodeParams p) {
  using T = Traits<D, G>;
  constexpr int V = T::kVec;
  extern __shared__ __align__(128) uint8_t smem[];

  // grid (kv head, row, split): every CTA of split 0 launches before any of
  // split 1, so a larger first chunk fills the SMs and the shorter ones fill
  // the tail
  const int split = blockIdx.z;
  const int kvh = blockIdx.x;
  const int b = blockIdx.y;                  // query row
  const int seq = b / p.rows_per_seq;        // its K/V stream
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool partial_out = p.out_acc != nullptr;

  allow_dependent_launch();
  // split 0 covers [0, c0), split s >= 1 covers [c0 + (s-1)*chunk, c0 + s*chunk)
  const int c0 = p.chunk0 > 0 ? p.chunk0 : p.chunk;
  const int tok_begin = split == 0 ? 0 : c0 + (split - 1) * p.chunk;
  if constexpr (!kPaged) {
    // With programmatic launch this CTA may be resident while the previous
    // grid drains.  Warm L2 with the first ring tiles of its chunk meanwhile,
    // bounded by the allocated rows (the length is not read before the wait):
    // one lane per (tile, K or V).  A prefetch cannot return stale data, so it
    // is safe even when the previous kernel writes the cache.
    if (p.l2_prefetch && p.rows_per_seq == 1 && threadIdx.x < 2 * T::kStages) {
      const int end = min(min(tok_begin + (split == 0 ? c0 : p.chunk), p.max_seq_len),
                          tok_begin + T::kStages * T::kTile);
      const int tok0 = tok_begin + (threadIdx.x >> 1) * T::kTile;
      if (tok0 < end) {
        const long long off = (long long)seq * p.kv_sb + (long long)kvh * p.kv_sh + (long long)tok0 * D;
        bulk_prefetch_l2(((threadIdx.x & 1) ? p.v : p.k) + off, (uint32_t)min(T::kTile, end - tok0) * T::kRowBytes);
      }
    }
  }
  grid_dependency_wait();  // the previous kernel's writes (q, lengths, cache, workspace) are visible from here
  const int len = seq_len_of(p, seq, b - seq * p.rows_per_seq);
  const int nsplit_b = len <= c0 ? 1 : 1 + (len - c0 + p.chunk - 1) / p.chunk;

  if (len == 0) {
    // No key is visible: the output is zero (the RTL normaliser maps l == 0
    // to 0).  One CTA per (b, kvh) writes it.
    if (split == 0) {
      for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        const int h = kvh * G + g;
        if (partial_out) {
          const long long row = (long long)b * p.n_q_heads + h;
          p.out_acc[row * D + d] = 0.f;
          if (d == 0) { p.out_ml[row * 2] = -INFINITY; p.out_ml[row * 2 + 1] = 0.f; }
        } else {
          p.o[b * p.o_sb + h * p.o_sh + d] = 0;
        }
      }
    }
    return;
  }
  if (tok_begin >= len) return;
  const int ntok = min(len - tok_begin, split == 0 ? c0 : p.chunk);
  const int ntiles = (ntok + T::kTile - 1) / T::kTile;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + T::kBarOff);
  uint64_t* empty = full + T::kStages;
  int* refill_round = reinterpret_cast<int*>(smem + T::kCntOff);
  int* flag = reinterpret_cast<int*>(smem + T::kFlagOff);
  float* pbuf = reinterpret_cast<float*>(smem + T::kPbufOff);
  float* cbuf = reinterpret_cast<float*>(smem + T::kCbufOff);

  const uint64_t pol = make_evict_first_policy();
  long long* pbase = reinterpret_cast<long long*>(smem + T::kPageOff);
  if constexpr (kPaged) {
    // validated block offsets of this CTA's chunk (the first kPageCache pages),
    // so a refill reads one shared-memory word
    const int first_page = tok_begin >> p.page_log2;
    const int npages = min(T::kPageCache, ((tok_begin + ntok - 1) >> p.page_log2) - first_page + 1);
    for (int i = threadIdx.x; i < npages; i += T::kThreads)
      pbase[i] = page_block(p.block_table, p.pages_per_seq, p.page_log2, p.num_pages, p.n_kv_heads, p.status, seq, kvh,
                            (first_page + i) << p.page_log2, D);
    __syncthreads();
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], T::kWarps);
      refill_round[s] = 0;
    }
    flag[0] = 0;  // error
    flag[1] = 0;  // last-CTA broadcast
    flag[2] = 0;  // tiles issued
    mbar_fence_init();
    if constexpr (!kPaged) {
      const int first = ntiles < T::kStages ? ntiles : T::kStages;
      for (int t = 0; t < first; ++t) issue_tile<D, G, false>(smem, full, t, ntok, p, seq, kvh, tok_begin, pbase, pol);
      flag[2] = first;
    }
  }
  if constexpr (kPaged) {
    if (warp == 0) {
      __syncwarp();  // lane 0's barrier initialisation is visible to the warp
      const int first = ntiles < T::kStages ? ntiles : T::kStages;
      for (int t = 0; t < first; ++t)
        issue_tile_paged_warp<D, G>(smem, full, t, ntok, p, seq, kvh, tok_begin, pbase, pol, lane);
      if (lane == 0) flag[2] = first;
    }
  }
  __syncthreads();

  const int half = lane / T::kLPT;            // which token row of the pass
  const int c = lane % T::kLPT;               // vector slot of the row
  // Pass order of this lane: reduce-scatter step s (< kHP) splits on pass bit
  // kLogIter - 1 - s with partner offset kLPT >> (s + 1); a lane whose offset
  // bit is set takes that pass bit flipped, so its kept half sits in the low slots.
  int xperm = 0;
#pragma unroll
  for (int s2 = 0; s2 < T::kHP; ++s2)
    xperm |= ((c >> (T::kLogLPT - 1 - s2)) & 1) << (T::kLogIter - 1 - s2);
  // Likewise the later steps split on a head bit: this lane keeps the query of
  // head g ^ yperm in register slot g, so those steps need no select either.
  int yperm = 0;
#pragma unroll
  for (int s2 = T::kHP; s2 < T::kH; ++s2)
    yperm |= ((c >> (T::kLogLPT - 1 - s2)) & 1) << (T::kLogG - 1 - (s2 - T::kLogIter));
  const int t_slot = c >> T::kR;              // finished-score slot after reduce-scatter
  const int my_g = t_slot % G;                // head of that score
  const int my_it = t_slot / G;               // pass of that score
  const int my_tw = my_it * T::kTPI + half;   // token (within the warp slice) of that score
  const bool dup_writer = (c & ((1 << T::kR) - 1)) == 0;
  const bool head_writer = dup_writer && lane < (G << T::kR);  // one lane per head, pass 0, row 0
  constexpr int V2 = V / 2;

  float2 qp[G][V2];
#pragma unroll
  for (int g = 0; g < G; ++g)
    load_bf16_pairs<V>(p.q + b * p.q_sb + (long long)(kvh * G + (g ^ yperm)) * p.q_sh + c * V, qp[g]);
  float2 acc[G][V2];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < V2; ++j) acc[g][j] = make_float2(0.f, 0.f);
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % T::kStages;
    const int round = i / T::kStages;
    // Paged cache: the block offset of the tile this warp may refill at the end
    // of the iteration is read now, so the refill does not wait on it.
    long long pre_base = -1;
    if constexpr (kPaged) {
      const int idx = ((tok_begin + (i + T::kStages) * T::kTile) >> p.page_log2) - (tok_begin >> p.page_log2);
      if (lane == 0 && idx < kPageCacheEntries) pre_base = pbase[idx];
    }
    if (!mbar_wait_bounded(&full[st], round & 1)) {
      ok = false;
      break;
    }
    const uint8_t* Kt = smem + st * T::kStageBytes + warp * T::kTokPerWarp * T::kRowBytes;
    const uint8_t* Vt = Kt + T::kHalfStage;
    const int nvalid = min(T::kTile, ntok - i * T::kTile) - warp * T::kTokPerWarp;

    // QK^T: ITER token rows x G heads of partial dot products over V dims,
    // accumulated as (even, odd) dim pairs with packed fp32 FMA.  Slot
    // it * G + g holds pass it ^ xperm of head g (see the reduce-scatter).
    float part[T::kNV];
#pragma unroll
    for (int it = 0; it < T::kIter; ++it) {
      const int tw = (it ^ xperm) * T::kTPI + half;
      float2 kp[V2];
      load_bf16_pairs_alu<V>(reinterpret_cast<const uint16_t*>(Kt + tw * T::kRowBytes) + c * V, kp);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float2 a2 = __fmul2_rn(qp[g][0], kp[0]);
#pragma unroll
        for (int j = 1; j < V2; ++j) a2 = __ffma2_rn(qp[g][j], kp[j], a2);
        part[it * G + g] = a2.x + a2.y;
      }
    }
    // Reduce-scatter over the row's lanes: each step halves the values a lane
    // keeps and adds the partner's matching half.  Each step's half boundary
    // is a bit of the pass index (first kHP steps) or of the head index; every
    // lane took its passes in the order it ^ xperm and holds head g ^ yperm in
    // slot g, so the half it keeps is always in its low slots and it simply
    // sends the high slots.
#pragma unroll
    for (int step = 0; step < T::kH; ++step) {
      const int off = T::kLPT >> (step + 1);
      const int nv = T::kNV >> step;
      // two kept values per packed FADD2 (the same two round-to-nearest sums)
#pragma unroll
      for (int j = 0; j + 1 < nv / 2; j += 2) {
        const float2 mine = make_float2(part[j], part[j + 1]);
        const float2 theirs = make_float2(__shfl_xor_sync(0xffffffffu, part[j + nv / 2], off),
                                          __shfl_xor_sync(0xffffffffu, part[j + 1 + nv / 2], off));
        const float2 sum = __fadd2_rn(mine, theirs);
        part[j] = sum.x;
        part[j + 1] = sum.y;
      }
      if ((nv / 2) & 1) part[nv / 2 - 1] += __shfl_xor_sync(0xffffffffu, part[nv - 1], off);
    }
#pragma unroll
    for (int step = 0; step < T::kR; ++step) {
      const int off = (T::kLPT >> T::kH) >> (step + 1);
      part[0] += __shfl_xor_sync(0xffffffffu, part[0], off);
    }
    const float s = (my_tw < nvalid) ? part[0] * p.scale_log2 : -INFINITY;

    // Online softmax for this lane's head over the warp's token slice.
    float tmax = s;
#pragma unroll
    for (int off = 1 << (T::kR + T::kLogG); off < 32; off <<= 1)
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    const float m_new = fmaxf(m_run, tmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float corr = ex2_ftz(m_run - m_use);
    const float pr = ex2_ftz(s - m_use);
    // this lane's share of the head's running sum (the head's lanes share
    // m_run, so their shares add up to l after the loop)
    l_run = fmaf(l_run, corr, pr);
    // The accumulator needs rescaling only if some head's running max moved.
    const bool moved = __any_sync(0xffffffffu, m_new != m_run);
    m_run = m_new;

    float* pb = pbuf + ((i & 1) * T::kWarps + warp) * (T::kTokPerWarp * G);
    float* cb = cbuf + ((i & 1) * T::kWarps + warp) * G;
    if (dup_writer) pb[my_tw * G + my_g] = pr;
    if (head_writer) cb[my_g] = corr;
    __syncwarp();

    // P.V with the rescale of the running accumulator.
    if (moved) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float cr = cb[g];
        const float2 cr2 = make_float2(cr, cr);
#pragma unroll
        for (int j = 0; j < V2; ++j) acc[g][j] = __fmul2_rn(acc[g][j], cr2);
      }
    }
    // Every warp row of a full tile holds a visible token: the per-row check
    // is only needed on the item's last (partial) tile.
    auto pv_row = [&](int tw) {
      float2 vp[V2];
      load_bf16_pairs_alu<V>(reinterpret_cast<const uint16_t*>(Vt + tw * T::kRowBytes) + c * V, vp);
      float pg[G];
      const float* prow = pb + tw * G;
      if constexpr (G % 4 == 0) {
#pragma unroll
        for (int g = 0; g < G; g += 4) {
          const float4 f = *reinterpret_cast<const float4*>(prow + g);
          pg[g] = f.x; pg[g + 1] = f.y; pg[g + 2] = f.z; pg[g + 3] = f.w;
        }
      } else if constexpr (G == 2) {
        const float2 f = *reinterpret_cast<const float2*>(prow);
        pg[0] = f.x; pg[1] = f.y;
      } else {
        pg[0] = prow[0];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float2 p2 = make_float2(pg[g], pg[g]);
#pragma unroll
        for (int j = 0; j < V2; ++j) acc[g][j] = __ffma2_rn(p2, vp[j], acc[g][j]);
      }
    };
    if (nvalid >= T::kTokPerWarp) {
#pragma unroll
      for (int it = 0; it < T::kIter; ++it) pv_row(it * T::kTPI + half);
    } else {
#pragma unroll
      for (int it = 0; it < T::kIter; ++it)
        if (it * T::kTPI + half < nvalid) pv_row(it * T::kTPI + half);
    }
    // Release the stage (mbarrier arrive: release semantics).  A warp that
    // then observes the release complete (test_wait: acquire) claims the
    // refill of tile i + kStages with one CAS; nobody blocks on it.
    __syncwarp();
    if constexpr (kPaged) {
      const int nxt = i + T::kStages;
      int claim = 0;
      if (lane == 0) {
        mbar_arrive(&empty[st]);
        claim = nxt < ntiles && mbar_test_wait(&empty[st], round & 1) &&
                atomicCAS(&refill_round[st], round, round + 1) == round;
      }
      if (__shfl_sync(0xffffffffu, claim, 0)) {
        issue_tile_paged_warp<D, G>(smem, full, nxt, ntok, p, seq, kvh, tok_begin, pbase, pol, lane, pre_base);
        if (lane == 0) atomicMax(&flag[2], nxt + 1);
      }
    } else if (lane == 0) {
      mbar_arrive(&empty[st]);
      const int nxt = i + T::kStages;
      if (nxt < ntiles && mbar_test_wait(&empty[st], round & 1) &&
          atomicCAS(&refill_round[st], round, round + 1) == round) {
        issue_tile<D, G, false>(smem, full, nxt, ntok, p, seq, kvh, tok_begin, pbase, pol, pre_base);
        atomicMax(&flag[2], nxt + 1);
      }
    }
  }

  // The head's running sum: add the shares of its lanes (duplicate lanes of
  // a score hold equal shares and are not added twice).
#pragma unroll
  for (int off = 1 << (T::kR + T::kLogG); off < 32; off <<= 1) l_run += __shfl_xor_sync(0xffffffffu, l_run, off);
  // Token rows of one pass were split across lane groups: add them up.
#pragma unroll
  for (int off = T::kLPT; off < 32; off <<= 1)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < V2; ++j) {
        acc[g][j].x += __shfl_xor_sync(0xffffffffu, acc[g][j].x, off);
        acc[g][j].y += __shfl_xor_sync(0xffffffffu, acc[g][j].y, off);
      }

  if (!ok) atomicExch(&flag[0], 1);
  __syncthreads();
  if (flag[0]) {
    if (threadIdx.x == 0) {
      atomicOr(p.status, kDevWaitTimeout);
      // Let copies already issued land before the CTA retires.
      const int issued = flag[2];
      for (int t = (issued > T::kStages ? issued - T::kStages : 0); t < issued; ++t)
        (void)mbar_wait_bounded(&full[t % T::kStages], (t / T::kStages) & 1);
    }
    return;
  }

  // ---- merge the warps (the ring is idle: every stage has been consumed) ----
  float* mw = reinterpret_cast<float*>(smem);            // [warps][G]
  float* lw = mw + T::kWarps * G;                         // [warps][G]
  float* aw = lw + T::kWarps * G;                         // [warps][G][D]
  if (half == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < V2; j += 2)
        *reinterpret_cast<float4*>(aw + (warp * G + g) * D + c * V + 2 * j) =
            make_float4(acc[g][j].x, acc[g][j].y, acc[g][j + 1].x, acc[g][j + 1].y);
  }
  if (head_writer) {
    mw[warp * G + my_g] = m_run;
    lw[warp * G + my_g] = l_run;
  }
  __syncthreads();

  const bool single = (nsplit_b == 1);
  const int tid = threadIdx.x;
  // Each thread finishes pairs of adjacent dims of one head.
  for (int idx = tid; idx < G * D / 2; idx += T::kThreads) {
    const int g = idx / (D / 2);
    const int d = (idx % (D / 2)) * 2;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < T::kWarps; ++w) M = fmaxf(M, mw[w * G + g]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int w = 0; w < T::kWarps; ++w) {
      const float sc = exp2f(mw[w * G + g] - Mu);
      L = fmaf(lw[w * G + g], sc, L);
      o0 = fmaf(aw[(w * G + g) * D + d], sc, o0);
      o1 = fmaf(aw[(w * G + g) * D + d + 1], sc, o1);
    }
    const int h = kvh * G + g;
    const long long row = (long long)b * p.n_q_heads + h;
    if (single) {
      if (partial_out) {
        *reinterpret_cast<float2*>(p.out_acc + row * D + d) = make_float2(o0, o1);
        if (d == 0) { p.out_ml[row * 2] = M; p.out_ml[row * 2 + 1] = L; }
      } else {
        const float inv = (L > 0.f) ? 1.f / L : 0.f;
        *reinterpret_cast<uint32_t*>(p.o + b * p.o_sb + h * p.o_sh + d) = pack2_bf16(o0 * inv, o1 * inv);
      }
    } else {
      const long long slot = row * p.nsplit + split;
      *reinterpret_cast<float2*>(p.part_acc + slot * D + d) = make_float2(o0, o1);
      if (d == 0) { p.part_ml[slot * 2] = M; p.part_ml[slot * 2 + 1] = L; }
    }
  }
  if (single) return;

  // ---- split-KV: the last CTA of this (b, kvh) merges all splits ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* ctr = p.counters + b * p.n_kv_heads + kvh;
    const int prev = atomicAdd(ctr, 1);
    const int last = (prev == nsplit_b - 1);
    if (last) *ctr = 0;  // every other split has arrived: reset for the next launch
    flag[1] = last;
  }
  __syncthreads();
  if (!flag[1]) return;
  __threadfence();
  merge_split_partials<D>(p, b, kvh, G, nsplit_b, partial_out, tid, T::kThreads);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

struct KernelInfo {
  const void* fn = nullptr;
  int threads = 0, smem = 0, tile = 0;
};

template <int D, int G>
KernelInfo info_for(bool paged) {
  using T = Traits<D, G>;
  const void* fn = paged ? reinterpret_cast<const void*>(&gqa_decode_kernel<D, G, true>)
                         : reinterpret_cast<const void*>(&gqa_decode_kernel<D, G, false>);
  return KernelInfo{fn, T::kThreads, T::kSmemBytes, T::kTile};
}

KernelInfo lookup(int D, int G, bool paged = false) {
#define LARA_CASE(d, g) \
  if (D == d && G == g) return info_for<d, g>(paged);
  LARA_CASE(128, 1) LARA_CASE(128, 2) LARA_CASE(128, 4) LARA_CASE(128, 8)
  LARA_CASE(64, 1) LARA_CASE(64, 2) LARA_CASE(64, 4) LARA_CASE(64, 8)
#undef LARA_CASE
  return KernelInfo{};
}

constexpr int kMaxDevices = 64;

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int occupancy(const KernelInfo& k) {
  int n = 0;
  cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, k.threads, k.smem);
  return n < 1 ? 1 : n;
}

}  // namespace

int device_sm_count() {
  static int cache[kMaxDevices] = {};
  const int dev = current_device();
  if (dev >= 0 && dev < kMaxDevices && cache[dev] > 0) return cache[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < kMaxDevices) cache[dev] = n;
  return n;
}

cudaError_t launch_with_pdl(const void* fn, dim3 grid, dim3 block, void** args, size_t smem, cudaStream_t stream) {
  static const bool enabled = [] {
    const char* e = std::getenv("LARA_PDL");
    return !(e && e[0] == '0');
  }();
  if (!enabled) return cudaLaunchKernel(fn, grid, block, args, smem, stream);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

int decode_tile_tokens(int head_dim, int group) { return lookup(head_dim, group).tile; }

int decode_chunk_granule(int head_dim, int group) {
  const int tile = decode_tile_tokens(head_dim, group);
  if (tile > 0) return tile;
  return decode_tc_selected(head_dim, group) ? 128 : 0;
}

WorkspaceLayout decode_workspace_layout(int batch, int n_q_heads, int n_kv_heads, int head_dim, int nsplit) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  WorkspaceLayout w;
  w.status_off = 0;
  w.counters_off = 256;
  w.ml_off = w.counters_off + up(sizeof(int) * (size_t)batch * n_kv_heads);
  const size_t rows = (size_t)batch * n_q_heads * (size_t)(nsplit > 1 ? nsplit : 0);
  w.acc_off = w.ml_off + up(sizeof(float) * rows * 2);
  w.total = w.acc_off + up(sizeof(float) * rows * head_dim);
  return w;
}

void decode_plan(int batch, int n_kv_heads, int n_q_heads, int head_dim, int max_tokens, const int32_t* lens_host,
                 int* nsplit_out, int* chunk_out) {
  const int group = n_kv_heads > 0 ? n_q_heads / n_kv_heads : 1;
  if (decode_tc_selected(head_dim, group)) {
    decode_tc_plan(batch, n_kv_heads, max_tokens, lens_host, nsplit_out, chunk_out);
    return;
  }
  const KernelInfo k = lookup(head_dim, group);
  const int tile = k.tile > 0 ? k.tile : 64;
  const int L = max_tokens < 1 ? 1 : max_tokens;
  const int cps = k.fn ? occupancy(k) : 1;
  // Tokens of latency a CTA spends before its stream runs (exposed when the
  // SM holds a single CTA, mostly hidden behind a neighbour otherwise).
  const double ovh = 2.0 * tile;
  bool uniform = true;
  long long total = 0;
  if (lens_host) {
    for (int b = 0; b < batch; ++b) {
      total += lens_host[b];
      if (lens_host[b] != lens_host[0]) uniform = false;
    }
  } else {
    total = (long long)batch * L;
  }
  const int max_tiles = (L + tile - 1) / tile;
  double best = 1e300;
  int best_s = 1, best_chunk = max_tiles * tile;
  for (int s = 1; s <= 256 && s <= max_tiles; ++s) {
    const int chunk = ((max_tiles + s - 1) / s) * tile;
    const int s_eff = (L + chunk - 1) / chunk;
    double cost;
    // Bandwidth-bound: the step ends when the SM with the most tokens to
    // stream is done; every CTA adds ~ovh tokens of prologue/epilogue.
    const long long sms = device_sm_count();
    if (uniform) {
      const int len0 = lens_host ? (lens_host[0] < 1 ? 1 : lens_host[0]) : L;
      const long long units = (long long)batch * n_kv_heads;
      const long long ctas = units * ((len0 + chunk - 1) / chunk);
      const long long per_sm = (ctas + sms - 1) / sms;
      const int per = len0 < chunk ? len0 : chunk;
      // An SM that only ever holds one CTA streams at about 70% of the rate
      // it reaches with two resident CTAs (config-2 split sweeps on B200);
      // with more CTAs per SM the neighbour hides each one's prologue.
      const double lone = (cps > 1 && per_sm == 1) ? 1.0 / 0.7 : 1.0;
      cost = (double)per_sm * (per + ovh) * lone;
      const int c0 = decode_first_chunk(s_eff, chunk, group, head_dim, units, L);
      if (c0 > 0 && len0 > chunk) {
        // Long first chunks, launched first, cover every SM; the short second
        // chunks then fill whichever SM frees a slot, so the busiest SM holds
        // its share of first chunks or the average load plus one short chunk.
        const double first = (double)((units + sms - 1) / sms) * (c0 + ovh);
        const double fill = (double)units * len0 / sms + (len0 - c0) + 2 * ovh;
        cost = first > fill ? first : fill;
      }
    } else {
      long long ctas = 0;
      for (int b = 0; b < batch; ++b) ctas += (lens_host[b] + chunk - 1) / chunk;
      ctas *= n_kv_heads;
      cost = ((double)total * n_kv_heads + (double)ctas * ovh) / (double)sms + 0.5 * chunk;
    }
    if (cost < best * (1.0 - 1e-6)) {
      best = cost;
      best_s = s_eff;
      best_chunk = chunk;
    }
  }
  *nsplit_out = best_s;
  *chunk_out = best_chunk;
}

int decode_first_chunk(int nsplit, int chunk, int group, int head_dim, long long units, int max_seq_len) {
  if (nsplit >= 1 && chunk > 0 && (long long)nsplit * chunk < max_seq_len) {
    // Splits 1.. take `chunk` tokens each and split 0 the rest, rounded up to
    // 128 tokens (a multiple of every kernel's tile, so either decode kernel
    // can run the plan).
    const int granule = decode_chunk_granule(head_dim, group);
    if (granule <= 0) return 0;
    const int g = 128 % granule == 0 ? 128 : granule;
    const long long rest = (long long)max_seq_len - (long long)(nsplit - 1) * chunk;
    return (int)((rest + g - 1) / g * g);
  }
  if (nsplit != 2 || decode_tc_selected(head_dim, group)) return 0;
  if (units < device_sm_count()) return 0;
  const int tile = decode_tile_tokens(head_dim, group);
  if (tile <= 0) return 0;
  const long long span = 2ll * chunk;
  const int c0 = (int)((span * 7 / 8) / tile * tile);
  return c0 > chunk ? c0 : 0;  // c0 + chunk >= 2 * chunk covers what the plan covered
}

cudaError_t decode_launch(const DecodeParams& p, cudaStream_t stream) {
  static const bool prefetch = [] {
    const char* e = std::getenv("LARA_L2_PREFETCH");
    return !(e && e[0] == '0');
  }();
  DecodeParams lp = p;
  lp.l2_prefetch = prefetch ? 1 : 0;
  const int group = p.n_q_heads / p.n_kv_heads;
  if (decode_tc_selected(p.head_dim, group)) {
    const cudaError_t e = decode_tc_launch(lp, stream);
    if (e != cudaErrorNotSupported) return e;
  }
  const KernelInfo k = lookup(p.head_dim, group, p.block_table != nullptr);
  if (!k.fn) return cudaErrorInvalidValue;
  if (p.chunk <= 0 || p.chunk % k.tile != 0 || p.nsplit <= 0) return cudaErrorInvalidValue;
  if (p.chunk0 < 0 || p.chunk0 % k.tile != 0) return cudaErrorInvalidValue;
  // The splits must cover every token a sequence may hold, or the last-CTA
  // merge of a longer sequence would never see all of its splits.
  const long long c0 = p.chunk0 > 0 ? p.chunk0 : p.chunk;
  if (c0 + (long long)(p.nsplit - 1) * p.chunk < (long long)p.max_seq_len) return cudaErrorInvalidValue;
  {
    // the shared-memory opt-in is per (kernel, device): set it once
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (!done.count({k.fn, dev})) {
      e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
      if (e != cudaSuccess) return e;
      done.insert({k.fn, dev});
    }
  }
  if (p.rows_per_seq < 1 || p.batch > 65535) return cudaErrorInvalidValue;
  if (p.nsplit > 65535) return cudaErrorInvalidValue;
  dim3 grid(p.n_kv_heads, p.batch, p.nsplit);
  void* args[] = {&lp};
  return launch_with_pdl(k.fn, grid, dim3(k.threads), args, k.smem, stream);
}

}  // namespace lara
