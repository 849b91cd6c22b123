// GQA decode attention on the 5th-generation tensor cores (tcgen05 + TMEM,
// sm_100a): a persistent kernel for head_dim 128 and groups of up to 16
// query heads per KV head.
//
// Same contract as the CUDA-core decode kernel (DecodeParams: query rows,
// per-row lengths, splits of `chunk` tokens, bf16 output or (m, l, acc)
// partials, last-arriver split merge), and the same arithmetic as the
// reference datapath (hw/rtl/attn_top.sv:301-625: QK^T, scale, online
// softmax per block, P.V, O = O*corr + dO, normalise by l).  The G query
// heads of a KV group are the N = 16 columns of two small MMAs per tile of
// 128 cached tokens:
//
//   S^T [128 tokens x 16]   = K_tile [128 x 128] . Q^T      A = K (K-major), B = Q (K-major)
//   O^T [128 dims x 16]     = V_tile^T [128 x 128] . P^T    A = V (MN-major), B = P^T (K-major)
//
// so the group's FLOPs (8 per cached byte at G = 8) leave the CUDA cores and
// the SM only streams K/V.  P is split as P_hi + P_lo (two bf16 terms, ~16
// significant bits) for a second PV pass, so the result keeps the accuracy
// of an fp32 P.
//
// One CTA per SM, 10 warps:
//   warp 4 (TMA)   takes work items (query row, kv head, split) from a ticket
//                  counter in the workspace and streams each item's Q (once)
//                  and K/V tiles back to back through a 3-stage ring of
//                  64 KB stages (tensor-map copies, 128-byte swizzle, L2
//                  evict-first, no multicast).  Each stage carries a small
//                  descriptor of its tile (row, head, token range, item
//                  boundaries); items without tokens travel as marker stages.
//   warp 5 (MMA)   one thread issues S(n+1) before PV(n), so the softmax of
//                  one tile overlaps the tensor core's work on the next.
//   warps 0-3      TMEM lane t: token t of a tile for the softmax (scale,
//                  length mask, per-head tile max by redux.sync and a 4-warp
//                  exchange, exp2, P_hi/P_lo into shared memory), and head
//                  dim t of the output (O^T of each tile added into registers
//                  with the online-softmax correction).  At an item's end
//                  they hand its O^T (TMEM), row maxima and per-warp row
//                  sums to the epilogue warps and go on with the next item.
//   warps 6-9      epilogue, TMEM lane t = head dim t: normalise and write
//                  the item's output, or write its split partial and, as the
//                  last split of the row to finish, merge the partials.  The
//                  global-memory round trips of an item's end (fence,
//                  arrival counter, merge) are off the streaming path.
//
// TMEM: S^T in columns [0, 32) (two buffers of 16), O^T in [32, 64), the
// epilogue hand-off in [64, 96) (two buffers of 16).
// Every wait is bounded by %globaltimer (the 128 softmax threads also meet on
// an mbarrier rather than bar.sync); on a timeout the CTA flags the status
// word, drains its own tensor-core work and copies, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

#include "common.cuh"
#include "decode_merge.cuh"
#include "lara_internal.h"
#include "tcgen05.cuh"

namespace lara {

using namespace tc;

namespace {

constexpr int kD = 128;                  // head_dim
constexpr int kTile = 128;               // tokens per tile (TMEM lanes of S^T)
constexpr int kN = 16;                   // MMA N: query heads of the group, padded
constexpr int kHalf = kTile * 128;       // [128 rows][64 bf16] with 128-byte swizzle
constexpr int kKVBytes = 2 * kHalf;      // one K (or V) tile
constexpr int kStages = 3;
constexpr int kOpBytes = 2 * kN * 128;   // [2 k-blocks][16 rows][128 B]: Q, or one of P_hi / P_lo
constexpr int kKOff = 0;
constexpr int kVOff = kKOff + kStages * kKVBytes;
constexpr int kQOff = kVOff + kStages * kKVBytes;   // two item buffers
constexpr int kPOff = kQOff + 2 * kOpBytes;         // two tile buffers x (P_hi, P_lo)
constexpr int kXOff = kPOff + 4 * kOpBytes;         // exchange: tile max [2][4][16], row sums [4][16], flag
constexpr int kMetaOff = kXOff + 1024;
constexpr int kBarOff = kMetaOff + 256;
constexpr int kPageCache = 512;                     // block-table entries of an item kept in shared memory
constexpr int kHandOff = kBarOff + 256;             // epilogue hand-off descriptors (two)
constexpr int kPageOff = kHandOff + 1024;
constexpr int kSmemAlloc = kPageOff + kPageCache * 4 + 1024;  // + slack for 1024-byte alignment
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kHandCol = 64;                   // TMEM columns of the hand-off buffers
constexpr int kTmaWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kThreads = 10 * 32;                   // warps 6-9 (epilogue): TMEM lane quarters 2, 3, 0, 1
constexpr unsigned kFull = 0xffffffffu;

enum : int { kEntryTile = 0, kEntryZero = 1, kEntryEnd = 2 };

// One ring stage's work, written by the producer before it arrives on the
// stage's full barrier.
struct Meta {
  int kind;      // kEntryTile, kEntryZero (a row with no visible key), kEntryEnd
  int row;       // query row
  int kvh;
  int split;
  int tok0;      // first token of the tile
  int tok_end;   // end of the item's tokens
  int nsplit_b;  // splits that hold tokens of this row
  int flags;     // bit 0: first tile of its item, bit 1: last tile
  int seq_kv;    // K/V sequence coordinate of the tensor maps
  int qslot;     // Q buffer of the item
  int qpar;      // phase parity of that buffer's load
  int pad[5];
};
static_assert(sizeof(Meta) == 64 && kStages * sizeof(Meta) <= 256, "stage descriptors");

struct Bars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t q_full[2];
  uint64_t q_free[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2];
  uint64_t sync;   // the 128 softmax threads
  uint64_t drain;
  uint64_t epi_full[2];  // hand-off written (128 softmax arrivals)
  uint64_t epi_free[2];  // hand-off read (128 epilogue arrivals)
  uint64_t esync;        // the 128 epilogue threads
  uint32_t tmem_base;
  int abort;
  int issued;      // ring entries pushed
  int q_issued;    // Q loads issued
  int last_split;  // epilogue: this CTA merges the row's splits
};
static_assert(sizeof(Bars) <= 256, "barrier block");

// An item's result handed from the softmax warps to the epilogue warps (its
// O^T columns travel in TMEM).
struct Hand {
  int kind;      // kEntryTile (an item's result) or kEntryEnd
  int row;
  int kvh;
  int split;
  int nsplit_b;
  int pad[3];
  float m[16];     // running max per head (log2 domain)
  float l[4][16];  // row-sum share of each softmax warp
};
static_assert(2 * sizeof(Hand) <= 1024, "hand-off block");

struct TcDecodeArgs {
  unsigned n_items;  // nsplit * batch * n_kv_heads
  int kv_shared;     // every row reads K/V sequence 0 (kv_sb == 0)
  int q_rows;        // rows of the Q box (min(16, n_q_heads))
  int page_box;      // paged cache: token rows per copy (min(128, page size)); 0 = contiguous cache
};

__device__ __forceinline__ float warp_max(float x) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ int row_len(const DecodeParams& p, int seq, int row_in_seq) {
  long long len = (long long)p.len_c0 + (long long)p.len_c1 * row_in_seq;
  if (p.lens) {
    const int l = p.lens[seq];
    if (l < 0 || l > p.max_seq_len) atomicOr(p.status, kDevBadLength);
    len += l;
  }
  return len < 0 ? 0 : (len > p.max_seq_len ? p.max_seq_len : (int)len);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(kFull, x, off);
  return x;
}

// Merge the split partials of (row b, kv head kvh) with the log-sum-exp rule
// (M = max m_s, L = sum l_s 2^(m_s - M), o = sum acc_s 2^(m_s - M) / L).
// Warp w takes heads w, w + 4, ...; lane i holds split i's weight and dims
// 4i .. 4i+3 of the accumulator, so every load of a pass is independent.
template <int G>
__device__ __forceinline__ void merge_splits_tc(const DecodeParams& p, int b, int kvh, int nsplit_b,
                                                bool partial_out, int warp, int lane) {
  for (int g = warp; g < G; g += 4) {
    const int h = kvh * G + g;
    const long long row = (long long)b * p.n_q_heads + h;
    const float* ml = p.part_ml + row * p.nsplit * 2;
    const float* pa = p.part_acc + row * p.nsplit * kD;
    float M = -INFINITY;
    for (int s = lane; s < nsplit_b; s += 32) M = fmaxf(M, __ldcg(ml + 2 * s));
    M = warp_max(M);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < nsplit_b; s0 += 32) {
      const int sl = s0 + lane;
      const float2 mls = sl < nsplit_b ? __ldcg(reinterpret_cast<const float2*>(ml + 2 * sl)) : make_float2(0.f, 0.f);
      const float w_lane = sl < nsplit_b ? exp2f(mls.x - Mu) : 0.f;
      L = fmaf(mls.y, w_lane, L);
      const int cnt = min(32, nsplit_b - s0);
#pragma unroll 8
      for (int j = 0; j < cnt; ++j) {
        const float w = __shfl_sync(kFull, w_lane, j);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(pa + (long long)(s0 + j) * kD) + lane);
        o.x = fmaf(a.x, w, o.x);
        o.y = fmaf(a.y, w, o.y);
        o.z = fmaf(a.z, w, o.z);
        o.w = fmaf(a.w, w, o.w);
      }
    }
    L = warp_sum(L);
    if (partial_out) {
      float2* dst = reinterpret_cast<float2*>(p.out_acc + row * kD + 4 * lane);  // out_acc is 8-byte aligned
      dst[0] = make_float2(o.x, o.y);
      dst[1] = make_float2(o.z, o.w);
      if (lane == 0) { p.out_ml[row * 2] = M; p.out_ml[row * 2 + 1] = L; }
    } else {
      const float inv = (L > 0.f) ? 1.f / L : 0.f;
      uint32_t* dst = reinterpret_cast<uint32_t*>(p.o + b * p.o_sb + h * p.o_sh + 4 * lane);
      dst[0] = pack2_bf16(o.x * inv, o.y * inv);
      dst[1] = pack2_bf16(o.z * inv, o.w * inv);
    }
  }
}

// Page holding token `tok` of a sequence whose block-table row is `bt_row`,
// for a token past the item's shared-memory cache (items of more than
// kPageCache pages); out of line so the per-tile copy path stays short.  An
// out-of-range entry flags the status word and reads page 0, so every copy
// stays in bounds and completes.
__device__ __noinline__ int page_uncached(const int32_t* bt_row, int tok, int page_log2, int num_pages, int* status) {
  int pg = __ldg(bt_row + (tok >> page_log2));
  if (pg < 0 || pg >= num_pages) {
    atomicOr(status, kDevBadPage);
    pg = 0;
  }
  return pg;
}

// 128-thread meeting point of the softmax warps on an mbarrier (bounded).
__device__ __forceinline__ bool group_sync(uint64_t* bar, uint32_t& phase, volatile int* abort) {
  mbar_arrive(bar);
  const bool ok = wait_or_abort(bar, phase & 1, abort);
  ++phase;
  return __all_sync(kFull, ok);
}

// kPaged: K/V in a page pool addressed through the block table; each cache
// layout gets its own instantiation, so a kernel holds only the copy code it
// runs (the per-tile loops are sensitive to instruction-cache pressure).
template <int G, bool kPaged>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const DecodeParams p, const TcDecodeArgs a) {
  constexpr int NC = G <= 8 ? 8 : 16;  // TMEM columns read per lane
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kBarOff);
  Meta* metas = reinterpret_cast<Meta*>(smem + kMetaOff);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned* queue = reinterpret_cast<unsigned*>(p.status + 32);  // [0] ticket, [1] finished CTAs

  allow_dependent_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_free[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->o_full[i], 1);
    }
    mbar_init(&bars->sync, 128);
    mbar_init(&bars->drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->epi_full[i], 128);
      mbar_init(&bars->epi_free[i], 128);
    }
    mbar_init(&bars->esync, 128);
    bars->abort = 0;
    bars->issued = 0;
    bars->q_issued = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x < 128) {
    // P^T rows >= G stay zero for the whole kernel, so padded heads add nothing
    uint4* pz = reinterpret_cast<uint4*>(smem + kPOff) + threadIdx.x * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) pz[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  // global memory (tickets, q, lengths, cache) only after the previous grid is done
  grid_dependency_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------ producer
    // Lane 0 issues every copy.  For a paged cache the whole warp first loads
    // the item's block-table entries into a shared-memory cache, so a tile
    // costs no dependent global load (one load latency per item).
    const uint64_t pol = make_evict_first_policy();
    const int per_split = p.batch * p.n_kv_heads;
    const int c0 = p.chunk0 > 0 ? p.chunk0 : p.chunk;
    const uint32_t q_bytes = 2u * 128u * (uint32_t)a.q_rows;
    int* pcache = reinterpret_cast<int*>(smem + kPageOff);
    const int32_t* bt_row = p.block_table;
    int pg0 = 0;  // page index held by cache entry 0 (current item)
    int n = 0, qi = 0;
    auto page_at = [&](int tok) -> int {  // cache entries are validated when loaded
      const int idx = (tok >> p.page_log2) - pg0;
      return idx < kPageCache ? pcache[idx] : page_uncached(bt_row, tok, p.page_log2, p.num_pages, p.status);
    };
    auto push = [&](const Meta& m, bool copies) -> bool {  // lane 0
      const int st = n % kStages;
      if (n >= kStages && !wait_or_abort(&bars->empty[st], ((n / kStages) - 1) & 1, abort)) return false;
      metas[st] = m;
      if (copies) {
        if constexpr (!kPaged) {
          uint8_t* ks = smem + kKOff + st * kKVBytes;
          uint8_t* vs = smem + kVOff + st * kKVBytes;
          mbar_arrive_expect_tx(&bars->full[st], 2 * kKVBytes);
          tma_load_4d_hint(ks, &tm_k, 0, m.tok0, m.kvh, m.seq_kv, &bars->full[st], pol);
          tma_load_4d_hint(ks + kHalf, &tm_k, 64, m.tok0, m.kvh, m.seq_kv, &bars->full[st], pol);
          tma_load_4d_hint(vs, &tm_v, 0, m.tok0, m.kvh, m.seq_kv, &bars->full[st], pol);
          tma_load_4d_hint(vs + kHalf, &tm_v, 64, m.tok0, m.kvh, m.seq_kv, &bars->full[st], pol);
        } else {
          // paged cache: the tile is page_box-row pieces of whole pages (tiles
          // start on 128-token boundaries); pieces past the item's end are not
          // loaded (their rows are masked, and V rows zeroed, by the softmax)
          uint8_t* ks = smem + kKOff + st * kKVBytes;
          uint8_t* vs = smem + kVOff + st * kKVBytes;
          const int bx = a.page_box;
          const int ps_mask = (1 << p.page_log2) - 1;
          if (bx == kTile) {
            // pages of >= 128 tokens: the tile is one piece of one page
            const int pg = page_at(m.tok0);
            const int in_page = m.tok0 & ps_mask;
            mbar_arrive_expect_tx(&bars->full[st], 2 * kKVBytes);
            tma_load_4d_hint(ks, &tm_k, 0, in_page, m.kvh, pg, &bars->full[st], pol);
            tma_load_4d_hint(ks + kHalf, &tm_k, 64, in_page, m.kvh, pg, &bars->full[st], pol);
            tma_load_4d_hint(vs, &tm_v, 0, in_page, m.kvh, pg, &bars->full[st], pol);
            tma_load_4d_hint(vs + kHalf, &tm_v, 64, in_page, m.kvh, pg, &bars->full[st], pol);
          } else {
            // pages of < 128 tokens (bx = page size): the tile starts on a page
            // boundary, so piece i is the whole of page pg0 + idx0 + i
            const int lg = p.page_log2;
            const int pieces = min(kTile >> lg, (m.tok_end - m.tok0 + bx - 1) >> lg);
            const int idx0 = (m.tok0 >> lg) - pg0;
            mbar_arrive_expect_tx(&bars->full[st], (uint32_t)pieces * 4u * (uint32_t)bx * 128u);
            for (int i = 0; i < pieces; ++i) {
              const int idx = idx0 + i;
              const int pg = idx < kPageCache ? pcache[idx]
                                              : page_uncached(bt_row, m.tok0 + (i << lg), lg, p.num_pages, p.status);
              const int off = (i << lg) * 128;
              tma_load_4d_hint(ks + off, &tm_k, 0, 0, m.kvh, pg, &bars->full[st], pol);
              tma_load_4d_hint(ks + kHalf + off, &tm_k, 64, 0, m.kvh, pg, &bars->full[st], pol);
              tma_load_4d_hint(vs + off, &tm_v, 0, 0, m.kvh, pg, &bars->full[st], pol);
              tma_load_4d_hint(vs + kHalf + off, &tm_v, 64, 0, m.kvh, pg, &bars->full[st], pol);
            }
          }
        }
      } else {
        mbar_arrive(&bars->full[st]);
      }
      bars->issued = ++n;
      return true;
    };
    // Paged caches: the same as push(m, true), called by the whole warp; lane
    // 0 keeps the ring, and when pages are shorter than a tile every lane
    // issues one (page piece, K or V, 64-column half) box, so a tile costs one
    // copy's issue latency instead of 4 x pieces copies in a row.
    auto push_tile_warp = [&](const Meta& m) -> bool {
      n = __shfl_sync(kFull, n, 0);
      const int st = n % kStages;
      int good = 1;
      if (lane == 0) {
        if (n >= kStages && !wait_or_abort(&bars->empty[st], ((n / kStages) - 1) & 1, abort))
          good = 0;
        else
          metas[st] = m;
      }
      if (!__shfl_sync(kFull, good, 0)) return false;
      uint8_t* ks = smem + kKOff + st * kKVBytes;
      uint8_t* vs = smem + kVOff + st * kKVBytes;
      const int bx = a.page_box;
      const int ps_mask = (1 << p.page_log2) - 1;
      if (bx == kTile) {
        if (lane == 0) {
          const int pg = page_at(m.tok0);
          const int in_page = m.tok0 & ps_mask;
          mbar_arrive_expect_tx(&bars->full[st], 2 * kKVBytes);
          tma_load_4d_hint(ks, &tm_k, 0, in_page, m.kvh, pg, &bars->full[st], pol);
          tma_load_4d_hint(ks + kHalf, &tm_k, 64, in_page, m.kvh, pg, &bars->full[st], pol);
          tma_load_4d_hint(vs, &tm_v, 0, in_page, m.kvh, pg, &bars->full[st], pol);
          tma_load_4d_hint(vs + kHalf, &tm_v, 64, in_page, m.kvh, pg, &bars->full[st], pol);
        }
      } else {
        const int lg = p.page_log2;
        const int pieces = min(kTile >> lg, (m.tok_end - m.tok0 + bx - 1) >> lg);
        if (lane == 0) mbar_arrive_expect_tx(&bars->full[st], (uint32_t)pieces * 4u * (uint32_t)bx * 128u);
        __syncwarp();
        const int i = lane >> 2;  // page piece
        if (i < pieces) {
          const int idx = (m.tok0 >> lg) - pg0 + i;
          const int pg = idx < kPageCache ? pcache[idx]
                                          : page_uncached(bt_row, m.tok0 + (i << lg), lg, p.num_pages, p.status);
          const int off = (i << lg) * 128 + ((lane & 1) ? kHalf : 0);
          const CUtensorMap* tm = (lane & 2) ? &tm_v : &tm_k;
          tma_load_4d_hint(((lane & 2) ? vs : ks) + off, tm, (lane & 1) * 64, 0, m.kvh, pg, &bars->full[st], pol);
        }
      }
      ++n;
      if (lane == 0) bars->issued = n;
      return true;
    };
    bool ok = true;
    // The next ticket is taken while the current item streams, and a row's
    // length is loaded once for its consecutive kv heads.
    unsigned next = 0;
    if (lane == 0) next = atomicAdd(queue, 1u);
    int len_row = -1, len = 0;
    while (true) {
      const unsigned item = __shfl_sync(kFull, next, 0);
      Meta m{};
      if (item >= a.n_items) {
        if (lane == 0) {
          m.kind = kEntryEnd;
          (void)push(m, false);
        }
        break;
      }
      if (lane == 0) next = atomicAdd(queue, 1u);
      const int split = (int)(item / (unsigned)per_split);
      const int rem = (int)(item - (unsigned)split * (unsigned)per_split);
      const int b = rem / p.n_kv_heads;
      const int kvh = rem - b * p.n_kv_heads;
      const int seq = b / p.rows_per_seq;
      if (b != len_row) {
        int l = 0;
        if (lane == 0) l = row_len(p, seq, b - seq * p.rows_per_seq);
        len = __shfl_sync(kFull, l, 0);
        len_row = b;
      }
      const int tok_begin = split == 0 ? 0 : c0 + (split - 1) * p.chunk;
      m.row = b;
      m.kvh = kvh;
      m.split = split;
      if (len == 0) {
        // no visible key: split 0 writes the zero output (the RTL normaliser maps l == 0 to 0)
        if (split != 0) continue;
        m.kind = kEntryZero;
        if (lane == 0) ok = push(m, false);
        if (!__shfl_sync(kFull, ok, 0)) break;
        continue;
      }
      if (tok_begin >= len) continue;
      const int ntok = min(len - tok_begin, split == 0 ? c0 : p.chunk);
      m.kind = kEntryTile;
      m.tok_end = tok_begin + ntok;
      m.nsplit_b = len <= c0 ? 1 : 1 + (len - c0 + p.chunk - 1) / p.chunk;
      m.seq_kv = a.kv_shared ? 0 : seq;
      if constexpr (kPaged) {
        bt_row = p.block_table + (long long)seq * p.pages_per_seq;
        pg0 = tok_begin >> p.page_log2;
        const int np = min(kPageCache, ((m.tok_end - 1) >> p.page_log2) - pg0 + 1);
        // four entries per lane in flight at a time, then checked and stored
        for (int i0 = 0; i0 < np; i0 += 128) {
          int v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + 32 * u + lane;
            v[u] = i < np ? __ldg(bt_row + pg0 + i) : 0;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + 32 * u + lane;
            if (i < np) {
              int pg = v[u];
              if (pg < 0 || pg >= p.num_pages) {
                atomicOr(p.status, kDevBadPage);
                pg = 0;  // keep every copy in bounds
              }
              pcache[i] = pg;
            }
          }
        }
        __syncwarp();
      }
      if (lane == 0) {
        // the item's query heads (rows past the group are never used)
        const int qs = qi & 1;
        if (qi >= 2 && !wait_or_abort(&bars->q_free[qs], ((qi - 2) >> 1) & 1, abort)) {
          ok = false;
        } else {
          uint8_t* qd = smem + kQOff + qs * kOpBytes;
          mbar_arrive_expect_tx(&bars->q_full[qs], q_bytes);
          tma_load_3d(qd, &tm_q, 0, kvh * G, b, &bars->q_full[qs]);
          tma_load_3d(qd + kOpBytes / 2, &tm_q, 64, kvh * G, b, &bars->q_full[qs]);
          m.qslot = qs;
          m.qpar = (qi >> 1) & 1;
          bars->q_issued = ++qi;
          if constexpr (!kPaged) {
            const int ntiles = (ntok + kTile - 1) / kTile;
            for (int j = 0; ok && j < ntiles; ++j) {
              m.tok0 = tok_begin + j * kTile;
              m.flags = (j == 0 ? 1 : 0) | (j == ntiles - 1 ? 2 : 0);
              ok = push(m, true);
            }
          }
        }
      }
      if constexpr (kPaged) {
        ok = __shfl_sync(kFull, ok, 0);
        m.qslot = __shfl_sync(kFull, m.qslot, 0);
        m.qpar = __shfl_sync(kFull, m.qpar, 0);
        const int ntiles = (ntok + kTile - 1) / kTile;
        for (int j = 0; ok && j < ntiles; ++j) {
          m.tok0 = tok_begin + j * kTile;
          m.flags = (j == 0 ? 1 : 0) | (j == ntiles - 1 ? 2 : 0);
          ok = push_tile_warp(m);
        }
      }
      // lane 0 is done with this item's cache entries
      if (!__shfl_sync(kFull, ok, 0)) break;
    }
  } else if (warp == kMmaWarp) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kTile, kN, 0, 0);
      const uint32_t id_pv = idesc_bf16(kD, kN, 0, 1);
      auto issue_s = [&](int n, const Meta& m) -> bool {
        const int slot = n & 1;
        if (m.kind != kEntryTile) {
          mbar_arrive(&bars->s_full[slot]);
          return true;
        }
        if ((m.flags & 1) && !wait_or_abort(&bars->q_full[m.qslot], m.qpar, abort)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_addr(smem + kKOff + (n % kStages) * kKVBytes);
        const uint32_t q_base = smem_addr(smem + kQOff + m.qslot * kOpBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ka = k_base + (kk >> 2) * kHalf + (kk & 3) * 32;
          const uint32_t qa = q_base + (kk >> 2) * (kOpBytes / 2) + (kk & 3) * 32;
          mma_ss(tmem + slot * kN, desc_sw128(ka, 16, 1024), desc_sw128(qa, 16, 1024), id_s, kk > 0);
        }
        mma_commit(&bars->s_full[slot]);
        if (m.flags & 2) mma_commit(&bars->q_free[m.qslot]);
        return true;
      };
      int n = 0;
      Meta cur{};
      bool ok = wait_or_abort(&bars->full[0], 0, abort);
      if (ok) {
        cur = metas[0];
        ok = issue_s(0, cur);
      }
      while (ok) {
        const bool more = cur.kind != kEntryEnd;
        Meta nxt{};
        if (more) {
          const int s1 = (n + 1) % kStages;
          if (!wait_or_abort(&bars->full[s1], ((n + 1) / kStages) & 1, abort)) break;
          nxt = metas[s1];
          if (!issue_s(n + 1, nxt)) break;
        }
        const int slot = n & 1;
        const int st = n % kStages;
        if (!wait_or_abort(&bars->p_full[slot], (n >> 1) & 1, abort)) break;
        tc_fence_after();
        if (cur.kind == kEntryTile) {
          const uint32_t v_base = smem_addr(smem + kVOff + st * kKVBytes);
          const uint32_t ph = smem_addr(smem + kPOff + slot * 2 * kOpBytes);
#pragma unroll
          for (int part = 0; part < 2; ++part) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t va = v_base + kk * 16 * 128;
              const uint32_t pa = ph + part * kOpBytes + (kk >> 2) * (kOpBytes / 2) + (kk & 3) * 32;
              mma_ss(tmem + 32 + slot * kN, desc_sw128(va, kHalf, 1024), desc_sw128(pa, 16, 1024), id_pv,
                     (part | kk) > 0);
            }
          }
          mma_commit(&bars->o_full[slot]);
          mma_commit(&bars->empty[st]);
        } else {
          mbar_arrive(&bars->o_full[slot]);
          mbar_arrive(&bars->empty[st]);
        }
        if (!more) break;
        cur = nxt;
        ++n;
      }
      mma_commit(&bars->drain);
      (void)mbar_wait_bounded(&bars->drain, 0);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------- softmax
    const int t = threadIdx.x;  // token of a tile (S^T lane) and head dim (O^T lane)
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    float* xmax = reinterpret_cast<float*>(smem + kXOff);  // [2][4][16]
    const bool partial_out = p.out_acc != nullptr;
    uint32_t sync_phase = 0;
    int xpar = 0;
    float m_run[G], l_part[G], o_acc[G], alpha_prev[G], alpha_cur[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_part[g] = 0.f;
      o_acc[g] = 0.f;
      alpha_prev[g] = 1.f;
      alpha_cur[g] = 1.f;
    }
    // P^T element (head g, token t) in the 128-byte-swizzled K-major layout
    const int p_off = (t >> 6) * (kOpBytes / 2) + (t & 7) * 2;
    const int p_chunk = (t & 63) >> 3;

    auto accumulate = [&](int n) -> bool {  // o_acc = o_acc * alpha + O^T(n)
      if (!__all_sync(kFull, wait_or_abort(&bars->o_full[n & 1], (n >> 1) & 1, abort))) return false;
      tc_fence_after();
      float ov[NC];
      if constexpr (NC == 8) tmem_ld8(lane_base + 32 + (n & 1) * kN, ov);
      else tmem_ld16(lane_base + 32 + (n & 1) * kN, ov);
      tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < G; ++g) o_acc[g] = fmaf(o_acc[g], alpha_prev[g], ov[g]);
      tc_fence_before();
      return true;
    };

    // An item's end: its O^T goes to the hand-off buffer in TMEM, the row
    // maxima and each warp's row-sum share to shared memory, and the
    // epilogue warps take it from there.
    Hand* hand = reinterpret_cast<Hand*>(smem + kHandOff);
    int hn = 0;  // items handed off
    auto handoff = [&](const Meta& m, int kind) -> bool {
      const int hs = hn & 1;
      if (hn >= 2 && !__all_sync(kFull, wait_or_abort(&bars->epi_free[hs], ((hn - 2) >> 1) & 1, abort)))
        return false;
      tc_fence_after();
      Hand& h = hand[hs];
      if (kind == kEntryTile) {
        uint32_t w[16];
#pragma unroll
        for (int g = 0; g < 16; ++g) w[g] = g < G ? __float_as_uint(o_acc[g]) : 0u;
        tmem_st16(lane_base + kHandCol + hs * 16, w);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float v = l_part[g];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
          if (lane == 0) h.l[warp][g] = v;
        }
        if (t == 0) {
          h.row = m.row;
          h.kvh = m.kvh;
          h.split = m.split;
          h.nsplit_b = m.nsplit_b;
#pragma unroll
          for (int g = 0; g < G; ++g) h.m[g] = m_run[g];
        }
        tmem_wait_st();
      }
      if (t == 0) h.kind = kind;
      tc_fence_before();
      mbar_arrive(&bars->epi_full[hs]);
      ++hn;
      return true;
    };

    auto softmax_tile = [&](int n, const Meta& m) -> bool {
      const int slot = n & 1;
      float sv[NC];
      if constexpr (NC == 8) tmem_ld8(lane_base + slot * kN, sv);
      else tmem_ld16(lane_base + slot * kN, sv);
      tmem_wait_ld();
      const bool valid = m.tok0 + t < m.tok_end;
      float* xb = xmax + xpar * 64;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sv[g] = valid ? sv[g] * p.scale_log2 : -INFINITY;
        const float wm = warp_max(sv[g]);
        if (lane == 0) xb[warp * 16 + g] = wm;
      }
      if (!valid) {
        // keys past the item's end carry p = 0; zero their V rows so stale
        // cache contents (NaN, Inf) cannot reach the P.V sum
        uint4* v0 = reinterpret_cast<uint4*>(smem + kVOff + (n % kStages) * kKVBytes + t * 128);
        uint4* v1 = reinterpret_cast<uint4*>(smem + kVOff + (n % kStages) * kKVBytes + kHalf + t * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v0[i] = make_uint4(0, 0, 0, 0);
          v1[i] = make_uint4(0, 0, 0, 0);
        }
      }
      if (!group_sync(&bars->sync, sync_phase, abort)) return false;
      uint8_t* ph = smem + kPOff + slot * 2 * kOpBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tmax = fmaxf(fmaxf(xb[g], xb[16 + g]), fmaxf(xb[32 + g], xb[48 + g]));
        const float m_new = fmaxf(m_run[g], tmax);
        alpha_cur[g] = (m_new == m_run[g]) ? 1.f : ex2_ftz(m_run[g] - m_new);
        m_run[g] = m_new;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float pr = ex2_ftz(sv[g] - m_use);
        l_part[g] = fmaf(l_part[g], alpha_cur[g], pr);
        // pr - bf16(pr) is exact in fp32; its bf16 rounding carries the next 8 bits
        const __nv_bfloat16 hb = __float2bfloat16_rn(pr);
        const __nv_bfloat16 lb = __float2bfloat16_rn(pr - __bfloat162float(hb));
        const int off = p_off + g * 128 + ((p_chunk ^ (g & 7)) << 4);
        *reinterpret_cast<__nv_bfloat16*>(ph + off) = hb;
        *reinterpret_cast<__nv_bfloat16*>(ph + kOpBytes + off) = lb;
      }
      xpar ^= 1;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_full[slot]);
      return true;
    };

    bool pending = false;  // O^T of the previous entry (a tile) not yet added
    bool ended = false;
    Meta item{};
    for (int n = 0;; ++n) {
      const int st = n % kStages;
      if (!__all_sync(kFull, wait_or_abort(&bars->full[st], (n / kStages) & 1, abort))) break;
      const Meta m = metas[st];
      const bool cont = m.kind == kEntryTile && !(m.flags & 1);
      if (pending && !cont) {
        // the previous item ended with tile n-1: finish it first
        if (!accumulate(n - 1) || !handoff(item, kEntryTile)) break;
        pending = false;
      }
      if (m.kind == kEntryTile && (m.flags & 1)) {
        item = m;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          m_run[g] = -INFINITY;
          l_part[g] = 0.f;
          o_acc[g] = 0.f;
        }
      }
      if (!__all_sync(kFull, wait_or_abort(&bars->s_full[n & 1], (n >> 1) & 1, abort))) break;
      tc_fence_after();
      if (m.kind == kEntryTile) {
        if (!softmax_tile(n, m)) break;
      } else {
        tc_fence_before();
        mbar_arrive(&bars->p_full[n & 1]);
      }
      if (pending && !accumulate(n - 1)) break;
      if (m.kind == kEntryTile) {
        pending = true;
#pragma unroll
        for (int g = 0; g < G; ++g) alpha_prev[g] = alpha_cur[g];
      } else if (m.kind == kEntryZero) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int h = m.kvh * G + g;
          const long long row = (long long)m.row * p.n_q_heads + h;
          if (partial_out) {
            p.out_acc[row * kD + t] = 0.f;
            if (t == 0) { p.out_ml[row * 2] = -INFINITY; p.out_ml[row * 2 + 1] = 0.f; }
          } else {
            p.o[m.row * p.o_sb + h * p.o_sh + t] = 0;
          }
        }
      } else {
        ended = true;  // end of work
        break;
      }
    }
    if (ended) (void)handoff(item, kEntryEnd);
  } else {
    // ------------------------------------------------------------ epilogue
    // Thread te owns head dim te (its TMEM lane) of every handed-off item.
    const int te = (warp & 3) * 32 + lane;
    const uint32_t e_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const Hand* hand = reinterpret_cast<const Hand*>(smem + kHandOff);
    const bool partial_out = p.out_acc != nullptr;
    uint32_t esync_phase = 0;
    for (int hn = 0;; ++hn) {
      const int hs = hn & 1;
      if (!__all_sync(kFull, wait_or_abort(&bars->epi_full[hs], (hn >> 1) & 1, abort))) break;
      tc_fence_after();
      const Hand& h = hand[hs];
      if (h.kind != kEntryTile) break;
      float ov[16];
      tmem_ld16(e_base + kHandCol + hs * 16, ov);
      const int b = h.row, kvh = h.kvh, split = h.split, nsplit_b = h.nsplit_b;
      float M[G], L[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        M[g] = h.m[g];
        L[g] = (h.l[0][g] + h.l[1][g]) + (h.l[2][g] + h.l[3][g]);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars->epi_free[hs]);  // the buffer may take the next item's result
      if (nsplit_b == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int hq = kvh * G + g;
          const long long row = (long long)b * p.n_q_heads + hq;
          if (partial_out) {
            p.out_acc[row * kD + te] = ov[g];
            if (te == 0) { p.out_ml[row * 2] = M[g]; p.out_ml[row * 2 + 1] = L[g]; }
          } else {
            const float inv = (L[g] > 0.f) ? 1.f / L[g] : 0.f;
            p.o[b * p.o_sb + hq * p.o_sh + te] = (uint16_t)f32_to_bf16_rne_bits(ov[g] * inv);
          }
        }
        continue;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const long long slot = ((long long)b * p.n_q_heads + kvh * G + g) * p.nsplit + split;
        p.part_acc[slot * kD + te] = ov[g];
        if (te == 0) { p.part_ml[slot * 2] = M[g]; p.part_ml[slot * 2 + 1] = L[g]; }
      }
      __threadfence();
      if (!group_sync(&bars->esync, esync_phase, abort)) break;
      if (te == 0) {
        int* ctr = p.counters + b * p.n_kv_heads + kvh;
        const int prev = atomicAdd(ctr, 1);
        const int last = (prev == nsplit_b - 1);
        if (last) *ctr = 0;  // every other split has arrived: reset for the next launch
        bars->last_split = last;
      }
      if (!group_sync(&bars->esync, esync_phase, abort)) break;
      // (thread 0 writes the next item's flag only after all 128 threads have
      // met again, so each reads this one first)
      if (*reinterpret_cast<volatile int*>(&bars->last_split)) {
        __threadfence();
        merge_splits_tc<G>(p, b, kvh, nsplit_b, partial_out, warp & 3, lane);
      }
    }
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(p.status, kDevWaitTimeout);
    if (threadIdx.x == kTmaWarp * 32) {
      // let this CTA's own copies land before its shared memory is released
      const int issued = bars->issued;
      for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
        (void)mbar_wait_bounded(&bars->full[j % kStages], (j / kStages) & 1);
      const int qn = bars->q_issued;
      for (int j = (qn > 2 ? qn - 2 : 0); j < qn; ++j) (void)mbar_wait_bounded(&bars->q_full[j & 1], (j >> 1) & 1);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (threadIdx.x == 0) {
    // the last CTA to finish resets the work queue for the next launch
    __threadfence();
    if (atomicAdd(queue + 1, 1u) == gridDim.x - 1) {
      queue[0] = 0;
      queue[1] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

enum class DecodePath { kAuto, kSimt, kTensor };

DecodePath path_override() {
  const char* e = std::getenv("LARA_DECODE_PATH");
  if (!e) return DecodePath::kAuto;
  if (std::strcmp(e, "simt") == 0) return DecodePath::kSimt;
  if (std::strcmp(e, "tc") == 0) return DecodePath::kTensor;
  return DecodePath::kAuto;
}

// Groups at or above this size run on the tensor cores by default: below 8
// query heads per KV head the CUDA-core kernel streams at the HBM rate with P
// kept in fp32 (config 2 under sustained load on B200: 0.955 of the copy
// peak at 1762 MHz; this kernel, forced with LARA_DECODE_PATH=tc, 0.981 at
// 1965 MHz, with the split-P representation error of its P.V).
constexpr int kAutoMinGroup = 8;

template <bool kPaged>
const void* kernel_for_layout(int group) {
  switch (group) {
    case 1: return reinterpret_cast<const void*>(&gqa_decode_tc_kernel<1, kPaged>);
    case 2: return reinterpret_cast<const void*>(&gqa_decode_tc_kernel<2, kPaged>);
    case 4: return reinterpret_cast<const void*>(&gqa_decode_tc_kernel<4, kPaged>);
    case 8: return reinterpret_cast<const void*>(&gqa_decode_tc_kernel<8, kPaged>);
    case 16: return reinterpret_cast<const void*>(&gqa_decode_tc_kernel<16, kPaged>);
    default: return nullptr;
  }
}

const void* kernel_for(int group, bool paged = false) {
  return paged ? kernel_for_layout<true>(group) : kernel_for_layout<false>(group);
}

bool stride_ok(long long elems) { return elems > 0 && (elems * 2) % 16 == 0 && elems * 2 < (1ll << 40); }

}  // namespace

bool decode_tc_selected(int head_dim, int group) {
  const DecodePath path = path_override();
  if (path == DecodePath::kSimt) return false;
  if (head_dim != kD || kernel_for(group) == nullptr || !tensor_maps_available()) return false;
  return path == DecodePath::kTensor || group >= kAutoMinGroup;
}

void decode_tc_plan(int batch, int n_kv_heads, int max_tokens, const int32_t* lens_host, int* nsplit_out,
                    int* chunk_out) {
  // Items are dispensed in ticket order (split-major) to whichever CTA (one
  // per SM) is free, so the plan simulates that list schedule for each
  // candidate and keeps the one whose last CTA finishes first.  An item
  // costs its tiles plus about one tile of stream time at its boundary
  // (B200 sweeps of configs 2 and 3: 1-3 us per item, one tile ~1.6 us).
  // Candidates: chunks of 2^k tiles with equal splits, and with a longer
  // split 0 (the plan's splits then cover less than max_tokens and split 0
  // takes the rest, decode_first_chunk): every row's first item is dispensed
  // before any short one, so long items start first and the short ones even
  // out the finish times, as a longest-first list schedule does.
  constexpr double kItemOverhead = 1.0;
  constexpr long long kMaxItems = 1 << 18;  // candidates with more items are not simulated
  const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
  const int L = max_tokens < 1 ? 1 : max_tokens;
  const int max_tiles = (L + kTile - 1) / kTile;
  std::vector<int> len(batch);
  for (int b = 0; b < batch; ++b)
    len[b] = lens_host ? (lens_host[b] < 0 ? 0 : (lens_host[b] > L ? L : lens_host[b])) : L;
  double best = 1e300;
  int best_chunk = max_tiles * kTile, best_s = 1;
  std::vector<double> heap;
  auto simulate = [&](long long c0, long long c, int ns) {
    heap.assign((size_t)sms, 0.0);  // min-heap of CTA finish times
    auto take = [&](double cost) {
      std::pop_heap(heap.begin(), heap.end(), std::greater<double>());
      heap.back() += cost;
      std::push_heap(heap.begin(), heap.end(), std::greater<double>());
    };
    for (int sp = 0; sp < ns; ++sp)
      for (int b = 0; b < batch; ++b) {
        const long long begin = sp == 0 ? 0 : c0 + (long long)(sp - 1) * c;
        if (len[b] == 0 && sp == 0) {
          for (int h = 0; h < n_kv_heads; ++h) take(kItemOverhead);
          continue;
        }
        if (begin >= len[b]) continue;
        const long long ntok = std::min<long long>(sp == 0 ? c0 : c, len[b] - begin);
        const double cost = (double)((ntok + kTile - 1) / kTile) + kItemOverhead;
        for (int h = 0; h < n_kv_heads; ++h) take(cost);
      }
    return *std::max_element(heap.begin(), heap.end());
  };
  auto consider = [&](int c, int ns) {
    const long long c0 = (long long)ns * c >= L ? c : ((L - (long long)(ns - 1) * c + kTile - 1) / kTile) * kTile;
    long long items = 0;
    for (int b = 0; b < batch; ++b) items += len[b] <= c0 ? 1 : 1 + (len[b] - c0 + c - 1) / c;
    if (items * n_kv_heads > kMaxItems) return;
    const double makespan = simulate(c0, c, ns);
    if (makespan < best * (1.0 - 1e-9)) {
      best = makespan;
      best_chunk = c;
      best_s = ns;
    }
  };
  // equal splits: chunks of 2^k tiles
  std::vector<int> chunks;
  for (long long chunk = kTile;; chunk *= 2) {
    if (chunk > (long long)max_tiles * kTile) chunk = (long long)max_tiles * kTile;
    chunks.push_back((int)chunk);
    consider((int)chunk, (L + (int)chunk - 1) / (int)chunk);
    if (chunk >= (long long)max_tiles * kTile) break;
  }
  // a longer split 0, for the best equal-split chunk, a quarter and half of
  // it, and twice it: split counts whose split 0 is about 1.5^j chunks long
  const int best_equal = best_chunk;
  for (const int c : chunks) {
    if (c != best_equal && c * 2 != best_equal && c * 4 != best_equal && c != best_equal * 2) continue;
    int last = (L + c - 1) / c;
    for (double m = 1.5; m * c < L; m *= 1.5) {
      const int ns = 1 + (int)((L - (long long)(m * c)) / c);
      if (ns >= 1 && ns < last) {
        consider(c, ns);
        last = ns;
      }
    }
  }
  *nsplit_out = best_s;
  *chunk_out = best_chunk;
}

cudaError_t decode_tc_launch(const DecodeParams& p, cudaStream_t stream) {
  const int group = p.n_kv_heads > 0 ? p.n_q_heads / p.n_kv_heads : 0;
  const bool paged = p.block_table != nullptr;
  const void* fn = kernel_for(group, paged);
  if (!fn || p.head_dim != kD) return cudaErrorNotSupported;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!al16(p.q) || !al16(p.k) || !al16(p.v) || !stride_ok(p.q_sh)) return cudaErrorNotSupported;
  if (p.batch > 1 && !stride_ok(p.q_sb)) return cudaErrorNotSupported;
  const bool kv_shared = !paged && p.kv_sb == 0;
  const long long nseq_kv = kv_shared ? 1 : (p.batch + p.rows_per_seq - 1) / p.rows_per_seq;
  if (!paged && !stride_ok(p.kv_sh)) return cudaErrorNotSupported;
  if (!paged && !kv_shared && nseq_kv > 1 && !stride_ok(p.kv_sb)) return cudaErrorNotSupported;
  // a paged tile is whole pieces of pages: splits start on 128-token boundaries
  if (paged && (p.chunk % kTile != 0 || p.chunk0 % kTile != 0 || p.page_log2 < 4)) return cudaErrorNotSupported;
  if (p.chunk <= 0 || p.nsplit <= 0 || p.chunk0 < 0 || p.rows_per_seq < 1) return cudaErrorInvalidValue;
  const long long c0 = p.chunk0 > 0 ? p.chunk0 : p.chunk;
  if (c0 + (long long)(p.nsplit - 1) * p.chunk < (long long)p.max_seq_len) return cudaErrorInvalidValue;
  const long long n_items = (long long)p.nsplit * p.batch * p.n_kv_heads;
  if (n_items >= (1ll << 31)) return cudaErrorInvalidValue;

  const int q_rows = p.n_q_heads < kN ? p.n_q_heads : kN;
  CUtensorMap mq, mk, mv;
  // Q: (d, head, row) with element strides (1, q_sh, q_sb)
  const cuuint64_t qd[3] = {(cuuint64_t)kD, (cuuint64_t)p.n_q_heads, (cuuint64_t)p.batch};
  const cuuint64_t qs[2] = {(cuuint64_t)p.q_sh * 2,
                            (cuuint64_t)(p.batch > 1 ? p.q_sb : p.q_sh * p.n_q_heads) * 2};
  const cuuint32_t qbox[3] = {64, (cuuint32_t)q_rows, 1};
  // K/V: (d, token, kv head, sequence) with element strides (1, D, kv_sh, kv_sb),
  // or for a paged cache (d, row in page, kv head, page) over the page pool
  const long long ps = paged ? (1ll << p.page_log2) : 0;
  const int page_box = paged ? (int)(ps < kTile ? ps : kTile) : 0;
  const cuuint64_t kd[4] = {(cuuint64_t)kD, (cuuint64_t)(paged ? ps : p.max_seq_len), (cuuint64_t)p.n_kv_heads,
                            (cuuint64_t)(paged ? p.num_pages : nseq_kv)};
  const cuuint64_t ks[3] = {
      (cuuint64_t)kD * 2, (cuuint64_t)(paged ? ps * kD : p.kv_sh) * 2,
      (cuuint64_t)(paged ? ps * kD * p.n_kv_heads : (nseq_kv > 1 ? p.kv_sb : p.kv_sh * p.n_kv_heads)) * 2};
  const cuuint32_t kbox[4] = {64, (cuuint32_t)(paged ? page_box : kTile), 1, 1};
  if (!make_tensor_map_bf16(&mq, p.q, 3, qd, qs, qbox) || !make_tensor_map_bf16(&mk, p.k, 4, kd, ks, kbox) ||
      !make_tensor_map_bf16(&mv, p.v, 4, kd, ks, kbox))
    return cudaErrorNotSupported;
  {
    // the shared-memory opt-in is per (kernel, device): set it once
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (!done.count({fn, dev})) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
      if (e != cudaSuccess) return e;
      done.insert({fn, dev});
    }
  }
  TcDecodeArgs a{};
  a.n_items = (unsigned)n_items;
  a.kv_shared = kv_shared ? 1 : 0;
  a.q_rows = q_rows;
  a.page_box = page_box;
  const int sms = device_sm_count();
  const unsigned grid = (unsigned)(n_items < sms ? n_items : sms);
  void* args[] = {&mq, &mk, &mv, const_cast<DecodeParams*>(&p), &a};
  return launch_with_pdl(fn, dim3(grid), dim3(kThreads), args, kSmemAlloc, stream);
}

}  // namespace lara
