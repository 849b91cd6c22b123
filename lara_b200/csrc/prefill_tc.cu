// Chunked prefill / dense attention on the 5th-generation tensor cores
// (tcgen05 + TMEM, sm_100a).
//
// One CTA computes 128 query rows of one query head of one sequence against
// the visible prefix of its KV cache ("cache + self" with the causal rule
// kv_pos <= q_pos of sw/board_performance.py:174-177), FlashAttention-style:
//
//   warp 5 (TMA)     : Q tile once, then K_j / V_j tiles of 128 keys into a
//                      2-stage ring (tensor-map copies with 128-byte swizzle,
//                      no multicast), mbarrier transaction counts.
//   warp 4 (MMA)     : one thread issues tcgen05.mma:
//                        S_j = Q . K_j^T   (A, B from shared memory, fp32 in TMEM,
//                                           double-buffered S so S_{j+1} overlaps
//                                           the softmax of S_j)
//                        O  += P_j . V_j   (A = P_j read from TMEM, B = V_j MN-major)
//                      and tcgen05.commit to mbarriers.
//   warps 0-7        : two threads per query row (TMEM lane), one per half of
//                      the 128 columns: load S_j, scale,
//                      causal/length mask, online softmax in log2 domain (fp32
//                      running max and sum; the pair exchanges row maxima
//                      through shared memory), P_j -> bf16 (round to nearest
//                      even) written back into the S buffer for the P.V MMA,
//                      rescale of the O accumulator in TMEM when the
//                      reference max moved, and the epilogue O / l -> bf16.
//
// KV tiles beyond the last key visible to any row of the tile are never
// loaded (the causal tile skip of hw/rtl/core/attn_core.sv:138-153); the
// diagonal tile is masked per element.  Every wait is bounded by
// %globaltimer; on a timeout the CTA flags the status word, drains its own
// tensor-core work and TMA copies (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "lara_internal.h"
#include "tcgen05.cuh"

namespace lara {

using namespace tc;

namespace {

constexpr int kTileM = 128;        // query rows per CTA (TMEM lanes)
constexpr int kTileN = 128;        // keys per KV tile
constexpr int kHead = 128;         // head_dim
constexpr int kHalfBytes = 128 * 128;  // one [128 rows x 64 bf16] swizzled half tile
constexpr int kTileBytes = 2 * kHalfBytes;  // [128 x 128] bf16 as two halves
constexpr int kStages = 2;
constexpr int kSoftmaxWarps = 8;   // two per TMEM lane quarter: each owns 64 of a row's 128 columns
constexpr int kMmaWarp = kSoftmaxWarps;
constexpr int kTmaWarp = kSoftmaxWarps + 1;
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
// The reference max used for exponentiation only moves when a row's max grows
// by more than this (log2 units), so O is rarely rescaled; p stays <= 2^8.
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kTmemCols = 512;  // S0 [0,128) S1 [128,256) O [256,384)

// shared memory map (offsets from a 1024-aligned base)
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kTileBytes;                 // K stages
constexpr int kVOff = kKOff + kStages * kTileBytes;       // V stages
constexpr int kBarOff = kVOff + kStages * kTileBytes;
constexpr int kRedOff = kBarOff + 256;                    // row-max / row-sum exchange [2][2][128] floats
constexpr int kSmemUsed = kRedOff + 2 * 2 * kTileM * 4;
constexpr int kSmemAlloc = kSmemUsed + 1024;  // + alignment slack

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int issued;  // KV tiles whose TMA copies were issued
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct TcArgs {
  int n_q;            // query rows per sequence
  int n_q_heads, n_kv_heads;
  uint16_t* o;
  long long o_sb, o_sr, o_sh;  // output strides (elements): sequence, row, head
  // Sequence b has kv_len = base + kv_add keys; query row i sees keys
  // j <= base + q_add + i (causal) -- base = base_lens[b] or 0.
  const int32_t* base_lens;
  int kv_add, q_add;
  int causal;
  int kv_rows;             // Lmax: rows per (sequence, kv head) in the K/V tensor map
  float scale_log2;
  int* status;
};

// kSplitP: P = P_hi + P_lo (two bf16 terms, ~16 significant bits) and two
// P.V MMA sets, so the result carries fp32-class P precision; without it P is
// one bf16 (the usual FlashAttention choice).
template <bool kSplitP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kBarOff);
  volatile int* abort = &bars->abort;

  const int h = blockIdx.x;
  const int qt = blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / (a.n_q_heads / a.n_kv_heads);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = qt * kTileM;

  // visible keys of this tile: rows q0 .. q_last see keys [0, min(kv_len, q_off + row + 1))
  const int base = a.base_lens ? a.base_lens[b] : 0;
  int kv_len = base + a.kv_add;
  kv_len = kv_len < 0 ? 0 : (kv_len > a.kv_rows ? a.kv_rows : kv_len);
  const int q_off = base + a.q_add;
  const int q_last = min(a.n_q, q0 + kTileM) - 1;
  long long kmax = (long long)kv_len - 1;
  if (a.causal) kmax = min(kmax, (long long)q_off + q_last);
  const int ntiles = kmax >= 0 ? (int)(kmax / kTileN) + 1 : 0;

  if (ntiles == 0) {
    // no row of this tile sees any key: zero output (l == 0 -> 0)
    if (threadIdx.x < kTileM) {
      const int r = q0 + threadIdx.x;
      if (r < a.n_q) {
        uint16_t* dst = a.o + b * a.o_sb + (long long)r * a.o_sr + (long long)h * a.o_sh;
        for (int d = 0; d < kHead; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  uint8_t* q_smem = smem + kQOff;
  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->s_full[0], 1);
    mbar_init(&bars->s_full[1], 1);
    mbar_init(&bars->p_full, kSoftmaxWarps * 32);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->issued = 0;
    mbar_fence_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tm_o = tmem + 256;

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->q_full, kTileBytes);
      tma_load_4d(q_smem, &tm_q, 0, h, q0, b, &bars->q_full);
      tma_load_4d(q_smem + kHalfBytes, &tm_q, 64, h, q0, b, &bars->q_full);
      const int zrow = b * a.n_kv_heads + kvh;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kStages;
        if (j >= kStages && !wait_or_abort(&bars->kv_empty[st], ((j / kStages) - 1) & 1, abort)) break;
        uint8_t* ks = smem + kKOff + st * kTileBytes;
        uint8_t* vs = smem + kVOff + st * kTileBytes;
        mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kTileBytes);
        tma_load_3d(ks, &tm_k, 0, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(ks + kHalfBytes, &tm_k, 64, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(vs, &tm_v, 0, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(vs + kHalfBytes, &tm_v, 64, j * kTileN, zrow, &bars->kv_full[st]);
        bars->issued = j + 1;
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kTileM, kTileN, 0);
      const uint32_t id_pv = idesc_bf16(kTileM, kTileN, 1);
      const uint32_t q_base = smem_addr(q_smem);
      bool ok = wait_or_abort(&bars->q_full, 0, abort);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int st = j % kStages;
          const int sb = j & 1;
          if (!wait_or_abort(&bars->kv_full[st], (j / kStages) & 1, abort)) break;
          tc_fence_after();
          const uint32_t k_base = smem_addr(smem + kKOff + st * kTileBytes);
          // S_j = Q . K_j^T over head_dim in 8 steps of 16
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
            mma_ss(tmem + sb * 128, desc_sw128(q_base + off, 16, 1024), desc_sw128(k_base + off, 16, 1024), id_s,
                   kk > 0);
          }
          mma_commit(&bars->s_full[sb]);
        }
        if (j >= 1) {
          // O += P_{j-1} . V_{j-1} once the softmax has written P and rescaled O
          const int jp = j - 1;
          if (!wait_or_abort(&bars->p_full, jp & 1, abort)) break;
          tc_fence_after();
          const int st = jp % kStages;
          const uint32_t v_base = smem_addr(smem + kVOff + st * kTileBytes);
          const uint32_t p_tmem = tmem + (jp & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(tm_o, p_tmem + kk * 8, desc_sw128(v_base + kk * 16 * 128, kHalfBytes, 1024), id_pv,
                   (jp > 0 || kk > 0) ? 1u : 0u);
          if constexpr (kSplitP) {
            // low-order part of P, stored in columns 64..127 of the S buffer
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_ts(tm_o, p_tmem + 64 + kk * 8, desc_sw128(v_base + kk * 16 * 128, kHalfBytes, 1024), id_pv, 1u);
          }
          mma_commit(&bars->o_full);
          mma_commit(&bars->kv_empty[st]);
        }
      }
      // drain: every tcgen05 op this thread issued is complete once `drain` fires
      mma_commit(&bars->drain);
      (void)mbar_wait_bounded(&bars->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;           // TMEM lane quarter
    const int ch = warp >> 2;               // column half of S (and of O)
    const int r = quarter * 32 + lane;      // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int q_row = q0 + r;
    const long long vis_row = a.causal ? min((long long)kv_len, (long long)q_off + q_row + 1) : (long long)kv_len;
    // every row of the tile sees keys [0, vis_min): tiles below it need no mask
    const long long vis_min = a.causal ? min((long long)kv_len, (long long)q_off + q0 + 1) : (long long)kv_len;
    float* red = reinterpret_cast<float*>(smem + kRedOff);  // [parity][half][row]
    const int pair_bar = 1 + quarter;
    float m_ref = -INFINITY, l_part = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      // every lane returns from the bounded wait; the vote keeps the warp's
      // decision uniform before any warp-collective tcgen05 instruction
      if (!__all_sync(0xffffffffu, wait_or_abort(&bars->s_full[sb], (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[64];
      tmem_ld32(tmem + lane_off + sb * 128 + ch * 64, sv);
      tmem_ld32(tmem + lane_off + sb * 128 + ch * 64 + 32, sv + 32);
      tmem_wait_ld();
      if ((long long)(j + 1) * kTileN > vis_min) {
        const long long vis = vis_row - (long long)j * kTileN - ch * 64;  // visible columns of this half
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= vis) sv[c] = -INFINITY;
      }
      float mx = sv[0];
#pragma unroll
      for (int c = 1; c < 64; ++c) mx = fmaxf(mx, sv[c]);
      float* rbuf = red + (j & 1) * 2 * kTileM;
      rbuf[ch * kTileM + r] = mx;
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      mx = fmaxf(rbuf[r], rbuf[kTileM + r]);
      const float m_tile = mx * a.scale_log2;  // scale > 0 keeps the order
      const bool move = m_tile > m_ref + kRescaleThreshold || (m_ref == -INFINITY && m_tile != -INFINITY);
      const float m_new = move ? m_tile : m_ref;
      const float corr = move ? exp2f(m_ref - m_new) : 1.f;
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      float sum = 0.f;
      uint32_t pw[32];
      uint32_t lw[kSplitP ? 32 : 1];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = exp2f(fmaf(sv[c], a.scale_log2, -m_use));
        const float p1 = exp2f(fmaf(sv[c + 1], a.scale_log2, -m_use));
        sum += p0 + p1;
        const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
        pw[c / 2] = *reinterpret_cast<const uint32_t*>(&pb);
        if constexpr (kSplitP) {
          // p - bf16(p) is exact in fp32; its bf16 rounding carries the next 8 bits
          const float2 hi = __bfloat1622float2(pb);
          const __nv_bfloat162 lb = __floats2bfloat162_rn(p0 - hi.x, p1 - hi.y);
          lw[c / 2] = *reinterpret_cast<const uint32_t*>(&lb);
        }
      }
      l_part = l_part * corr + sum;
      // P_j (bf16 pairs along keys): high part in columns [0,64), low part in [64,128)
      tmem_st32(tmem + lane_off + sb * 128 + ch * 32, pw);
      if constexpr (kSplitP) tmem_st32(tmem + lane_off + sb * 128 + 64 + ch * 32, lw);
      tmem_wait_st();
      if (j >= 1) {
        // O holds sum_{i<j} P_i V_i at the old reference max once PV_{j-1} is done
        if (!__all_sync(0xffffffffu, wait_or_abort(&bars->o_full, (j - 1) & 1, abort))) {
          ok = false;
          break;
        }
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            float ov[32];
            tmem_ld32(tm_o + lane_off + ch * 64 + c, ov);
            tmem_wait_ld();
            uint32_t ow[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) ow[i] = __float_as_uint(ov[i] * corr);
            tmem_st32(tm_o + lane_off + ch * 64 + c, ow);
          }
          tmem_wait_st();
        }
      }
      m_ref = m_new;
      tc_fence_before();
      mbar_arrive(&bars->p_full);
    }
    // epilogue: O / l -> bf16 (l = sum of the two halves' partial sums)
    if (ok && __all_sync(0xffffffffu, wait_or_abort(&bars->o_full, (ntiles - 1) & 1, abort))) {
      tc_fence_after();
      float* lbuf = red + (ntiles & 1) * 2 * kTileM;
      lbuf[ch * kTileM + r] = l_part;
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      const float l_tot = lbuf[r] + lbuf[kTileM + r];
      const float inv = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
      uint16_t* dst = a.o + b * a.o_sb + (long long)q_row * a.o_sr + (long long)h * a.o_sh + ch * 64;
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        float ov[32];
        tmem_ld32(tm_o + lane_off + ch * 64 + c, ov);
        tmem_wait_ld();
        if (q_row < a.n_q) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack2_bf16(ov[i] * inv, ov[i + 1] * inv);
            w.y = pack2_bf16(ov[i + 2] * inv, ov[i + 3] * inv);
            w.z = pack2_bf16(ov[i + 4] * inv, ov[i + 5] * inv);
            w.w = pack2_bf16(ov[i + 6] * inv, ov[i + 7] * inv);
            *reinterpret_cast<uint4*>(dst + c + i) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(a.status, kDevWaitTimeout);
    // copies issued by the TMA warp must land before the CTA retires
    if (threadIdx.x == kTmaWarp * 32) {
      (void)mbar_wait_bounded(&bars->q_full, 0);
      const int issued = bars->issued;
      for (int t = (issued > kStages ? issued - kStages : 0); t < issued; ++t)
        (void)mbar_wait_bounded(&bars->kv_full[t % kStages], (t / kStages) & 1);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host: tensor maps
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

namespace {
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

bool make_tensor_map_bf16(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                          const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tensor_maps_available() { return encode_fn() != nullptr; }

bool prefill_tc_supported(int head_dim, int n_q_heads, int n_kv_heads) {
  return head_dim == kHead && n_kv_heads > 0 && n_q_heads % n_kv_heads == 0 && tensor_maps_available();
}

cudaError_t prefill_tc_launch(const PrefillTcParams& p, cudaStream_t stream) {
  if (!prefill_tc_supported(p.head_dim, p.n_q_heads, p.n_kv_heads) || p.batch < 1 || p.n_q < 1 ||
      p.batch > 65535 || p.kv_rows < 1)
    return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv;
  // Q: (d, head, row, sequence) with element strides (1, q_sh, q_sr, q_sb)
  const cuuint64_t qd[4] = {(cuuint64_t)kHead, (cuuint64_t)p.n_q_heads, (cuuint64_t)p.n_q, (cuuint64_t)p.batch};
  const cuuint64_t qs[3] = {(cuuint64_t)p.q_sh * 2, (cuuint64_t)p.q_sr * 2, (cuuint64_t)p.q_sb * 2};
  const cuuint32_t qbox[4] = {64, 1, (cuuint32_t)kTileM, 1};
  // K/V: (d, token, sequence * kv_head) over a [B][Hkv][Lmax][D] cache
  const cuuint64_t kd[3] = {(cuuint64_t)kHead, (cuuint64_t)p.kv_rows, (cuuint64_t)p.batch * p.n_kv_heads};
  const cuuint64_t ks[2] = {(cuuint64_t)kHead * 2, (cuuint64_t)p.kv_rows * kHead * 2};
  const cuuint32_t kbox[3] = {64, (cuuint32_t)kTileN, 1};
  if (!make_tensor_map_bf16(&mq, p.q, 4, qd, qs, qbox) || !make_tensor_map_bf16(&mk, p.k, 3, kd, ks, kbox) ||
      !make_tensor_map_bf16(&mv, p.v, 3, kd, ks, kbox))
    return cudaErrorInvalidValue;
  TcArgs a{};
  a.n_q = p.n_q;
  a.n_q_heads = p.n_q_heads;
  a.n_kv_heads = p.n_kv_heads;
  a.o = p.o;
  a.o_sb = p.o_sb;
  a.o_sr = p.o_sr;
  a.o_sh = p.o_sh;
  a.base_lens = p.base_lens;
  a.kv_add = p.kv_add;
  a.q_add = p.q_add;
  a.causal = p.causal;
  a.kv_rows = p.kv_rows;
  a.scale_log2 = p.scale_log2;
  a.status = p.status;
  dim3 grid(p.n_q_heads, (p.n_q + kTileM - 1) / kTileM, p.batch);
  if (p.split_p) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemAlloc);
    if (e != cudaSuccess) return e;
    prefill_tc_kernel<true><<<grid, kThreads, kSmemAlloc, stream>>>(mq, mk, mv, a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemAlloc);
    if (e != cudaSuccess) return e;
    prefill_tc_kernel<false><<<grid, kThreads, kSmemAlloc, stream>>>(mq, mk, mv, a);
  }
  return cudaGetLastError();
}

}  // namespace lara
