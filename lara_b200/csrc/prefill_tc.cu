// Chunked prefill / dense attention on the 5th-generation tensor cores
// (tcgen05 + TMEM, sm_100a).
//
// One CTA computes two tiles of 128 query rows (A: q0 .. q0+127, B: q0+128 ..
// q0+255) of one query head of one sequence against the visible prefix of its
// KV cache ("cache + self" with the causal rule kv_pos <= q_pos of
// sw/board_performance.py:174-177), FlashAttention-style, with the two tiles
// in ping-pong so the tensor core works on one while the other's softmax runs:
//
//   warp 9 (TMA)     : Q_A and Q_B once, then K_j / V_j tiles of 128 keys into
//                      a 2-stage ring (tensor-map copies with 128-byte
//                      swizzle, no multicast), mbarrier transaction counts.
//   warp 8 (MMA)     : one thread issues tcgen05.mma in the order
//                      PV_A(j), S_A(j+1), PV_B(j), S_B(j+1):
//                        S_t = Q_t . K^T   (A, B from shared memory, fp32 in TMEM)
//                        O_t += P_t . V    (A = P_t read from TMEM, B = V MN-major)
//                      and tcgen05.commit to mbarriers.  TMEM: S_A | S_B | O_A | O_B.
//   warps 0-7        : softmax of tile A, then tile B: two threads per query row
//                      (TMEM lane), 64 scores each: scale, causal/length mask,
//                      online softmax in log2 domain (fp32 running max and
//                      sum; the pair exchanges row maxima through shared
//                      memory), P -> bf16 (round to nearest even; by default split
//                      into P_hi + P_lo for ~16 significant bits) written back
//                      into the S columns for the P.V MMA, rescale of O_t in
//                      TMEM when the reference max moved, epilogue O_t / l -> bf16.
//
// KV tiles beyond the last key visible to any row of the CTA are never loaded
// (the causal tile skip of hw/rtl/core/attn_core.sv:138-153); the diagonal
// tiles are masked per element.  Every wait is bounded by %globaltimer; on a
// timeout the CTA flags the status word, drains its own tensor-core work and
// TMA copies (bounded), frees TMEM and returns.
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
// The reference max used for exponentiation only moves when a row's max grows
// by more than this (log2 units), so O is rarely rescaled; p stays <= 2^8.
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kTmemCols = 512;  // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)

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

// ---------------------------------------------------------------------------
// Two query tiles per CTA ("ping-pong"): rows q0 .. q0+127 (tile A) and
// q0+128 .. q0+255 (tile B) of one head share every K/V tile.  TMEM holds
// S_A | S_B | O_A | O_B (128 columns each).  The MMA thread interleaves the
// tiles -- PV_A(j), S_A(j+1), PV_B(j), S_B(j+1) -- so the tensor core works
// on one tile while the other tile's softmax runs.  Softmax: all 8 warps do
// tile A then tile B, two threads per query row (64 scores each).
// ---------------------------------------------------------------------------
constexpr int kPPStages = 2;
constexpr int kPPQOff = 0;                                  // Q_A, then Q_B
constexpr int kPPKOff = 2 * kTileBytes;
constexpr int kPPVOff = kPPKOff + kPPStages * kTileBytes;
constexpr int kPPBarOff = kPPVOff + kPPStages * kTileBytes;
constexpr int kPPRedOff = kPPBarOff + 256;                   // row max / sum exchange [2][<= 4][128] floats
constexpr int kPPSmemAlloc = kPPRedOff + 2 * 4 * kTileM * 4 + 1024;

// Warp roles for kRowThreads softmax threads per query row: 1 (warps 0-3 on
// tile A, 4-7 on tile B), 2 (8 warps, both tiles in turn) or 4 (16 warps);
// the MMA and TMA warps follow the softmax warps.
template <int kRowThreads>
struct PPLayout {
  static constexpr int kSoftmaxWarps = kRowThreads == 4 ? 16 : 8;
  static constexpr int kMmaWarp = kSoftmaxWarps;
  static constexpr int kTmaWarp = kSoftmaxWarps + 1;
  static constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
};

struct PPBars {
  uint64_t q_full;
  uint64_t kv_full[kPPStages];
  uint64_t kv_empty[kPPStages];
  uint64_t s_full[2];  // per tile
  uint64_t p_full[2];  // per tile: 256 softmax threads
  uint64_t o_full[2];  // per tile
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int issued;
};
static_assert(sizeof(PPBars) <= 256, "barrier block");

template <bool kSplitP, int kRowThreads>
__global__ void __launch_bounds__(PPLayout<kRowThreads>::kThreads, 1)
    prefill_pp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PPBars* bars = reinterpret_cast<PPBars*>(smem + kPPBarOff);
  volatile int* abort = &bars->abort;

  const int h = blockIdx.x;
  const int b = blockIdx.z;
  const int kvh = h / (a.n_q_heads / a.n_kv_heads);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.y * 2 * kTileM;

  const int base = a.base_lens ? a.base_lens[b] : 0;
  int kv_len = base + a.kv_add;
  kv_len = kv_len < 0 ? 0 : (kv_len > a.kv_rows ? a.kv_rows : kv_len);
  const int q_off = base + a.q_add;
  const int q_last = min(a.n_q, q0 + 2 * kTileM) - 1;
  long long kmax = (long long)kv_len - 1;
  if (a.causal) kmax = min(kmax, (long long)q_off + q_last);
  const int ntiles = kmax >= 0 ? (int)(kmax / kTileN) + 1 : 0;

  if (ntiles == 0) {
    if (threadIdx.x < 2 * kTileM) {
      const int r = q0 + threadIdx.x;
      if (r < a.n_q) {
        uint16_t* dst = a.o + b * a.o_sb + (long long)r * a.o_sr + (long long)h * a.o_sh;
        for (int d = 0; d < kHead; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kPPStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], kRowThreads > 1 ? PPLayout<kRowThreads>::kSoftmaxWarps * 32 : kTileM);
      mbar_init(&bars->o_full[t], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->issued = 0;
    mbar_fence_init();
  }
  if (warp == PPLayout<kRowThreads>::kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == PPLayout<kRowThreads>::kTmaWarp) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      uint8_t* q_smem = smem + kPPQOff;
      mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t) {
        tma_load_4d(q_smem + t * kTileBytes, &tm_q, 0, h, q0 + t * kTileM, b, &bars->q_full);
        tma_load_4d(q_smem + t * kTileBytes + kHalfBytes, &tm_q, 64, h, q0 + t * kTileM, b, &bars->q_full);
      }
      const int zrow = b * a.n_kv_heads + kvh;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kPPStages;
        if (j >= kPPStages && !wait_or_abort(&bars->kv_empty[st], ((j / kPPStages) - 1) & 1, abort)) break;
        uint8_t* ks = smem + kPPKOff + st * kTileBytes;
        uint8_t* vs = smem + kPPVOff + st * kTileBytes;
        mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kTileBytes);
        tma_load_3d(ks, &tm_k, 0, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(ks + kHalfBytes, &tm_k, 64, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(vs, &tm_v, 0, j * kTileN, zrow, &bars->kv_full[st]);
        tma_load_3d(vs + kHalfBytes, &tm_v, 64, j * kTileN, zrow, &bars->kv_full[st]);
        bars->issued = j + 1;
      }
    }
  } else if (warp == PPLayout<kRowThreads>::kMmaWarp) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kTileM, kTileN, 0);
      const uint32_t id_pv = idesc_bf16(kTileM, kTileN, 1);
      const uint32_t q_base = smem_addr(smem + kPPQOff);
      auto issue_s = [&](int t, int j) {
        const uint32_t k_base = smem_addr(smem + kPPKOff + (j % kPPStages) * kTileBytes);
        const uint32_t qb = q_base + t * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_ss(tmem + t * 128, desc_sw128(qb + off, 16, 1024), desc_sw128(k_base + off, 16, 1024), id_s, kk > 0);
        }
        mma_commit(&bars->s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_base = smem_addr(smem + kPPVOff + (j % kPPStages) * kTileBytes);
        const uint32_t p_tmem = tmem + t * 128;
        const uint32_t o_tmem = tmem + 256 + t * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ts(o_tmem, p_tmem + kk * 8, desc_sw128(v_base + kk * 16 * 128, kHalfBytes, 1024), id_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        if constexpr (kSplitP) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(o_tmem, p_tmem + 64 + kk * 8, desc_sw128(v_base + kk * 16 * 128, kHalfBytes, 1024), id_pv, 1u);
        }
        mma_commit(&bars->o_full[t]);
      };
      bool ok = wait_or_abort(&bars->q_full, 0, abort) && wait_or_abort(&bars->kv_full[0], 0, abort);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const bool more = j + 1 < ntiles;
        // tile A: PV_A(j), then S_A(j+1) (in-order issue keeps P_A(j) intact until PV_A(j) has read it)
        if (!wait_or_abort(&bars->p_full[0], j & 1, abort)) break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!wait_or_abort(&bars->kv_full[(j + 1) % kPPStages], ((j + 1) / kPPStages) & 1, abort)) break;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        // tile B
        if (!wait_or_abort(&bars->p_full[1], j & 1, abort)) break;
        tc_fence_after();
        issue_pv(1, j);
        mma_commit(&bars->kv_empty[j % kPPStages]);
        if (more) issue_s(1, j + 1);
      }
      mma_commit(&bars->drain);
      (void)mbar_wait_bounded(&bars->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax
    if constexpr (kRowThreads > 1) {
      // All softmax warps take tile A then tile B: kRowThreads threads per
      // query row (warps w, w + 4, ... share a TMEM lane quarter), each owning
      // CW of the 128 columns; they exchange row maxima (and, at the end, row
      // sums) through shared memory under a named barrier of the row group.
      constexpr int RT = kRowThreads;
      constexpr int CW = 128 / RT;         // columns per thread
      const int quarter = warp & 3;
      const int ch = warp >> 2;            // column slice
      const int r = quarter * 32 + lane;   // row within a tile
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const int pair_bar = 1 + quarter;
      const int bar_threads = 32 * RT;
      float* red = reinterpret_cast<float*>(smem + kPPRedOff);  // [parity][slice][row]
      // Per-tile state in scalars selected by the tile index: the tile loop
      // below is not unrolled, so one copy of its body serves both tiles and
      // the kernel's hot code stays small enough for the instruction cache.
      float m_ref0 = -INFINITY, m_ref1 = -INFINITY, l_part0 = 0.f, l_part1 = 0.f;
      const long long vis_row0 =
          a.causal ? min((long long)kv_len, (long long)q_off + q0 + r + 1) : (long long)kv_len;
      const long long vis_row1 =
          a.causal ? min((long long)kv_len, (long long)q_off + q0 + kTileM + r + 1) : (long long)kv_len;
      const long long vis_min0 = a.causal ? min((long long)kv_len, (long long)q_off + q0 + 1) : (long long)kv_len;
      const long long vis_min1 =
          a.causal ? min((long long)kv_len, (long long)q_off + q0 + kTileM + 1) : (long long)kv_len;
      bool ok = true;
      int step = 0;  // parity of the exchange buffer
      for (int j = 0; ok && j < ntiles; ++j) {
  #pragma unroll 1
        for (int t = 0; t < 2; ++t, ++step) {
          const float m_ref_t = t ? m_ref1 : m_ref0;
          const long long vis_row_t = t ? vis_row1 : vis_row0;
          const long long vis_min_t = t ? vis_min1 : vis_min0;
          const uint32_t s_tm = tmem + lane_off + t * 128;
          const uint32_t o_tm = tmem + lane_off + 256 + t * 128 + ch * CW;
          if (!__all_sync(0xffffffffu, wait_or_abort(&bars->s_full[t], j & 1, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
          float sv[CW];
  #pragma unroll
          for (int c = 0; c < CW; c += 32) tmem_ld32(s_tm + ch * CW + c, sv + c);
          tmem_wait_ld();
          if ((long long)(j + 1) * kTileN > vis_min_t) {
            const long long vis = vis_row_t - (long long)j * kTileN - ch * CW;  // visible columns of this slice
  #pragma unroll
            for (int c = 0; c < CW; ++c)
              if (c >= vis) sv[c] = -INFINITY;
          }
          // three-input max.f32 (sm_100): two new scores per instruction, 4 chains
          float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
  #pragma unroll
          for (int c = 4; c < CW; c += 2)
            asm("max.f32 %0, %0, %1, %2;" : "+f"(mx4[(c >> 1) & 3]) : "f"(sv[c]), "f"(sv[c + 1]));
          float* rbuf = red + (step & 1) * RT * kTileM;
          rbuf[ch * kTileM + r] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          asm volatile("bar.sync %0, %1;" ::"r"(pair_bar), "r"(bar_threads) : "memory");
          float mx = rbuf[r];
  #pragma unroll
          for (int c2 = 1; c2 < RT; ++c2) mx = fmaxf(mx, rbuf[c2 * kTileM + r]);
          const float m_tile = mx * a.scale_log2;  // scale > 0 keeps the order
          const bool move = m_tile > m_ref_t + kRescaleThreshold || (m_ref_t == -INFINITY && m_tile != -INFINITY);
          const float m_new = move ? m_tile : m_ref_t;
          const float corr = move ? ex2_ftz(m_ref_t - m_new) : 1.f;
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
          // packed fp32 pairs: scale-and-shift, sum and the split residual each
          // take one FFMA2 / FADD2 per two scores; exp2 is the MUFU instruction
          // (ex2.approx.ftz, relative error ~2^-22, far below the 2^-16 of split P)
          float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
          const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
          const float2 nm2 = make_float2(-m_use, -m_use);
  #pragma unroll
          for (int c = 0; c < CW; c += 32) {
            uint32_t pw[16];
            uint32_t lw[kSplitP ? 16 : 1];
  #pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float2 x = __ffma2_rn(make_float2(sv[c + i], sv[c + i + 1]), sc2, nm2);
              float2 pp;
              pp.x = ex2_ftz(x.x);
              pp.y = ex2_ftz(x.y);
              sum2[(i >> 1) & 1] = __fadd2_rn(sum2[(i >> 1) & 1], pp);
              const __nv_bfloat162 pb = __floats2bfloat162_rn(pp.x, pp.y);
              const uint32_t hw = *reinterpret_cast<const uint32_t*>(&pb);
              pw[i / 2] = hw;
              if constexpr (kSplitP) {
                // pp - bf16(pp) is exact in fp32; its bf16 rounding carries the next 8 bits
                const float2 hi = make_float2(__uint_as_float(hw << 16), __uint_as_float(hw & 0xFFFF0000u));
                const float2 d = __fadd2_rn(pp, make_float2(-hi.x, -hi.y));
                const __nv_bfloat162 lb = __floats2bfloat162_rn(d.x, d.y);
                lw[i / 2] = *reinterpret_cast<const uint32_t*>(&lb);
              }
            }
            // P as bf16 pairs along keys: high part in columns [0, 64), low part in [64, 128)
            tmem_st16(s_tm + ch * (CW / 2) + c / 2, pw);
            if constexpr (kSplitP) tmem_st16(s_tm + 64 + ch * (CW / 2) + c / 2, lw);
          }
          const float l_new = (t ? l_part1 : l_part0) * corr + ((sum2[0].x + sum2[0].y) + (sum2[1].x + sum2[1].y));
          if (t) l_part1 = l_new; else l_part0 = l_new;
          tmem_wait_st();
          if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
            // O_t must hold PV_t(j-1) before it is rescaled
            if (!__all_sync(0xffffffffu, wait_or_abort(&bars->o_full[t], (j - 1) & 1, abort))) {
              ok = false;
              break;
            }
            tc_fence_after();
  #pragma unroll
            for (int c = 0; c < CW; c += 32) {
              float ov[32];
              tmem_ld32(o_tm + c, ov);
              tmem_wait_ld();
              uint32_t ow[32];
  #pragma unroll
              for (int i = 0; i < 32; ++i) ow[i] = __float_as_uint(ov[i] * corr);
              tmem_st32(o_tm + c, ow);
            }
            tmem_wait_st();
          }
          if (t) m_ref1 = m_new; else m_ref0 = m_new;
          tc_fence_before();
          mbar_arrive(&bars->p_full[t]);
        }
      }
      // epilogue: O_t / l -> bf16 (l = the pair's two partial sums)
  #pragma unroll 1
      for (int t = 0; ok && t < 2; ++t, ++step) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&bars->o_full[t], (ntiles - 1) & 1, abort))) break;
        tc_fence_after();
        float* lbuf = red + (step & 1) * RT * kTileM;
        lbuf[ch * kTileM + r] = t ? l_part1 : l_part0;
        asm volatile("bar.sync %0, %1;" ::"r"(pair_bar), "r"(bar_threads) : "memory");
        float l_tot = lbuf[r];
  #pragma unroll
        for (int c2 = 1; c2 < RT; ++c2) l_tot += lbuf[c2 * kTileM + r];
        const float inv = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
        const int q_row = q0 + t * kTileM + r;
        const uint32_t o_tm = tmem + lane_off + 256 + t * 128 + ch * CW;
        uint16_t* dst = a.o + b * a.o_sb + (long long)q_row * a.o_sr + (long long)h * a.o_sh + ch * CW;
  #pragma unroll
        for (int c = 0; c < CW; c += 32) {
          float ov[32];
          tmem_ld32(o_tm + c, ov);
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
    } else {
      const int t = warp >> 2;             // query tile
      const int quarter = warp & 3;        // TMEM lane quarter
      const int r = quarter * 32 + lane;   // row within the tile
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const uint32_t s_tm = tmem + lane_off + t * 128;
      const uint32_t o_tm = tmem + lane_off + 256 + t * 128;
      const int q_row = q0 + t * kTileM + r;
      const long long vis_row = a.causal ? min((long long)kv_len, (long long)q_off + q_row + 1) : (long long)kv_len;
      const long long vis_min =
          a.causal ? min((long long)kv_len, (long long)q_off + q0 + t * kTileM + 1) : (long long)kv_len;
      float m_ref = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&bars->s_full[t], j & 1, abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[128];
  #pragma unroll
        for (int c = 0; c < 128; c += 32) tmem_ld32(s_tm + c, sv + c);
        tmem_wait_ld();
        if ((long long)(j + 1) * kTileN > vis_min) {
          const long long vis = vis_row - (long long)j * kTileN;
  #pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= vis) sv[c] = -INFINITY;
        }
        // eight independent max / sum chains instead of one 128-long chain
        // three-input max.f32 (sm_100): two new scores per instruction
        float mx8[8];
  #pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
  #pragma unroll
        for (int c = 8; c < 128; c += 2)
          asm("max.f32 %0, %0, %1, %2;" : "+f"(mx8[(c >> 1) & 7]) : "f"(sv[c]), "f"(sv[c + 1]));
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_tile = mx * a.scale_log2;
        const bool move = m_tile > m_ref + kRescaleThreshold || (m_ref == -INFINITY && m_tile != -INFINITY);
        const float m_new = move ? m_tile : m_ref;
        const float corr = move ? ex2_ftz(m_ref - m_new) : 1.f;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        // packed fp32 pairs: scale-and-shift, sum and the split residual each take
        // one FFMA2 / FADD2 per two scores; exp2 is the MUFU instruction
        // (ex2.approx.ftz, relative error ~2^-22, far below the 2^-16 of split P)
        float2 sum4[4];
  #pragma unroll
        for (int i = 0; i < 4; ++i) sum4[i] = make_float2(0.f, 0.f);
        const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
        const float2 nm2 = make_float2(-m_use, -m_use);
  #pragma unroll
        for (int c = 0; c < 128; c += 32) {
          uint32_t pw[16];
          uint32_t lw[kSplitP ? 16 : 1];
  #pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 x = __ffma2_rn(make_float2(sv[c + i], sv[c + i + 1]), sc2, nm2);
            float2 pp;
            pp.x = ex2_ftz(x.x);
            pp.y = ex2_ftz(x.y);
            sum4[(i >> 1) & 3] = __fadd2_rn(sum4[(i >> 1) & 3], pp);
            const __nv_bfloat162 pb = __floats2bfloat162_rn(pp.x, pp.y);
            const uint32_t hw = *reinterpret_cast<const uint32_t*>(&pb);
            pw[i / 2] = hw;
            if constexpr (kSplitP) {
              // pp - bf16(pp) is exact in fp32; its bf16 rounding carries the next 8 bits
              const float2 hi = make_float2(__uint_as_float(hw << 16), __uint_as_float(hw & 0xFFFF0000u));
              const float2 d = __fadd2_rn(pp, make_float2(-hi.x, -hi.y));
              const __nv_bfloat162 lb = __floats2bfloat162_rn(d.x, d.y);
              lw[i / 2] = *reinterpret_cast<const uint32_t*>(&lb);
            }
          }
          // P_j as bf16 pairs along keys: high part in columns [0, 64), low part in [64, 128)
          tmem_st16(s_tm + c / 2, pw);
          if constexpr (kSplitP) tmem_st16(s_tm + 64 + c / 2, lw);
        }
        const float sum = ((sum4[0].x + sum4[0].y) + (sum4[1].x + sum4[1].y)) +
                          ((sum4[2].x + sum4[2].y) + (sum4[3].x + sum4[3].y));
        l_run = l_run * corr + sum;
        tmem_wait_st();
        if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
          // O_t must hold PV_t(j-1) before it is rescaled
          if (!__all_sync(0xffffffffu, wait_or_abort(&bars->o_full[t], (j - 1) & 1, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
  #pragma unroll
          for (int c = 0; c < 128; c += 32) {
            float ov[32];
            tmem_ld32(o_tm + c, ov);
            tmem_wait_ld();
            uint32_t ow[32];
  #pragma unroll
            for (int i = 0; i < 32; ++i) ow[i] = __float_as_uint(ov[i] * corr);
            tmem_st32(o_tm + c, ow);
          }
          tmem_wait_st();
        }
        m_ref = m_new;
        tc_fence_before();
        mbar_arrive(&bars->p_full[t]);
      }
      // epilogue: O_t / l -> bf16
      if (ok && __all_sync(0xffffffffu, wait_or_abort(&bars->o_full[t], (ntiles - 1) & 1, abort))) {
        tc_fence_after();
        const float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
        uint16_t* dst = a.o + b * a.o_sb + (long long)q_row * a.o_sr + (long long)h * a.o_sh;
  #pragma unroll
        for (int c = 0; c < 128; c += 32) {
          float ov[32];
          tmem_ld32(o_tm + c, ov);
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
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(a.status, kDevWaitTimeout);
    if (threadIdx.x == PPLayout<kRowThreads>::kTmaWarp * 32) {
      (void)mbar_wait_bounded(&bars->q_full, 0);
      const int issued = bars->issued;
      for (int j = (issued > kPPStages ? issued - kPPStages : 0); j < issued; ++j)
        (void)mbar_wait_bounded(&bars->kv_full[j % kPPStages], (j / kPPStages) & 1);
    }
  }
  __syncthreads();
  if (warp == PPLayout<kRowThreads>::kMmaWarp) {
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
  dim3 grid2(p.n_q_heads, (p.n_q + 2 * kTileM - 1) / (2 * kTileM), p.batch);
  // split P: several softmax threads per row (one per row would spill); bf16 P:
  // one thread per row, warps 0-3 on tile A and 4-7 on tile B
  auto launch = [&](auto kernel, int threads) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPPSmemAlloc);
    if (e != cudaSuccess) return e;
    kernel<<<grid2, threads, kPPSmemAlloc, stream>>>(mq, mk, mv, a);
    return cudaSuccess;
  };
  cudaError_t e;
  if (p.split_p) {
    // two threads per row: four (16 softmax warps) measured 761 vs 773 TFLOP/s on config 5
    e = launch(prefill_pp_kernel<true, 2>, PPLayout<2>::kThreads);
  } else {
    e = launch(prefill_pp_kernel<false, 1>, PPLayout<1>::kThreads);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace lara
