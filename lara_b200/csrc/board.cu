// Board-arithmetic ("fidelity") attention: the bf16 words LARA's FPGA
// datapath produces, bit for bit.
//
// The default kernels compute with IEEE fp32 and a true exp.  The FPGA
// instead runs its own fp32 adder/multiplier, a 1024-entry exp table with
// linear interpolation, P truncated to bf16 before P.V, the O correction
// applied per 16-token block, and a 256-entry reciprocal table for the final
// normalisation.  Board test cases carry the FPGA's output words
// (sw/board_matrix.py compares them bit for bit), so this mode reproduces
// that arithmetic and its order of operations:
//
//   fp32_add / fp32_mul / bf16_mul_to_fp32   hw/rtl/pkg/attn_pkg.sv:404-597
//   exp lookup                               hw/rtl/core/softmax_engine.sv:501-705
//   softmax block update                     hw/rtl/core/softmax_engine.sv:858-1312
//   Phase A (scores) / Phase B (P.V)         hw/rtl/core/attn_tile.sv:156-329,
//                                            hw/rtl/attn_top.sv:640-700,822-825
//   O accumulate, normalise, bf16 output     hw/rtl/mem/output_buffer.sv:199-286,885
//   tile schedule + causal tile limit        hw/rtl/core/attn_core.sv:107-154
//
// Arithmetic.  On normal operands whose result is normal, the RTL's adder and
// multiplier round to nearest even exactly as IEEE-754 does (their 56-bit
// aligned sum with sticky bit, and the 48-bit product with guard/round/sticky,
// are correctly rounded), and a bf16 x bf16 product is exact.  Each primitive
// therefore issues the hardware fadd.rn / fmul.rn and keeps that result when
// the operands and the result are normal; every other case (zeros, denormals,
// infinities, NaN, exponent overflow or underflow, where the RTL's 8-bit
// exponent arithmetic wraps) takes a bit-level restatement of the RTL
// function.  The library is built without flush-to-zero, so the hardware
// results are the IEEE ones.
//
// Schedule.  One CTA per (32-row Q tile, query head), 256 threads.  For every
// 16-token block of the KV tiles the causal limit admits (the RTL processes
// exactly these), the block's K/V rows are staged in shared memory; each
// thread forms two score dot products (sequential over the 128 dims from a
// cleared accumulator), one warp carries the per-row max / correction / row
// sum recurrences, and each thread owns 16 output columns of one row for P.V
// and the O update.  Rows are independent in the RTL, so running all 32 rows
// of a Q tile together reproduces its two 16-row micro tiles.
#include <cstdint>

#include "../../include/lara_b200.h"
#include "lara_internal.h"

namespace {

#include "board_luts.inc"

constexpr int kD = 128;
constexpr int kTileQ = 32;    // attn_pkg.sv:191
constexpr int kTileKv = 64;   // attn_pkg.sv:192
constexpr int kBlock = 16;    // TILE_COLS / TILE_ROWS
constexpr int kThreads = 256;
constexpr int kRowStride = kD + 2;  // halves; 65 words, so 16 rows start in 16 different banks
constexpr uint32_t kNegInf = 0xFF800000u, kOne = 0x3F800000u, kNegEight = 0xC1000000u, kQNaN = 0x7FC00000u;
constexpr uint32_t kInvSqrtD = 0x3DB504F3u;  // attn_pkg.sv:241

__device__ uint32_t g_exp_lut[1024];
__device__ uint32_t g_recip_lut[256];

__device__ __forceinline__ bool is_zero(uint32_t a) { return (a & 0x7FFFFFFFu) == 0; }
__device__ __forceinline__ uint32_t expo(uint32_t a) { return (a >> 23) & 0xFFu; }
__device__ __forceinline__ bool normal(uint32_t a) { return expo(a) - 1u < 254u; }

// --- bit-level restatements of the RTL functions (slow paths) -------------

__device__ __noinline__ uint32_t add_rtl(uint32_t a, uint32_t b) {
  const uint64_t M56 = (1ull << 56) - 1;
  const bool a_nan = expo(a) == 0xFF && (a & 0x7FFFFFu), b_nan = expo(b) == 0xFF && (b & 0x7FFFFFu);
  if (a_nan || b_nan) return kQNaN;
  if (is_zero(a)) return b;
  if (is_zero(b)) return a;
  const uint32_t sa = a >> 31, sb = b >> 31;
  const uint32_t ea = expo(a) ? expo(a) : 1u, eb = expo(b) ? expo(b) : 1u;
  const uint32_t ma = (expo(a) ? 0x800000u : 0u) | (a & 0x7FFFFFu);
  const uint32_t mb = (expo(b) ? 0x800000u : 0u) | (b & 0x7FFFFFu);
  const bool a_larger = ea > eb || (ea == eb && ma >= mb);
  const uint32_t e_large = a_larger ? ea : eb, s_large = a_larger ? sa : sb;
  const uint64_t large_ext = uint64_t(a_larger ? ma : mb) << 32, small_ext = uint64_t(a_larger ? mb : ma) << 32;
  const int shift = int(a_larger ? ea - eb : eb - ea);
  const uint64_t sticky_mask = shift <= 0 ? 0ull : (shift >= 56 ? M56 : (M56 >> (56 - shift)));
  const uint64_t sticky = (small_ext & sticky_mask) ? 1ull : 0ull;
  const uint64_t small_sh = shift >= 56 ? sticky : ((small_ext >> shift) | sticky);
  const uint64_t sum = ((sa ^ sb) ? large_ext - small_sh : large_ext + small_sh) & ((1ull << 57) - 1);
  if (sum == 0) return 0u;
  uint32_t e_res;
  uint64_t norm;
  if ((sum >> 56) & 1) {
    e_res = (e_large + 1u) & 0xFFu;
    norm = (sum >> 1) | (sum & 1);
  } else {
    // leading zeros of bits [55:32], counted within 8-bit groups, at most 24
    const uint32_t top = uint32_t(sum >> 32) & 0xFFFFFFu;
    const int lz = top ? __clz(top) - 8 : 24;
    norm = (sum << lz) & M56;
    e_res = (e_large - uint32_t(lz)) & 0xFFu;
  }
  const uint32_t keep = uint32_t(norm >> 32) & 0xFFFFFFu;
  const bool guard = (norm >> 31) & 1, round = (norm >> 30) & 1, st = (norm & ((1ull << 30) - 1)) != 0;
  const uint32_t mr = keep + ((guard && (round || st || (keep & 1))) ? 1u : 0u);
  uint32_t frac = mr & 0x7FFFFFu;
  if ((mr >> 24) & 1) {
    e_res = (e_res + 1u) & 0xFFu;
    frac = 0;
  }
  return (s_large << 31) | (e_res << 23) | frac;
}

__device__ __noinline__ uint32_t mul_rtl(uint32_t a, uint32_t b) {
  const bool a_nan = expo(a) == 0xFF && (a & 0x7FFFFFu), b_nan = expo(b) == 0xFF && (b & 0x7FFFFFu);
  if (a_nan || b_nan) return kQNaN;
  if (is_zero(a) || is_zero(b)) return (a ^ b) & 0x80000000u;
  const bool a_inf = expo(a) == 0xFF, b_inf = expo(b) == 0xFF;  // NaN handled above
  if (a_inf || b_inf) return ((a ^ b) & 0x80000000u) | 0x7F800000u;
  const uint64_t p = uint64_t(0x800000u | (a & 0x7FFFFFu)) * uint64_t(0x800000u | (b & 0x7FFFFFu));
  const bool hi = (p >> 47) & 1;
  uint32_t ep = (expo(a) + expo(b) - (hi ? 126u : 127u)) & 0xFFu;
  const int sh = hi ? 24 : 23;
  const uint32_t keep = 0x800000u | uint32_t((p >> sh) & 0x7FFFFFu);
  const bool guard = (p >> (sh - 1)) & 1, round = (p >> (sh - 2)) & 1;
  const bool st = (p & ((1ull << (sh - 2)) - 1)) != 0;
  uint32_t mr = keep + ((guard && (round || st || (keep & 1))) ? 1u : 0u);
  if ((mr >> 24) & 1) {
    ep = (ep + 1u) & 0xFFu;
    mr = 0x800000u;
  }
  return ((a ^ b) & 0x80000000u) | (ep << 23) | (mr & 0x7FFFFFu);
}

__device__ __noinline__ uint32_t bmul_rtl(uint32_t a, uint32_t b) {  // a, b: bf16 words
  const uint32_t ea = (a >> 7) & 0xFFu, eb = (b >> 7) & 0xFFu;
  const uint32_t p = (0x80u | (a & 0x7Fu)) * (0x80u | (b & 0x7Fu));
  const uint32_t sign = ((a ^ b) >> 15) & 1u;
  const uint32_t ep9 = (ea + eb - 127u) & 0x1FFu;
  const bool nrm = (p >> 15) & 1;
  const uint32_t en = nrm ? (((ep9 & 0xFFu) + 1u) & 0xFFu) : (ep9 & 0xFFu);
  const uint32_t mn = nrm ? ((p & 0x7FFFu) << 8) : ((p & 0x3FFFu) << 9);
  const bool a_zero = ea == 0, b_zero = eb == 0;
  const bool a_inf = ea == 0xFF && !(a & 0x7F), b_inf = eb == 0xFF && !(b & 0x7F);
  const bool a_nan = ea == 0xFF && (a & 0x7F), b_nan = eb == 0xFF && (b & 0x7F);
  if (a_nan || b_nan) return kQNaN;
  if ((a_inf && b_zero) || (a_zero && b_inf)) return kQNaN;
  if (a_inf || b_inf) return (sign << 31) | 0x7F800000u;
  if (a_zero || b_zero) return sign << 31;
  return (sign << 31) | (en << 23) | mn;
}

// --- primitives: hardware result where it provably equals the RTL's -------

__device__ __forceinline__ uint32_t fadd(uint32_t a, uint32_t b) {
  if (is_zero(a)) return b;
  if (is_zero(b)) return a;
  if (normal(a) && normal(b)) {
    const uint32_t r = __float_as_uint(__fadd_rn(__uint_as_float(a), __uint_as_float(b)));
    if (normal(r) || r == 0u) return r;  // exact cancellation gives +0 in both
  }
  return add_rtl(a, b);
}

__device__ __forceinline__ uint32_t fsub(uint32_t a, uint32_t b) { return fadd(a, b ^ 0x80000000u); }

__device__ __forceinline__ uint32_t fmul(uint32_t a, uint32_t b) {
  if (normal(a) && normal(b)) {
    const uint32_t r = __float_as_uint(__fmul_rn(__uint_as_float(a), __uint_as_float(b)));
    if (normal(r)) return r;
  }
  return mul_rtl(a, b);
}

// exact bf16 x bf16 product (attn_pkg.sv:546-597); a, b are bf16 words
__device__ __forceinline__ uint32_t bmul(uint32_t a, uint32_t b) {
  if (((a >> 7) & 0xFFu) - 1u < 254u && ((b >> 7) & 0xFFu) - 1u < 254u) {
    const uint32_t r = __float_as_uint(__fmul_rn(__uint_as_float(a << 16), __uint_as_float(b << 16)));
    if (normal(r)) return r;
  }
  return bmul_rtl(a, b);
}

// attn_pkg.sv:354-369
__device__ __forceinline__ bool fgt(uint32_t a, uint32_t b) {
  if (a == b) return false;
  if ((a >> 31) != (b >> 31)) return b >> 31;
  return (a >> 31) ? (a & 0x7FFFFFFFu) < (b & 0x7FFFFFFFu) : (a & 0x7FFFFFFFu) > (b & 0x7FFFFFFFu);
}
__device__ __forceinline__ uint32_t fmax_rtl(uint32_t a, uint32_t b) { return fgt(a, b) ? a : b; }

// softmax_engine.sv:570-705 (x already known to be in [-8, 0] or outside it)
__device__ __forceinline__ uint32_t exp_lookup(uint32_t x, const uint32_t* lut) {
  if (fgt(kNegEight, x)) return 0u;
  if (fgt(x, 0u)) return kOne;
  // Q8.23, truncated toward zero (softmax_engine.sv:524-545); |x| <= 8 here
  int64_t xq = 0;
  if (!is_zero(x)) {
    const int shift = int(expo(x)) - 127;
    const int64_t m = int64_t(0x800000u | (x & 0x7FFFFFu));
    xq = shift >= 0 ? (m << shift) : ((-shift) >= 63 ? 0 : (m >> (-shift)));
    if (x >> 31) xq = -xq;
  }
  int64_t n = xq + 67108864;
  n = n < 0 ? 0 : (n > 67108864 ? 67108864 : n);
  const int64_t num = (n << 10) - n;  // (x + 8) * 1023 in Q8.26
  const int idx = int(num >> 26);
  const int64_t rem = num - (int64_t(idx) << 26);
  if (idx >= 1023) return lut[1023];
  // Q26 remainder to fp32, truncating (softmax_engine.sv:547-567)
  uint32_t frac = 0;
  if (rem > 0) {
    const int bit = 63 - __clzll(rem);
    const int64_t residual = rem - (int64_t(1) << bit);
    const uint32_t mant = bit < 23 ? uint32_t(residual << (23 - bit)) : uint32_t(residual >> (bit - 23));
    frac = ((uint32_t(127 + bit - 26) & 0xFFu) << 23) | (mant & 0x7FFFFFu);
  }
  return fadd(lut[idx], fmul(fsub(lut[idx + 1], lut[idx]), frac));
}

// output_buffer.sv:199-224
__device__ __forceinline__ uint32_t recip_lut_bits(uint32_t v, const uint32_t* rlut) {
  const uint32_t e = expo(v), frac = v & 0x7FFFFFu, s = v & 0x80000000u;
  if (e == 0xFF && frac) return kQNaN;
  if (is_zero(v)) return s | 0x7F800000u;
  if (e == 0xFF) return s;
  if (frac == 0) return s | (((254u - e) & 0xFFu) << 23);
  return s | (((253u - e) & 0xFFu) << 23) | (rlut[frac >> 15] & 0x7FFFFFu);
}

// attn_pkg.sv:617-626
__device__ __forceinline__ uint32_t to_bf16(uint32_t a) {
  const uint32_t upper = a >> 16;
  return (upper + (((a >> 15) & 1u) && ((a & 0x7FFFu) || (upper & 1u)) ? 1u : 0u)) & 0xFFFFu;
}

struct BoardParams {
  const uint16_t* q;  // [Hq][L][128]
  const uint16_t* k;  // [Hkv][L][128]
  const uint16_t* v;
  uint16_t* o;
  int L, group, causal, q_pos_base, kv_pos_base;
};

__global__ void __launch_bounds__(kThreads) board_attention_kernel(const BoardParams p) {
  __shared__ uint32_t s_exp[1024];
  __shared__ uint32_t s_recip[256];
  __shared__ __align__(16) uint16_t s_q[kTileQ * kRowStride];
  __shared__ __align__(16) uint16_t s_k[kBlock * kRowStride];
  __shared__ __align__(16) uint16_t s_v[kBlock * kD];
  __shared__ uint32_t s_scaled[kTileQ][kBlock];  // scaled scores, then P (fp32 words)
  __shared__ uint8_t s_masked[kTileQ][kBlock];
  __shared__ uint32_t s_corr[kTileQ];
  __shared__ uint32_t s_mnew[kTileQ];

  const int tid = threadIdx.x, qt = blockIdx.x, h = blockIdx.y;
  const int L = p.L;
  const int n_kv_tiles = (L + kTileKv - 1) / kTileKv;
  const int active_q = min(kTileQ, L - qt * kTileQ);
  const int q_start = p.q_pos_base + qt * kTileQ;
  int limit = n_kv_tiles - 1;  // attn_core.sv:137-152
  if (p.causal) {
    const int q_end = q_start + active_q - 1;
    const int t = q_end >= p.kv_pos_base ? (q_end - p.kv_pos_base) >> 6 : 0;
    limit = min(limit, t);
  }
  const uint16_t* qh = p.q + (size_t(h) * L + size_t(qt) * kTileQ) * kD;
  const uint16_t* kh = p.k + size_t(h / p.group) * L * kD;
  const uint16_t* vh = p.v + size_t(h / p.group) * L * kD;

  for (int i = tid; i < 1024; i += kThreads) s_exp[i] = g_exp_lut[i];
  if (tid < 256) s_recip[tid] = g_recip_lut[tid];
  for (int i = tid; i < kTileQ * (kD / 2); i += kThreads) {
    const int r = i / (kD / 2), c = i % (kD / 2);
    const uint32_t w = r < active_q ? reinterpret_cast<const uint32_t*>(qh + size_t(r) * kD)[c] : 0u;
    reinterpret_cast<uint32_t*>(s_q + r * kRowStride)[c] = w;
  }

  // score ownership: row sr, columns sc0, sc0 + 1
  const int sr = tid >> 3, sc0 = (tid & 7) * 2;
  // P.V ownership: row pr, columns pd0 + 16 j + {0, 1}, j = 0..7
  const int pr = tid >> 3, pd0 = (tid & 7) * 2;
  uint32_t O[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) O[j] = 0u;
  uint32_t m_row = kNegInf, l_row = 0u;  // valid in warp 0, lane = row
  const int q_pos_s = q_start + sr;

  for (int kt = 0; kt <= limit; ++kt) {
    const int active_kv = min(kTileKv, L - kt * kTileKv);
    const int nsb = (active_kv + kBlock - 1) / kBlock;
    for (int sb = 0; sb < nsb; ++sb) {
      const bool first = kt == 0 && sb == 0;
      const int col0 = kt * kTileKv + sb * kBlock;
      const int cols = min(kBlock, active_kv - sb * kBlock);
      __syncthreads();  // previous block's readers are done with s_k / s_v / s_scaled
      for (int i = tid; i < kBlock * (kD / 2); i += kThreads) {
        const int r = i / (kD / 2), c = i % (kD / 2);
        const bool in = col0 + r < L;
        const uint32_t kw = in ? reinterpret_cast<const uint32_t*>(kh + size_t(col0 + r) * kD)[c] : 0u;
        const uint32_t vw = in ? reinterpret_cast<const uint32_t*>(vh + size_t(col0 + r) * kD)[c] : 0u;
        reinterpret_cast<uint32_t*>(s_k + r * kRowStride)[c] = kw;
        reinterpret_cast<uint32_t*>(s_v + r * kD)[c] = vw;
      }
      __syncthreads();

      // Phase A: scores, sequential over depth from a cleared accumulator
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = sc0 + cc;
        const bool masked = sr >= active_q || c >= cols || (p.causal && q_pos_s < p.kv_pos_base + col0 + c);
        uint32_t scaled = kNegInf;
        if (!masked) {
          const uint32_t* qrow = reinterpret_cast<const uint32_t*>(s_q + sr * kRowStride);
          const uint32_t* krow = reinterpret_cast<const uint32_t*>(s_k + c * kRowStride);
          uint32_t s = 0u;
#pragma unroll 4
          for (int d2 = 0; d2 < kD / 2; ++d2) {
            const uint32_t qw = qrow[d2], kw = krow[d2];
            s = fadd(s, bmul(qw & 0xFFFFu, kw & 0xFFFFu));
            s = fadd(s, bmul(qw >> 16, kw >> 16));
          }
          scaled = fmul(s, kInvSqrtD);
        }
        s_scaled[sr][c] = scaled;
        s_masked[sr][c] = masked;
      }
      __syncthreads();

      // row max, new running max and correction (softmax_engine.sv:858-1062)
      if (tid < kTileQ) {
        uint32_t row_max = kNegInf;
#pragma unroll
        for (int c = 0; c < kBlock; ++c) row_max = fmax_rtl(row_max, s_scaled[tid][c]);
        const uint32_t m_old = first ? kNegInf : m_row;
        const uint32_t m_new = fmax_rtl(m_old, row_max);
        s_mnew[tid] = m_new;
        s_corr[tid] = first ? 0u : exp_lookup(fsub(m_old, m_new), s_exp);
        m_row = m_new;
      }
      __syncthreads();
      // P = exp(scaled - m_new); masked keys give exactly 0 (softmax_engine.sv:1211-1234)
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint32_t sv = s_scaled[sr][sc0 + cc];
        s_scaled[sr][sc0 + cc] = s_masked[sr][sc0 + cc] ? 0u : exp_lookup(fsub(sv, s_mnew[sr]), s_exp);
      }
      __syncthreads();
      // left-to-right row sum and l update (softmax_engine.sv:1075-1312)
      if (tid < kTileQ) {
        uint32_t row_sum = 0u;
#pragma unroll
        for (int c = 0; c < kBlock; ++c) row_sum = fadd(row_sum, s_scaled[tid][c]);
        l_row = first ? row_sum : fadd(fmul(l_row, s_corr[tid]), row_sum);
      }
      // Phase B: P truncated to its top 16 bits, sequential over the 16 keys;
      // then O = add(mul(O, corr), dO) (output_buffer.sv:226-267)
      if (pr < active_q) {
        const uint32_t corr = s_corr[pr];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t d0 = 0u, d1 = 0u;
#pragma unroll 4
          for (int kk = 0; kk < kBlock; ++kk) {
            const uint32_t pw = s_scaled[pr][kk] >> 16;
            const uint32_t vw = reinterpret_cast<const uint32_t*>(s_v + kk * kD)[(pd0 + 16 * j) >> 1];
            d0 = fadd(d0, bmul(pw, vw & 0xFFFFu));
            d1 = fadd(d1, bmul(pw, vw >> 16));
          }
          O[2 * j] = fadd(fmul(O[2 * j], corr), d0);
          O[2 * j + 1] = fadd(fmul(O[2 * j + 1], corr), d1);
        }
      }
    }
  }

  __syncthreads();
  if (tid < kTileQ) s_corr[tid] = l_row;  // final l per row
  __syncthreads();
  if (pr < active_q) {
    const uint32_t l = s_corr[pr];
    const uint32_t r = recip_lut_bits(l, s_recip);
    uint16_t* orow = p.o + (size_t(h) * L + size_t(qt) * kTileQ + pr) * kD;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t a = is_zero(l) ? 0u : fmul(O[2 * j], r);
      const uint32_t b = is_zero(l) ? 0u : fmul(O[2 * j + 1], r);
      reinterpret_cast<uint32_t*>(orow)[(pd0 + 16 * j) >> 1] = to_bf16(a) | (to_bf16(b) << 16);
    }
  }
}

bool g_tables_ready[64] = {};

}  // namespace

extern "C" int lara_attention_dense_board(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                                          int n_q_heads, int n_kv_heads, int head_dim, int seq_len, int causal,
                                          int q_pos_base, int kv_pos_base, void* stream) {
  LARA_NVTX("lara_attention_dense_board");
  if (head_dim != kD)
    return lara::set_last_error(LARA_ERR_UNSUPPORTED, "board arithmetic is defined for head_dim 128 only");
  if (n_q_heads < 1 || n_kv_heads < 1 || n_q_heads % n_kv_heads || seq_len < 1)
    return lara::set_last_error(LARA_ERR_BAD_CFG, "bad board-arithmetic geometry");
  if (q_pos_base < 0 || kv_pos_base < 0 || q_pos_base + seq_len > 65536 || kv_pos_base + seq_len > 65536)
    return lara::set_last_error(LARA_ERR_BAD_CFG, "position base + seq_len exceeds the 16-bit position range");
  if (!q || !k || !v || !o || (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                               reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 3)
    return lara::set_last_error(LARA_ERR_STREAM_DEST, "null or misaligned buffer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return lara::set_last_error(LARA_ERR_CUDA, "cudaGetDevice failed");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!g_tables_ready[dev]) {
    if (cudaMemcpyToSymbolAsync(g_exp_lut, kBoardExpLut, sizeof(kBoardExpLut), 0, cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_recip_lut, kBoardRecipLut, sizeof(kBoardRecipLut), 0, cudaMemcpyHostToDevice,
                                st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return lara::set_last_error(LARA_ERR_CUDA, "uploading the board lookup tables failed");
    g_tables_ready[dev] = true;
  }
  BoardParams p{q, k, v, o, seq_len, n_q_heads / n_kv_heads, causal ? 1 : 0, q_pos_base, kv_pos_base};
  dim3 grid((seq_len + kTileQ - 1) / kTileQ, n_q_heads);
  board_attention_kernel<<<grid, kThreads, 0, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return lara::set_last_error(LARA_ERR_CUDA, std::string("board attention launch: ") + cudaGetErrorString(e));
  return LARA_OK;
}
