// Layer prologue on the GPU: RMSNorm -> QKV projection -> RoPE -> head-major
// bf16 q/k/v, the host half of AttentionAccelerator.run_layer
// (sw/attn_driver.py:552-586), whose helper module (host_attention.py) the
// reference does not ship.  The contract restated here:
//
//   x_n   = rms_weight ? bf16(fp32(fp32(x * inv) * rms_weight)) : x with
//           inv = fp32(1 / sqrt(mean(x^2) + eps)) from an fp64 mean (the
//           y = x / sqrt(mean(x^2) + eps) * gamma of hw/rtl/ext/rms_norm/rms_norm.sv:7)
//   [q|k|v] = x_n @ W, W = [Wq | Wk | Wv] stored [hidden][Hq*D + 2*Hkv*D]
//           (the [IN_DIM][OUT_DIM] weight stream of
//           hw/rtl/ext/qkv_projection/qkv_projection.sv:8-10,32-35), fp32
//           accumulation
//   RoPE  on q (position q_pos_base + t) and k (kv_pos_base + t): dims
//         (2i, 2i+1) rotate by pos * theta_i, theta_i = base^(-2i/D)
//         (the dim-pair rotation of hw/rtl/core/rope_engine.sv:1-11; theta
//         table hw/data/rope_theta.hex for base 10000), fp32, exact sin/cos
//   out   bf16 (round to nearest even) q[Hq][L][D], k/v[Hkv][L][D]: the
//         run_attention layout.
//
// rmsnorm_kernel is HBM-bound (one CTA per token).  qkv_rope_kernel is a
// tcgen05 GEMM with the RoPE / bf16 / head-scatter epilogue fused: one CTA
// per 128 tokens x 128 output columns (one head of q, k or v, since D = 128),
// a 4-stage TMA ring of 64-wide K slices (A = x_n K-major, B = W MN-major,
// both 128-byte swizzled, no multicast), one thread issuing
// tcgen05.mma.cta_group::1.kind::f16 into a 128x128 fp32 TMEM accumulator,
// and 4 epilogue warps reading TMEM rows (one token per thread).  Every wait
// is bounded; on a timeout the CTA flags the status word, drains its copies
// and tensor-core work, frees TMEM and returns.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "../../include/lara_b200.h"
#include "common.cuh"
#include "lara_internal.h"
#include "tcgen05.cuh"

namespace lara {

using namespace tc;

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;       // 16 KB: [128 tokens][64] bf16, swizzled rows of 128 B
constexpr int kBChunk = kBK * 64 * 2;        // 8 KB: [64 k][64 n] bf16
constexpr int kBBytes = (kBN / 64) * kBChunk;  // [64 k][256 n] as four 64-column chunks
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kSmemAlloc = kBarOff + 256 + 1024;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kTmemCols = 2 * kBN;         // two accumulators: tile i uses columns (i & 1) * 256
constexpr int kHead = 128;

struct PBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int issued;  // K slices whose copies were issued
};
static_assert(sizeof(PBars) <= 256, "barrier block");

struct ProArgs {
  uint16_t* q;             // [batch][Hq][L][D]
  uint16_t* k;             // [batch][Hkv][L][D]
  uint16_t* v;
  int L, rows, nk;          // tokens per sequence, batch * L, K slices of 64
  int n_q_heads, n_kv_heads, n_cols;
  int m_tiles, n_tiles;
  const float2* rope_q;     // [D/2][L] (cos, sin) at position q_pos_base + t
  const float2* rope_k;     // [D/2][L] at kv_pos_base + t
  int* status;
};

struct RopeArgs {
  float2* rope_q;
  float2* rope_k;
  int L, q_pos_base, kv_pos_base;
  float theta[kHead / 2];
};

// Persistent: CTA c handles tiles c, c + grid, ...; tile t covers rows
// (t / n_tiles) * 128 and columns (t % n_tiles) * 256, so the CTAs resident at
// one time share a few A row tiles while W stays in L2.
__global__ void __launch_bounds__(kThreads, 1)
    qkv_rope_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ ProArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PBars* bars = reinterpret_cast<PBars*>(smem + kBarOff);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles_total = a.m_tiles * a.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], kEpiWarps * 32);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->issued = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles_total; t += gridDim.x) {
        const int m0 = (t / a.n_tiles) * kBM, n0 = (t % a.n_tiles) * kBN;
        for (int kb = 0; kb < a.nk; ++kb, ++g) {
          const int st = g % kStages;
          if (g >= kStages && !wait_or_abort(&bars->empty[st], ((g / kStages) - 1) & 1, abort)) {
            ok = false;
            break;
          }
          uint8_t* as = smem + st * kStageBytes;
          uint8_t* bs = as + kABytes;
          mbar_arrive_expect_tx(&bars->full[st], kStageBytes);
          tma_load_2d(as, &tm_a, kb * kBK, m0, &bars->full[st]);
#pragma unroll
          for (int c = 0; c < kBN / 64; ++c) tma_load_2d(bs + c * kBChunk, &tm_b, n0 + 64 * c, kb * kBK, &bars->full[st]);
          bars->issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kBM, kBN, 1);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles_total; t += gridDim.x, ++i) {
        const int ab = i & 1;
        if (i >= 2 && !wait_or_abort(&bars->acc_empty[ab], ((i >> 1) - 1) & 1, abort)) break;
        tc_fence_after();
        const uint32_t acc = tmem + ab * kBN;
        for (int kb = 0; kb < a.nk; ++kb, ++g) {
          const int st = g % kStages;
          if (!wait_or_abort(&bars->full[st], (g / kStages) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_addr(smem + st * kStageBytes);
          const uint32_t b_base = a_base + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_ss(acc, desc_sw128(a_base + kk * 32, 16, 1024), desc_sw128(b_base + kk * 16 * 128, kBChunk, 1024),
                   idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars->empty[st]);
        }
        if (ok) mma_commit(&bars->acc_full[ab]);
      }
      mma_commit(&bars->drain);
      (void)mbar_wait_bounded(&bars->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 (warps 2..5 -> quarters 2,3,0,1)
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int n_q_cols = a.n_q_heads * kHead, n_kv_cols = a.n_kv_heads * kHead;
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles_total; t += gridDim.x, ++i) {
      const int ab = i & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(&bars->acc_full[ab], (i >> 1) & 1, abort))) break;
      tc_fence_after();
      const int r = (t / a.n_tiles) * kBM + row;  // row of the [batch * L] token matrix
      const int n0 = (t % a.n_tiles) * kBN;
      const bool live = r < a.rows;
      const int rr = live ? r : a.rows - 1;
      const int b = rr / a.L, tok = rr % a.L;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        const int n = n0 + c;  // 32 columns inside one head (D = 128)
        if (n >= a.n_cols) break;  // ragged last column tile (TMA filled it with zeros)
        uint16_t* dst;
        const float2* rope = nullptr;
        if (n < n_q_cols) {
          dst = a.q + (((long long)b * a.n_q_heads + n / kHead) * a.L + tok) * kHead + (n % kHead);
          rope = a.rope_q;
        } else if (n < n_q_cols + n_kv_cols) {
          dst = a.k + (((long long)b * a.n_kv_heads + (n - n_q_cols) / kHead) * a.L + tok) * kHead + (n % kHead);
          rope = a.rope_k;
        } else {
          const int nv = n - n_q_cols - n_kv_cols;
          dst = a.v + (((long long)b * a.n_kv_heads + nv / kHead) * a.L + tok) * kHead + (nv % kHead);
        }
        float x[32];
        tmem_ld32(tmem + lane_off + ab * kBN + c, x);
        tmem_wait_ld();
        if (rope) {
          const int p0 = (n % kHead) >> 1;
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 cs = __ldg(rope + (long long)(p0 + (j >> 1)) * a.L + tok);  // lanes: consecutive tokens
            const float x0 = x[j], x1 = x[j + 1];
            x[j] = x0 * cs.x - x1 * cs.y;
            x[j + 1] = x0 * cs.y + x1 * cs.x;
          }
        }
        if (live) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 w;
            w.x = pack2_bf16(x[j], x[j + 1]);
            w.y = pack2_bf16(x[j + 2], x[j + 3]);
            w.z = pack2_bf16(x[j + 4], x[j + 5]);
            w.w = pack2_bf16(x[j + 6], x[j + 7]);
            *reinterpret_cast<uint4*>(dst + j) = w;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {
    if (threadIdx.x == 0) atomicOr(a.status, kDevWaitTimeout);
    if (threadIdx.x == 0) {
      const int issued = bars->issued;
      for (int g = (issued > kStages ? issued - kStages : 0); g < issued; ++g)
        (void)mbar_wait_bounded(&bars->full[g % kStages], (g / kStages) & 1);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// (cos, sin) of pos * theta_i for every dim pair i and token t, pos = base + t;
// laid out [pair][token] so a warp's 32 tokens read one contiguous run.
__global__ void rope_table_kernel(const __grid_constant__ RopeArgs r) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (kHead / 2) * r.L) return;
  const int i = idx / r.L, t = idx % r.L;
  float sn, cs;
  sincosf((float)(r.q_pos_base + t) * r.theta[i], &sn, &cs);
  r.rope_q[idx] = make_float2(cs, sn);
  if (r.rope_k != r.rope_q) {
    sincosf((float)(r.kv_pos_base + t) * r.theta[i], &sn, &cs);
    r.rope_k[idx] = make_float2(cs, sn);
  }
}

// One CTA per token.  The statistic is computed so that its fp32 value is
// reproducible: mean(x^2) accumulated in fp64, inv = fp32(1 / sqrt(mean + eps))
// from the fp64 value (IEEE sqrt and division, one rounding to fp32), then
// y = bf16(fp32(fp32(x * inv) * w)).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                      uint16_t* __restrict__ y, int hidden, float eps) {
  __shared__ double red[8];
  const uint16_t* xr = x + (size_t)blockIdx.x * hidden;
  uint16_t* yr = y + (size_t)blockIdx.x * hidden;
  double ss = 0.0;
  for (int i = threadIdx.x * 8; i < hidden; i += 256 * 8) {
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr + i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fma((double)f[j], (double)f[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  double tot = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = (float)(1.0 / sqrt(tot / (double)hidden + (double)eps));
  for (int i = threadIdx.x * 8; i < hidden; i += 256 * 8) {
    float f[8], g[8], o8[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr + i), f);
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(w + i), g);
#pragma unroll
    for (int j = 0; j < 8; ++j) o8[j] = __fmul_rn(__fmul_rn(f[j], inv), g[j]);
    uint4 o;
    o.x = pack2_bf16(o8[0], o8[1]);
    o.y = pack2_bf16(o8[2], o8[3]);
    o.z = pack2_bf16(o8[4], o8[5]);
    o.w = pack2_bf16(o8[6], o8[7]);
    *reinterpret_cast<uint4*>(yr + i) = o;
  }
}

constexpr size_t kStatusBytes = 256;

}  // namespace

// workspace: status word | x_n bf16 [batch * L][hidden] | rope tables 2 x [D/2][L] float2
size_t prologue_workspace_bytes(int batch, int seq_len, int hidden) {
  if (batch < 1 || seq_len < 1 || hidden < 1) return 0;
  const size_t xn = ((size_t)batch * seq_len * hidden * 2 + 255) / 256 * 256;
  return kStatusBytes + xn + 2 * (size_t)(kHead / 2) * seq_len * sizeof(float2);
}

}  // namespace lara

using namespace lara;

extern "C" size_t lara_layer_prologue_workspace_bytes(int batch, int seq_len, int hidden) {
  return prologue_workspace_bytes(batch, seq_len, hidden);
}

extern "C" int lara_layer_prologue(const uint16_t* x, const uint16_t* rms_weight, const uint16_t* w_qkv, uint16_t* q,
                                   uint16_t* k, uint16_t* v, int batch, int seq_len, int hidden, int n_q_heads,
                                   int n_kv_heads, int head_dim, int q_pos_base, int kv_pos_base, float rms_eps,
                                   float rope_base, void* workspace, size_t workspace_bytes, void* stream) {
  LARA_NVTX("lara_layer_prologue");
  if (head_dim != kHead)
    return set_last_error(LARA_ERR_UNSUPPORTED, "the fused projection kernel is built for head_dim 128");
  if (batch < 1 || seq_len < 1 || hidden < kBK || hidden % kBK || n_q_heads < 1 || n_kv_heads < 1 ||
      n_q_heads % n_kv_heads || (long long)batch * seq_len > (1ll << 30))
    return set_last_error(LARA_ERR_BAD_CFG, "bad prologue geometry (hidden must be a positive multiple of 64)");
  if (!(rms_eps >= 0.f) || !(rope_base > 1.f)) return set_last_error(LARA_ERR_BAD_CFG, "bad eps or RoPE base");
  if (q_pos_base < 0 || kv_pos_base < 0 || q_pos_base + seq_len > (1 << 24) || kv_pos_base + seq_len > (1 << 24))
    return set_last_error(LARA_ERR_BAD_CFG, "positions must lie in [0, 2^24) (exact in fp32)");
  if (!x || !w_qkv || !q || !k || !v || !workspace)
    return set_last_error(LARA_ERR_STREAM_DEST, "null pointer");
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_qkv) |
                       reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(workspace) |
                       reinterpret_cast<uintptr_t>(rms_weight);
  if (al & 15) return set_last_error(LARA_ERR_STREAM_DEST, "buffers must be 16-byte aligned");
  if (workspace_bytes < prologue_workspace_bytes(batch, seq_len, hidden))
    return set_last_error(LARA_ERR_RESULT_LEN, "prologue workspace too small");
  if (!tensor_maps_available()) return set_last_error(LARA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows = batch * seq_len;
  int* status = static_cast<int*>(workspace);
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  uint16_t* xn = reinterpret_cast<uint16_t*>(wsb + kStatusBytes);
  float2* rope_q = reinterpret_cast<float2*>(wsb + kStatusBytes + ((size_t)rows * hidden * 2 + 255) / 256 * 256);
  float2* rope_k = q_pos_base == kv_pos_base ? rope_q : rope_q + (size_t)(kHead / 2) * seq_len;
  RopeArgs r{};
  r.rope_q = rope_q;
  r.rope_k = rope_k;
  r.L = seq_len;
  r.q_pos_base = q_pos_base;
  r.kv_pos_base = kv_pos_base;
  for (int i = 0; i < kHead / 2; ++i) r.theta[i] = (float)std::pow((double)rope_base, -2.0 * i / (double)kHead);
  const int n_rope = (kHead / 2) * seq_len;
  rope_table_kernel<<<(n_rope + 255) / 256, 256, 0, st>>>(r);
  const uint16_t* a_src = x;
  if (rms_weight) {
    rmsnorm_kernel<<<rows, 256, 0, st>>>(x, rms_weight, xn, hidden, rms_eps);
    a_src = xn;
  }
  const int n_total = (n_q_heads + 2 * n_kv_heads) * kHead;
  CUtensorMap ma, mb;
  const cuuint64_t ad[2] = {(cuuint64_t)hidden, (cuuint64_t)rows};
  const cuuint64_t as[1] = {(cuuint64_t)hidden * 2};
  const cuuint32_t abox[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  const cuuint64_t bd[2] = {(cuuint64_t)n_total, (cuuint64_t)hidden};
  const cuuint64_t bs[1] = {(cuuint64_t)n_total * 2};
  const cuuint32_t bbox[2] = {64, (cuuint32_t)kBK};
  if (!make_tensor_map_bf16(&ma, a_src, 2, ad, as, abox) || !make_tensor_map_bf16(&mb, w_qkv, 2, bd, bs, bbox))
    return set_last_error(LARA_ERR_CUDA, "tensor map encoding failed");
  ProArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.L = seq_len;
  a.rows = rows;
  a.nk = hidden / kBK;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.n_cols = n_total;
  a.m_tiles = (rows + kBM - 1) / kBM;
  a.n_tiles = (n_total + kBN - 1) / kBN;
  a.rope_q = rope_q;
  a.rope_k = rope_k;
  a.status = status;
  cudaError_t e = cudaFuncSetAttribute(qkv_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return set_last_error(LARA_ERR_CUDA, std::string("prologue: ") + cudaGetErrorString(e));
  const long long tiles = (long long)a.m_tiles * a.n_tiles;
  const int grid = (int)std::min<long long>(tiles, (long long)device_sm_count());
  qkv_rope_kernel<<<grid, kThreads, kSmemAlloc, st>>>(ma, mb, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(LARA_ERR_CUDA, std::string("prologue launch: ") + cudaGetErrorString(e));
  return LARA_OK;
}
