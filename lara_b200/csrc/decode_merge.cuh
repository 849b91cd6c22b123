// Split-KV merge shared by the decode kernels (sm_100a).
//
// Split s of query row b leaves an unnormalised partial state per head h:
// m (running max, log2 domain), l (sum of exp2(score - m)) and acc[D]
// (sum of exp2(score - m) * v).  The last split of a (row, kv head) to
// finish combines them with the log-sum-exp rule
//   M = max_s m_s,  L = sum_s l_s 2^(m_s - M),  o = sum_s acc_s 2^(m_s - M) / L
// and writes bf16 o, or (M, L, acc) in partial-output mode.
#pragma once

#include <cmath>

#include "common.cuh"
#include "lara_internal.h"

namespace lara {

constexpr int kPreloadSplits = 8;  // split counts up to this merge from registers loaded in one batch

template <int D>
__device__ __forceinline__ void merge_split_partials(const DecodeParams& p, int b, int kvh, int group, int nsplit_b,
                                                     bool partial_out, int tid, int nthreads) {
  for (int idx = tid; idx < group * D / 2; idx += nthreads) {
    const int g = idx / (D / 2);
    const int d = (idx % (D / 2)) * 2;
    const int h = kvh * group + g;
    const long long row = (long long)b * p.n_q_heads + h;
    const float* ml = p.part_ml + row * p.nsplit * 2;
    const float* pa = p.part_acc + row * p.nsplit * D;
    float M = -INFINITY, L = 0.f, o0 = 0.f, o1 = 0.f;
    if (nsplit_b <= kPreloadSplits) {
      // All partials are loaded at once, so the merge at the end of the
      // kernel waits on one L2 round trip rather than one per dependent load.
      float2 mlv[kPreloadSplits], av[kPreloadSplits];
#pragma unroll
      for (int s2 = 0; s2 < kPreloadSplits; ++s2)
        if (s2 < nsplit_b) {
          mlv[s2] = __ldcg(reinterpret_cast<const float2*>(ml + s2 * 2));
          av[s2] = __ldcg(reinterpret_cast<const float2*>(pa + (long long)s2 * D + d));
        }
#pragma unroll
      for (int s2 = 0; s2 < kPreloadSplits; ++s2)
        if (s2 < nsplit_b) M = fmaxf(M, mlv[s2].x);
      const float Mu = (M == -INFINITY) ? 0.f : M;
#pragma unroll
      for (int s2 = 0; s2 < kPreloadSplits; ++s2)
        if (s2 < nsplit_b) {
          const float sc = exp2f(mlv[s2].x - Mu);
          L = fmaf(mlv[s2].y, sc, L);
          o0 = fmaf(av[s2].x, sc, o0);
          o1 = fmaf(av[s2].y, sc, o1);
        }
    } else {
      for (int s2 = 0; s2 < nsplit_b; ++s2) M = fmaxf(M, __ldcg(ml + s2 * 2));
      const float Mu = (M == -INFINITY) ? 0.f : M;
      for (int s2 = 0; s2 < nsplit_b; ++s2) {
        const float sc = exp2f(__ldcg(ml + s2 * 2) - Mu);
        L = fmaf(__ldcg(ml + s2 * 2 + 1), sc, L);
        const float2 a = __ldcg(reinterpret_cast<const float2*>(pa + (long long)s2 * D + d));
        o0 = fmaf(a.x, sc, o0);
        o1 = fmaf(a.y, sc, o1);
      }
    }
    if (partial_out) {
      *reinterpret_cast<float2*>(p.out_acc + row * D + d) = make_float2(o0, o1);
      if (d == 0) { p.out_ml[row * 2] = M; p.out_ml[row * 2 + 1] = L; }
    } else {
      const float inv = (L > 0.f) ? 1.f / L : 0.f;
      *reinterpret_cast<uint32_t*>(p.o + b * p.o_sb + h * p.o_sh + d) = pack2_bf16(o0 * inv, o1 * inv);
    }
  }
}

}  // namespace lara
