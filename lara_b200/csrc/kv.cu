// KV-cache append, bf16 packing and the split-KV log-sum-exp combine.
//
// * kv_append: the B200 replacement for the per-group K/V cache write of
//   hw/rtl/mem/kv_cache_ram.sv:45-91 (write address token*128+dim): new
//   rows land at position lens[b] of each (sequence, kv head) row of the HBM
//   cache [B, Hkv, Lmax, D]; lens[b] then advances by n_new.
// * kv_append_paged: the same write into a paged cache (page pool plus a
//   per-sequence block table).
// * pack_bf16: the reference's host packer fp32_to_bf16_u16
//   (sw/attn_driver.py:88-98) as a device kernel with the same integer steps.
// * lse_combine: merges P partial results (m in log2 domain, l, unnormalised
//   acc[D]) of the same query rows, e.g. the per-GPU partials of a sequence
//   split across GPUs:  M = max m_i, L = sum l_i 2^(m_i-M),
//   O = sum acc_i 2^(m_i-M) / L, bf16 RNE out (l == 0 -> 0, as the RTL
//   normaliser does, hw/rtl/mem/output_buffer.sv:271-286).
#include "common.cuh"
#include "lara_internal.h"

namespace lara {

namespace {

// One 16-byte vector per thread; row r = ((b * Hkv + h) * n_new + t).
__global__ void kv_append_kernel(uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                                 const int32_t* __restrict__ lens, const uint16_t* __restrict__ k_new,
                                 const uint16_t* __restrict__ v_new, int batch, int n_kv_heads, int head_dim,
                                 int max_seq_len, int n_new, int* status) {
  const int vec_per_row = head_dim / 8;
  const long long total = (long long)batch * n_kv_heads * n_new * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec_per_row;
    const int vec = (int)(i % vec_per_row);
    const int t = (int)(row % n_new);
    const long long bh = row / n_new;
    const int b = (int)(bh / n_kv_heads);
    const int len = lens[b];
    const long long pos = (long long)len + t;
    if (len < 0 || pos >= max_seq_len) {
      if (status) atomicOr(status, kDevAppendOverflow);
      continue;
    }
    const long long dst = (bh * max_seq_len + pos) * head_dim + vec * 8;
    const long long src = row * head_dim + vec * 8;
    *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(k_new + src);
    *reinterpret_cast<uint4*>(v_cache + dst) = *reinterpret_cast<const uint4*>(v_new + src);
  }
}

// Paged cache: row (b, h, t) lands in page block_table[b][pos >> page_log2],
// row pos & (page - 1), pos = lens[b] + t, of the pool [pages][Hkv][page][D].
__global__ void kv_append_paged_kernel(uint16_t* __restrict__ k_pages, uint16_t* __restrict__ v_pages,
                                       const int32_t* __restrict__ block_table, const int32_t* __restrict__ lens,
                                       const uint16_t* __restrict__ k_new, const uint16_t* __restrict__ v_new,
                                       int batch, int n_kv_heads, int head_dim, int page_log2, int pages_per_seq,
                                       int num_pages, int n_new, int* status) {
  const int vec_per_row = head_dim / 8;
  const long long max_seq_len = (long long)pages_per_seq << page_log2;
  const long long total = (long long)batch * n_kv_heads * n_new * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec_per_row;
    const int vec = (int)(i % vec_per_row);
    const int t = (int)(row % n_new);
    const long long bh = row / n_new;
    const int b = (int)(bh / n_kv_heads), h = (int)(bh % n_kv_heads);
    const int len = lens[b];
    const long long pos = (long long)len + t;
    if (len < 0 || pos >= max_seq_len) {
      if (status) atomicOr(status, kDevAppendOverflow);
      continue;
    }
    const int page = block_table[(long long)b * pages_per_seq + (pos >> page_log2)];
    if (page < 0 || page >= num_pages) {
      if (status) atomicOr(status, kDevBadPage);
      continue;
    }
    const long long in_page = pos & ((1ll << page_log2) - 1);
    const long long dst = ((((long long)page * n_kv_heads + h) << page_log2) + in_page) * head_dim + vec * 8;
    const long long src = row * head_dim + vec * 8;
    *reinterpret_cast<uint4*>(k_pages + dst) = *reinterpret_cast<const uint4*>(k_new + src);
    *reinterpret_cast<uint4*>(v_pages + dst) = *reinterpret_cast<const uint4*>(v_new + src);
  }
}

__global__ void lens_add_kernel(int32_t* lens, int batch, int n_new, int max_seq_len) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) {
    const int l = lens[b] + n_new;
    lens[b] = l > max_seq_len ? max_seq_len : l;
  }
}

__global__ void pack_bf16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, size_t n) {
  const size_t nvec = n / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nvec; i += (size_t)gridDim.x * blockDim.x) {
    const float4 f = reinterpret_cast<const float4*>(src)[i];
    uint2 w;
    w.x = pack2_bf16(f.x, f.y);
    w.y = pack2_bf16(f.z, f.w);
    reinterpret_cast<uint2*>(dst)[i] = w;
  }
  // tail (fewer than 4 elements), one thread
  if (blockIdx.x == 0 && threadIdx.x == 0)
    for (size_t i = nvec * 4; i < n; ++i) dst[i] = (uint16_t)f32_to_bf16_rne_bits(src[i]);
}

// One warp per output row; lanes stride over the head dims.  Part i of row r
// has (m, l) at part_ml[i * ml_stride + r * 2] and acc at
// part_acc[i * acc_stride + r * head_dim] (strides in floats), so partials
// gathered from several devices can stay packed per device.
__global__ void lse_combine_kernel(const float* __restrict__ part_ml, long long ml_stride,
                                   const float* __restrict__ part_acc, long long acc_stride, int num_parts,
                                   int rows, int head_dim, uint16_t* __restrict__ o, float* __restrict__ out_ml,
                                   float* __restrict__ out_acc) {
  const int warps_per_block = blockDim.x / 32;
  const int row = blockIdx.x * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int i = 0; i < num_parts; ++i) M = fmaxf(M, part_ml[i * ml_stride + row * 2]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  for (int i = 0; i < num_parts; ++i) {
    const float* ml = part_ml + i * ml_stride + row * 2;
    L = fmaf(ml[1], exp2f(ml[0] - Mu), L);
  }
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  for (int d = lane * 2; d < head_dim; d += 64) {
    float o0 = 0.f, o1 = 0.f;
    for (int i = 0; i < num_parts; ++i) {
      const float sc = exp2f(part_ml[i * ml_stride + row * 2] - Mu);
      const float2 a = *reinterpret_cast<const float2*>(part_acc + i * acc_stride + (long long)row * head_dim + d);
      o0 = fmaf(a.x, sc, o0);
      o1 = fmaf(a.y, sc, o1);
    }
    if (o) {
      *reinterpret_cast<uint32_t*>(o + (long long)row * head_dim + d) = pack2_bf16(o0 * inv, o1 * inv);
    } else {
      out_acc[(long long)row * head_dim + d] = o0;
      out_acc[(long long)row * head_dim + d + 1] = o1;
    }
  }
  if (!o && lane == 0) {
    out_ml[row * 2] = M;
    out_ml[row * 2 + 1] = L;
  }
}

int grid_for(long long work, int threads) {
  const long long want = (work + threads - 1) / threads;
  const long long cap = (long long)device_sm_count() * 16;
  return (int)(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace

cudaError_t kv_append_launch(uint16_t* k_cache, uint16_t* v_cache, int32_t* lens, const uint16_t* k_new,
                             const uint16_t* v_new, int batch, int n_kv_heads, int head_dim, int max_seq_len,
                             int n_new, int* status, cudaStream_t stream) {
  if (n_new <= 0) return cudaSuccess;
  const long long work = (long long)batch * n_kv_heads * n_new * (head_dim / 8);
  kv_append_kernel<<<grid_for(work, 256), 256, 0, stream>>>(k_cache, v_cache, lens, k_new, v_new, batch, n_kv_heads,
                                                           head_dim, max_seq_len, n_new, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  lens_add_kernel<<<(batch + 255) / 256, 256, 0, stream>>>(lens, batch, n_new, max_seq_len);
  return cudaGetLastError();
}

cudaError_t kv_append_paged_launch(uint16_t* k_pages, uint16_t* v_pages, const int32_t* block_table, int32_t* lens,
                                   const uint16_t* k_new, const uint16_t* v_new, int batch, int n_kv_heads,
                                   int head_dim, int page_log2, int pages_per_seq, int num_pages, int n_new,
                                   int* status, cudaStream_t stream) {
  if (n_new <= 0) return cudaSuccess;
  const long long work = (long long)batch * n_kv_heads * n_new * (head_dim / 8);
  kv_append_paged_kernel<<<grid_for(work, 256), 256, 0, stream>>>(k_pages, v_pages, block_table, lens, k_new, v_new,
                                                                 batch, n_kv_heads, head_dim, page_log2,
                                                                 pages_per_seq, num_pages, n_new, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long cap = (long long)pages_per_seq << page_log2;
  lens_add_kernel<<<(batch + 255) / 256, 256, 0, stream>>>(lens, batch, n_new, (int)(cap > 0x7fffffff ? 0x7fffffff : cap));
  return cudaGetLastError();
}

cudaError_t pack_bf16_launch(const float* src, uint16_t* dst, size_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  pack_bf16_kernel<<<grid_for((long long)(n / 4 + 1), 256), 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t lse_combine_launch(const float* part_ml, long long ml_stride, const float* part_acc, long long acc_stride,
                               int num_parts, int rows, int head_dim, uint16_t* o, float* out_ml, float* out_acc,
                               cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int warps = 8;
  lse_combine_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, stream>>>(
      part_ml, ml_stride, part_acc, acc_stride, num_parts, rows, head_dim, o, out_ml, out_acc);
  return cudaGetLastError();
}

}  // namespace lara
