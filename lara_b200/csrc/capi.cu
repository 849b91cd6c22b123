// C ABI of liblara_b200.so (declared in include/lara_b200.h).
//
// Host-side validation mirrors the reference driver: a bad length or shape is
// rejected before any launch (sw/attn_driver.py:347-349,366-372,486-490), and
// device-side problems come back as status bits in the workspace, which the
// context reads after every transaction (the sticky ERROR_CODE CSR of
// hw/rtl/axi/attn_axi_lite_slave.sv:174-207).
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/lara_b200.h"
#include "lara_internal.h"

using lara::DecodeParams;


namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(LARA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define LARA_CUDA(call)                                \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_geometry(int batch, int hq, int hkv, int d, int lmax) {
  if (batch < 1 || hq < 1 || hkv < 1 || d < 1 || lmax < 1)
    return fail(LARA_ERR_BAD_CFG, "geometry must be positive: batch=%d hq=%d hkv=%d d=%d lmax=%d", batch, hq, hkv,
                d, lmax);
  if (hq % hkv != 0) return fail(LARA_ERR_BAD_CFG, "n_q_heads (%d) must be a multiple of n_kv_heads (%d)", hq, hkv);
  if (lara::decode_chunk_granule(d, hq / hkv) == 0)
    return fail(LARA_ERR_UNSUPPORTED, "no kernel compiled for head_dim=%d group=%d (supported: head_dim 64/128 with "
                "group 1, 2, 4, 8; head_dim 128 with group 16 on the tensor-core kernel)", d, hq / hkv);
  if (batch > 65535) return fail(LARA_ERR_BAD_CFG, "batch %d exceeds 65535", batch);
  return LARA_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int resolve_plan(int batch, int hq, int hkv, int d, int lmax, const int32_t* lens_host, int* nsplit, int* chunk) {
  if (*nsplit > 0 && *chunk > 0) {
    const int tile = lara::decode_chunk_granule(d, hq / hkv);
    if (*chunk % tile != 0)
      return fail(LARA_ERR_BAD_CFG, "chunk_tokens (%d) must be a multiple of the kernel tile (%d)", *chunk, tile);
    // splits that do not cover lmax leave the rest to split 0 (decode_first_chunk)
    return LARA_OK;
  }
  lara::decode_plan(batch, hkv, hq, d, lmax, lens_host, nsplit, chunk);
  return LARA_OK;
}

int decode_common(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* lens, uint16_t* o,
                  float* out_ml, float* out_acc, int batch, int hq, int hkv, int d, int lmax, float scale, int nsplit,
                  int chunk, void* ws, size_t ws_bytes, void* stream, const int32_t* block_table = nullptr,
                  int page_log2 = 0, int pages_per_seq = 0, int num_pages = 0) {
  int rc = check_geometry(batch, hq, hkv, d, lmax);
  if (rc) return rc;
  if (!q || !k || !v || !lens || !ws || (!o && !out_acc))
    return fail(LARA_ERR_STREAM_DEST, "null tensor or workspace pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || (o && !aligned(o, 4)) || !aligned(ws, 256) ||
      (out_acc && !aligned(out_acc, 8)))
    return fail(LARA_ERR_STREAM_DEST, "q/k/v must be 16-byte aligned, o 4-byte, workspace 256-byte");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(LARA_ERR_BAD_CFG, "scale must be positive and finite");
  rc = resolve_plan(batch, hq, hkv, d, lmax, nullptr, &nsplit, &chunk);
  if (rc) return rc;
  const lara::WorkspaceLayout w = lara::decode_workspace_layout(batch, hq, hkv, d, nsplit);
  if (ws_bytes < w.total)
    return fail(LARA_ERR_RESULT_LEN, "workspace has %zu bytes, %zu needed for %d splits", ws_bytes, w.total, nsplit);
  DecodeParams p{};
  p.q = q; p.q_sb = (long long)hq * d; p.q_sh = d;
  p.k = k; p.v = v; p.kv_sb = (long long)hkv * lmax * d; p.kv_sh = (long long)lmax * d;
  p.o = o; p.o_sb = (long long)hq * d; p.o_sh = d;
  p.lens = lens; p.len_c0 = 0; p.len_c1 = 0; p.rows_per_seq = 1; p.max_seq_len = lmax;
  p.batch = batch; p.n_q_heads = hq; p.n_kv_heads = hkv; p.head_dim = d;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.chunk = chunk; p.nsplit = nsplit;
  char* base = static_cast<char*>(ws);
  p.status = reinterpret_cast<int*>(base + w.status_off);
  p.counters = reinterpret_cast<int*>(base + w.counters_off);
  p.part_ml = reinterpret_cast<float*>(base + w.ml_off);
  p.part_acc = reinterpret_cast<float*>(base + w.acc_off);
  p.out_ml = out_ml; p.out_acc = out_acc;
  p.block_table = block_table; p.page_log2 = page_log2; p.pages_per_seq = pages_per_seq; p.num_pages = num_pages;
  p.chunk0 = lara::decode_first_chunk(nsplit, chunk, hq / hkv, d, (long long)batch * hkv, lmax);
  cudaError_t e = lara::decode_launch(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return LARA_OK;
}

// Paged-cache geometry: page a power of two in [16, 65536], and the per
// sequence capacity pages_per_seq * page_size representable as int.
int check_paged(int page_size, int pages_per_seq, int num_pages, int* page_log2) {
  if (page_size < 16 || page_size > 65536 || (page_size & (page_size - 1)))
    return fail(LARA_ERR_BAD_CFG, "page_size must be a power of two in [16, 65536], got %d", page_size);
  if (pages_per_seq < 1 || num_pages < 1 || (long long)pages_per_seq * page_size > 0x7fffffffll)
    return fail(LARA_ERR_BAD_CFG, "bad paged-cache geometry");
  int l = 0;
  while ((1 << l) < page_size) ++l;
  *page_log2 = l;
  return LARA_OK;
}

// Which kernel runs prefill / dense attention: the tcgen05 tensor-core
// kernel for head_dim 128 (default), or the CUDA-core streaming kernel.
// LARA_ATTN_PATH=stream|tc overrides (tc fails if the geometry has no
// tensor-core kernel).
enum class AttnPath { kAuto, kStream, kTensor };

AttnPath attn_path_override() {
  const char* e = std::getenv("LARA_ATTN_PATH");
  if (!e) return AttnPath::kAuto;
  if (std::strcmp(e, "stream") == 0) return AttnPath::kStream;
  if (std::strcmp(e, "tc") == 0) return AttnPath::kTensor;
  return AttnPath::kAuto;
}

// Launch the tensor-core kernel if selected; returns LARA_OK when it ran,
// -1 when the streaming kernel should run instead, or an error code.
int try_tensor_path(lara::PrefillTcParams tp, cudaStream_t st) {
  const AttnPath path = attn_path_override();
  // By default P is split into two bf16 terms (P_hi + P_lo, ~16 significant
  // bits, two P.V passes) so the output meets the <= 2 ulp parity bound;
  // LARA_TC_SPLIT_P=0 rounds P to one bf16 (RNE, the FlashAttention choice:
  // faster, error ~1 bf16 ulp of the head vector's largest element).
  const char* sp = std::getenv("LARA_TC_SPLIT_P");
  tp.split_p = (sp && std::strcmp(sp, "0") == 0) ? 0 : 1;
  if (path == AttnPath::kStream) return -1;
  if (!lara::prefill_tc_supported(tp.head_dim, tp.n_q_heads, tp.n_kv_heads)) {
    if (path == AttnPath::kTensor)
      return fail(LARA_ERR_UNSUPPORTED, "LARA_ATTN_PATH=tc but no tensor-core kernel for head_dim=%d", tp.head_dim);
    return -1;
  }
  const cudaError_t e = lara::prefill_tc_launch(tp, st);
  if (e == cudaSuccess) return LARA_OK;
  if (e == cudaErrorInvalidValue && path != AttnPath::kTensor) {
    cudaGetLastError();  // tensor map not encodable for this shape: stream instead
    return -1;
  }
  return cuda_fail(e, "tensor-core attention launch");
}

// Split 0's tokens for a plan from decode_plan on the dense and prefill rows:
// the rest of max_seq_len when the splits do not cover it, else equal splits.
int rest_first_chunk(int nsplit, int chunk, int hq, int hkv, int d, int lmax) {
  return (long long)nsplit * chunk < lmax ? lara::decode_first_chunk(nsplit, chunk, hq / hkv, d, 0, lmax) : 0;
}

size_t dense_ws_bytes(int hq, int hkv, int d, int L, int* nsplit, int* chunk) {
  lara::decode_plan(L, hkv, hq, d, L, nullptr, nsplit, chunk);
  return lara::decode_workspace_layout(L, hq, hkv, d, *nsplit).total;
}

int dense_common(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int hq, int hkv, int d, int L,
                 int q_pos_base, int kv_pos_base, int causal, float scale, void* ws, size_t ws_bytes, void* stream) {
  int rc = check_geometry(L, hq, hkv, d, L);
  if (rc) return rc;
  if (!q || !k || !v || !o || !ws) return fail(LARA_ERR_STREAM_DEST, "null tensor or workspace pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 4) || !aligned(ws, 256))
    return fail(LARA_ERR_STREAM_DEST, "q/k/v must be 16-byte aligned, o 4-byte, workspace 256-byte");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(LARA_ERR_BAD_CFG, "scale must be positive and finite");
  if (ws_bytes < 256) return fail(LARA_ERR_RESULT_LEN, "workspace has %zu bytes, at least 256 needed", ws_bytes);
  {
    lara::PrefillTcParams tp{};
    tp.q = q; tp.q_sb = (long long)hq * L * d; tp.q_sr = d; tp.q_sh = (long long)L * d;
    tp.k = k; tp.v = v; tp.kv_rows = L;
    tp.o = o; tp.o_sb = tp.q_sb; tp.o_sr = d; tp.o_sh = (long long)L * d;
    tp.batch = 1; tp.n_q = L; tp.n_q_heads = hq; tp.n_kv_heads = hkv; tp.head_dim = d;
    tp.base_lens = nullptr; tp.kv_add = L; tp.q_add = q_pos_base - kv_pos_base; tp.causal = causal ? 1 : 0;
    tp.scale_log2 = scale * 1.4426950408889634f;
    tp.status = static_cast<int*>(ws);
    const int r = try_tensor_path(tp, static_cast<cudaStream_t>(stream));
    if (r != -1) return r;
  }
  int nsplit = 0, chunk = 0;
  const size_t need = dense_ws_bytes(hq, hkv, d, L, &nsplit, &chunk);
  if (ws_bytes < need) return fail(LARA_ERR_RESULT_LEN, "workspace has %zu bytes, %zu needed", ws_bytes, need);
  const lara::WorkspaceLayout w = lara::decode_workspace_layout(L, hq, hkv, d, nsplit);
  DecodeParams p{};
  // Query row i of every head is an independent "sequence" b = i that
  // shares the group's K/V (batch stride 0) and sees a prefix of the keys.
  p.q = q; p.q_sb = d; p.q_sh = (long long)L * d;
  p.k = k; p.v = v; p.kv_sb = 0; p.kv_sh = (long long)L * d;
  p.o = o; p.o_sb = d; p.o_sh = (long long)L * d;
  p.lens = nullptr;
  if (causal) {
    // key j visible iff kv_pos_base + j <= q_pos_base + i  <=>  j < q_pos_base - kv_pos_base + i + 1
    p.len_c0 = q_pos_base - kv_pos_base + 1;
    p.len_c1 = 1;
  } else {
    p.len_c0 = L;
    p.len_c1 = 0;
  }
  p.rows_per_seq = L;
  p.max_seq_len = L;
  p.batch = L; p.n_q_heads = hq; p.n_kv_heads = hkv; p.head_dim = d;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.chunk = chunk; p.nsplit = nsplit;
  p.chunk0 = rest_first_chunk(nsplit, chunk, hq, hkv, d, L);
  char* base = static_cast<char*>(ws);
  p.status = reinterpret_cast<int*>(base + w.status_off);
  p.counters = reinterpret_cast<int*>(base + w.counters_off);
  p.part_ml = reinterpret_cast<float*>(base + w.ml_off);
  p.part_acc = reinterpret_cast<float*>(base + w.acc_off);
  cudaError_t e = lara::decode_launch(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dense launch");
  return LARA_OK;
}

size_t prefill_ws_bytes(int batch, int n_new, int hq, int hkv, int d, int lmax, int* nsplit, int* chunk) {
  lara::decode_plan(batch * n_new, hkv, hq, d, lmax, nullptr, nsplit, chunk);
  return lara::decode_workspace_layout(batch * n_new, hq, hkv, d, *nsplit).total;
}

int prefill_common(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* cached_lens, uint16_t* o,
                   int batch, int n_new, int hq, int hkv, int d, int lmax, int causal, float scale, void* ws,
                   size_t ws_bytes, void* stream) {
  if (batch < 1 || n_new < 1) return fail(LARA_ERR_BAD_CFG, "batch and n_new must be >= 1");
  if ((long long)batch * n_new > 65535)
    return fail(LARA_ERR_BAD_CFG, "batch*n_new (%lld) exceeds 65535 query rows", (long long)batch * n_new);
  int rc = check_geometry(batch * n_new, hq, hkv, d, lmax);
  if (rc) return rc;
  if (!q || !k || !v || !cached_lens || !o || !ws) return fail(LARA_ERR_STREAM_DEST, "null tensor or workspace pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 4) || !aligned(ws, 256))
    return fail(LARA_ERR_STREAM_DEST, "q/k/v must be 16-byte aligned, o 4-byte, workspace 256-byte");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(LARA_ERR_BAD_CFG, "scale must be positive and finite");
  if (ws_bytes < 256) return fail(LARA_ERR_RESULT_LEN, "workspace has %zu bytes, at least 256 needed", ws_bytes);
  {
    lara::PrefillTcParams tp{};
    tp.q = q; tp.q_sb = (long long)n_new * hq * d; tp.q_sr = (long long)hq * d; tp.q_sh = d;
    tp.k = k; tp.v = v; tp.kv_rows = lmax;
    tp.o = o; tp.o_sb = tp.q_sb; tp.o_sr = tp.q_sr; tp.o_sh = d;
    tp.batch = batch; tp.n_q = n_new; tp.n_q_heads = hq; tp.n_kv_heads = hkv; tp.head_dim = d;
    tp.base_lens = cached_lens; tp.kv_add = n_new; tp.q_add = 0; tp.causal = causal ? 1 : 0;
    tp.scale_log2 = scale * 1.4426950408889634f;
    tp.status = static_cast<int*>(ws);
    const int r = try_tensor_path(tp, static_cast<cudaStream_t>(stream));
    if (r != -1) return r;
  }
  int nsplit = 0, chunk = 0;
  const size_t need = prefill_ws_bytes(batch, n_new, hq, hkv, d, lmax, &nsplit, &chunk);
  if (ws_bytes < need) return fail(LARA_ERR_RESULT_LEN, "workspace has %zu bytes, %zu needed", ws_bytes, need);
  const lara::WorkspaceLayout w = lara::decode_workspace_layout(batch * n_new, hq, hkv, d, nsplit);
  DecodeParams p{};
  p.q = q; p.q_sb = (long long)hq * d; p.q_sh = d;
  p.k = k; p.v = v; p.kv_sb = (long long)hkv * lmax * d; p.kv_sh = (long long)lmax * d;
  p.o = o; p.o_sb = (long long)hq * d; p.o_sh = d;
  p.lens = cached_lens;
  p.rows_per_seq = n_new;
  p.len_c0 = causal ? 1 : n_new;
  p.len_c1 = causal ? 1 : 0;
  p.max_seq_len = lmax;
  p.batch = batch * n_new; p.n_q_heads = hq; p.n_kv_heads = hkv; p.head_dim = d;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.chunk = chunk; p.nsplit = nsplit;
  p.chunk0 = rest_first_chunk(nsplit, chunk, hq, hkv, d, lmax);
  char* base = static_cast<char*>(ws);
  p.status = reinterpret_cast<int*>(base + w.status_off);
  p.counters = reinterpret_cast<int*>(base + w.counters_off);
  p.part_ml = reinterpret_cast<float*>(base + w.ml_off);
  p.part_acc = reinterpret_cast<float*>(base + w.acc_off);
  cudaError_t e = lara::decode_launch(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return LARA_OK;
}

std::string describe_status(int bits) {
  std::string s;
  if (bits & lara::kDevWaitTimeout) s += " wait-timeout";
  if (bits & lara::kDevBadLength) s += " bad-sequence-length";
  if (bits & lara::kDevAppendOverflow) s += " append-overflow";
  if (bits & lara::kDevBadPage) s += " bad-page-index";
  return s.empty() ? std::string(" unknown") : s;
}

}  // namespace

namespace lara {
int set_last_error(int code, const std::string& message) {
  g_last_error = message;
  return code;
}
}  // namespace lara

// ===========================================================================
// stateless API
// ===========================================================================

extern "C" {

int lara_abi_version(void) { return LARA_ABI_VERSION; }

const char* lara_last_error_string(void) { return g_last_error.c_str(); }

const char* lara_status_name(int status) {
  switch (status) {
    case LARA_OK: return "LARA_OK";
    case LARA_ERR_BAD_CFG: return "LARA_ERR_BAD_CFG";
    case LARA_ERR_BUSY_START: return "LARA_ERR_BUSY_START";
    case LARA_ERR_STREAM_LEN: return "LARA_ERR_STREAM_LEN";
    case LARA_ERR_STREAM_DEST: return "LARA_ERR_STREAM_DEST";
    case LARA_ERR_RESULT_LEN: return "LARA_ERR_RESULT_LEN";
    case LARA_ERR_CUDA: return "LARA_ERR_CUDA";
    case LARA_ERR_TIMEOUT: return "LARA_ERR_TIMEOUT";
    case LARA_ERR_UNSUPPORTED: return "LARA_ERR_UNSUPPORTED";
    case LARA_ERR_DEVICE: return "LARA_ERR_DEVICE";
    default: return "LARA_ERR_UNKNOWN";
  }
}

int lara_decode_plan(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len,
                     const int32_t* lens_host, int* num_splits, int* chunk_tokens) {
  int rc = check_geometry(batch, n_q_heads, n_kv_heads, head_dim, max_seq_len);
  if (rc) return rc;
  if (!num_splits || !chunk_tokens) return fail(LARA_ERR_STREAM_DEST, "null output pointer");
  lara::decode_plan(batch, n_kv_heads, n_q_heads, head_dim, max_seq_len, lens_host, num_splits, chunk_tokens);
  return LARA_OK;
}

int lara_decode_kernel(int n_q_heads, int n_kv_heads, int head_dim) {
  if (n_q_heads < 1 || n_kv_heads < 1 || n_q_heads % n_kv_heads) return LARA_DECODE_KERNEL_CUDA_CORE;
  return lara::decode_tc_selected(head_dim, n_q_heads / n_kv_heads) ? LARA_DECODE_KERNEL_TENSOR
                                                                     : LARA_DECODE_KERNEL_CUDA_CORE;
}

size_t lara_decode_workspace_bytes(int batch, int n_q_heads, int n_kv_heads, int head_dim, int num_splits) {
  if (batch < 1 || n_q_heads < 1 || n_kv_heads < 1 || head_dim < 1) return 0;
  return lara::decode_workspace_layout(batch, n_q_heads, n_kv_heads, head_dim, num_splits < 1 ? 1 : num_splits).total;
}

int lara_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace) return fail(LARA_ERR_STREAM_DEST, "null workspace");
  LARA_CUDA(cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)));
  return LARA_OK;
}

int lara_workspace_status(void* workspace, void* stream, int* device_status) {
  if (!workspace || !device_status) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int bits = 0;
  LARA_CUDA(cudaMemcpyAsync(&bits, workspace, sizeof(int), cudaMemcpyDeviceToHost, st));
  LARA_CUDA(cudaStreamSynchronize(st));
  LARA_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), st));
  *device_status = bits;
  return LARA_OK;
}

int lara_gqa_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* seq_lens,
                    uint16_t* o, int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len,
                    float scale, int num_splits, int chunk_tokens, void* workspace, size_t workspace_bytes,
                    void* stream) {
  LARA_NVTX("lara_gqa_decode");
  if (!o) return fail(LARA_ERR_STREAM_DEST, "null output pointer");
  return decode_common(q, k_cache, v_cache, seq_lens, o, nullptr, nullptr, batch, n_q_heads, n_kv_heads, head_dim,
                       max_seq_len, scale, num_splits, chunk_tokens, workspace, workspace_bytes, stream);
}

int lara_gqa_decode_partial(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            const int32_t* seq_lens, float* part_ml, float* part_acc, int batch, int n_q_heads,
                            int n_kv_heads, int head_dim, int max_seq_len, float scale, int num_splits,
                            int chunk_tokens, void* workspace, size_t workspace_bytes, void* stream) {
  LARA_NVTX("lara_gqa_decode_partial");
  if (!part_ml || !part_acc) return fail(LARA_ERR_STREAM_DEST, "null partial output pointer");
  return decode_common(q, k_cache, v_cache, seq_lens, nullptr, part_ml, part_acc, batch, n_q_heads, n_kv_heads,
                       head_dim, max_seq_len, scale, num_splits, chunk_tokens, workspace, workspace_bytes, stream);
}

int lara_lse_combine(const float* part_ml, const float* part_acc, int num_parts, int rows, int head_dim, uint16_t* o,
                     void* stream) {
  LARA_NVTX("lara_lse_combine");
  if (!part_ml || !part_acc || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (num_parts < 1 || rows < 1 || head_dim < 2 || head_dim % 2)
    return fail(LARA_ERR_BAD_CFG, "num_parts, rows must be >= 1 and head_dim even");
  if (!aligned(part_acc, 8) || !aligned(o, 4)) return fail(LARA_ERR_STREAM_DEST, "misaligned buffer");
  cudaError_t e = lara::lse_combine_launch(part_ml, 2LL * rows, part_acc, (long long)rows * head_dim, num_parts, rows,
                                           head_dim, o, nullptr, nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lse_combine launch");
  return LARA_OK;
}

int lara_lse_combine_strided(const float* part_ml, long long ml_part_stride, const float* part_acc,
                             long long acc_part_stride, int num_parts, int rows, int head_dim, uint16_t* o,
                             void* stream) {
  if (!part_ml || !part_acc || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (num_parts < 1 || rows < 1 || head_dim < 2 || head_dim % 2)
    return fail(LARA_ERR_BAD_CFG, "num_parts, rows must be >= 1 and head_dim even");
  if (ml_part_stride < 2LL * rows || acc_part_stride < (long long)rows * head_dim || ml_part_stride % 2 ||
      acc_part_stride % 2)
    return fail(LARA_ERR_BAD_CFG, "part strides must be even and cover rows*2 / rows*head_dim floats");
  if (!aligned(part_ml, 8) || !aligned(part_acc, 8) || !aligned(o, 4))
    return fail(LARA_ERR_STREAM_DEST, "misaligned buffer");
  cudaError_t e = lara::lse_combine_launch(part_ml, ml_part_stride, part_acc, acc_part_stride, num_parts, rows,
                                           head_dim, o, nullptr, nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lse_combine launch");
  return LARA_OK;
}

int lara_kv_append(uint16_t* k_cache, uint16_t* v_cache, int32_t* seq_lens, const uint16_t* k_new,
                   const uint16_t* v_new, int batch, int n_kv_heads, int head_dim, int max_seq_len, int n_new,
                   void* workspace, void* stream) {
  LARA_NVTX("lara_kv_append");
  if (!k_cache || !v_cache || !seq_lens || !k_new || !v_new) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (batch < 1 || n_kv_heads < 1 || head_dim < 8 || head_dim % 8 || max_seq_len < 1 || n_new < 0)
    return fail(LARA_ERR_BAD_CFG, "bad append geometry");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(k_new, 16) || !aligned(v_new, 16))
    return fail(LARA_ERR_STREAM_DEST, "cache and new rows must be 16-byte aligned");
  int* status = workspace ? static_cast<int*>(workspace) : nullptr;
  cudaError_t e = lara::kv_append_launch(k_cache, v_cache, seq_lens, k_new, v_new, batch, n_kv_heads, head_dim,
                                         max_seq_len, n_new, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  return LARA_OK;
}

int lara_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages,
                          const int32_t* block_table, const int32_t* seq_lens, uint16_t* o, int batch, int n_q_heads,
                          int n_kv_heads, int head_dim, int page_size, int pages_per_seq, int num_pages, float scale,
                          int num_splits, int chunk_tokens, void* workspace, size_t workspace_bytes, void* stream) {
  LARA_NVTX("lara_gqa_decode_paged");
  int page_log2 = 0;
  int rc = check_paged(page_size, pages_per_seq, num_pages, &page_log2);
  if (rc) return rc;
  if (!block_table) return fail(LARA_ERR_STREAM_DEST, "null block table");
  return decode_common(q, k_pages, v_pages, seq_lens, o, nullptr, nullptr, batch, n_q_heads, n_kv_heads, head_dim,
                       pages_per_seq * page_size, scale, num_splits, chunk_tokens, workspace, workspace_bytes, stream,
                       block_table, page_log2, pages_per_seq, num_pages);
}

int lara_kv_append_paged(uint16_t* k_pages, uint16_t* v_pages, const int32_t* block_table, int32_t* seq_lens,
                         const uint16_t* k_new, const uint16_t* v_new, int batch, int n_kv_heads, int head_dim,
                         int page_size, int pages_per_seq, int num_pages, int n_new, void* workspace, void* stream) {
  LARA_NVTX("lara_kv_append_paged");
  if (!k_pages || !v_pages || !block_table || !seq_lens || !k_new || !v_new)
    return fail(LARA_ERR_STREAM_DEST, "null pointer");
  int page_log2 = 0;
  int rc = check_paged(page_size, pages_per_seq, num_pages, &page_log2);
  if (rc) return rc;
  if (batch < 1 || n_kv_heads < 1 || head_dim < 8 || head_dim % 8 || n_new < 0)
    return fail(LARA_ERR_BAD_CFG, "bad append geometry");
  if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || !aligned(k_new, 16) || !aligned(v_new, 16))
    return fail(LARA_ERR_STREAM_DEST, "pages and new rows must be 16-byte aligned");
  int* status = workspace ? static_cast<int*>(workspace) : nullptr;
  cudaError_t e = lara::kv_append_paged_launch(k_pages, v_pages, block_table, seq_lens, k_new, v_new, batch,
                                               n_kv_heads, head_dim, page_log2, pages_per_seq, num_pages, n_new,
                                               status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged append launch");
  return LARA_OK;
}

int lara_pack_bf16(const float* src, uint16_t* dst, size_t n, void* stream) {
  if (n == 0) return LARA_OK;
  if (!src || !dst) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (!aligned(src, 16) || !aligned(dst, 8)) return fail(LARA_ERR_STREAM_DEST, "src 16-byte, dst 8-byte alignment");
  cudaError_t e = lara::pack_bf16_launch(src, dst, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pack launch");
  return LARA_OK;
}

size_t lara_prefill_workspace_bytes(int batch, int n_new, int n_q_heads, int n_kv_heads, int head_dim,
                                    int max_seq_len) {
  if (batch < 1 || n_new < 1 || (long long)batch * n_new > 65535) return 0;
  if (check_geometry(batch * n_new, n_q_heads, n_kv_heads, head_dim, max_seq_len) != LARA_OK) return 0;
  int ns = 0, ch = 0;
  return prefill_ws_bytes(batch, n_new, n_q_heads, n_kv_heads, head_dim, max_seq_len, &ns, &ch);
}

int lara_gqa_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* cached_lens,
                     uint16_t* o, int batch, int n_new, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len,
                     int causal, float scale, void* workspace, size_t workspace_bytes, void* stream) {
  LARA_NVTX("lara_gqa_prefill");
  return prefill_common(q, k_cache, v_cache, cached_lens, o, batch, n_new, n_q_heads, n_kv_heads, head_dim,
                        max_seq_len, causal, scale, workspace, workspace_bytes, stream);
}

size_t lara_dense_workspace_bytes(int n_q_heads, int n_kv_heads, int head_dim, int seq_len) {
  if (check_geometry(seq_len, n_q_heads, n_kv_heads, head_dim, seq_len) != LARA_OK) return 0;
  int ns = 0, ch = 0;
  return dense_ws_bytes(n_q_heads, n_kv_heads, head_dim, seq_len, &ns, &ch);
}

int lara_attention_dense(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int n_q_heads,
                         int n_kv_heads, int head_dim, int seq_len, int q_pos_base, int kv_pos_base, int causal,
                         float scale, void* workspace, size_t workspace_bytes, void* stream) {
  LARA_NVTX("lara_attention_dense");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(LARA_ERR_BAD_CFG, "scale must be positive and finite");
  return dense_common(q, k, v, o, n_q_heads, n_kv_heads, head_dim, seq_len, q_pos_base, kv_pos_base, causal, scale,
                      workspace, workspace_bytes, stream);
}

}  // extern "C"

// ===========================================================================
// context API
// ===========================================================================

struct lara_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev[5] = {};  // start, kernels begin, kernels end, end; [4] = prologue end (run_layer)
  int batch = 1, hq = 32, hkv = 8, d = 128, lmax = 512;
  int seq_len = 1, q_pos_base = 0, kv_pos_base = 0, causal = 1;
  int arithmetic = LARA_ARITH_IEEE;  // dense transactions: IEEE fp32 or board arithmetic
  uint16_t* k_cache = nullptr;
  uint16_t* v_cache = nullptr;
  int32_t* lens_dev = nullptr;
  int32_t* lens_prev_dev = nullptr;  // lengths before the last prefill append
  std::vector<int32_t> lens_host;
  uint16_t* pq = nullptr;  // prefill q/o [B][n][Hq][D]
  uint16_t* po = nullptr;
  size_t p_cap = 0;
  uint16_t* q_buf = nullptr;  // decode q / o [B][Hq][D]
  uint16_t* o_buf = nullptr;
  uint16_t* new_k = nullptr;  // append staging [B][Hkv][n][D]
  uint16_t* new_v = nullptr;
  size_t new_cap = 0;
  uint16_t* dq = nullptr;  // dense q/o [Hq][L][D], k/v [Hkv][L][D]
  uint16_t* dk = nullptr;
  uint16_t* dv = nullptr;
  uint16_t* dout = nullptr;
  int dense_cap = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* status_host = nullptr;  // pinned
  uint16_t* lx = nullptr;      // run_layer: x [L][hidden], w_qkv [hidden][(Hq+2Hkv)D], rms weight [hidden]
  uint16_t* lw = nullptr;
  uint16_t* lg = nullptr;
  size_t lx_cap = 0, lw_cap = 0, lg_cap = 0;
  void* lws = nullptr;          // prologue workspace (status word first)
  size_t lws_bytes = 0;
  uint64_t layer_prologue_ns = 0, layer_attention_ns = 0;
  int plan_split = 0, plan_chunk = 0;
  bool plan_valid = false;
  lara_perf perf{};
  bool have_perf = false;
  bool perf_pending = false;  // events of the last transaction not yet read
  bool async_pending = false; // lara_decode / lara_prefill issued, lara_sync not yet called
  cudaStream_t copy_in = nullptr;   // pipelined host-buffer prefill: host -> device copies
  cudaStream_t copy_out = nullptr;  // and device -> host copies
  std::vector<cudaEvent_t> seq_ev;  // two per sequence: inputs copied, output computed
};

namespace {

void ctx_free_cache(lara_ctx* c) {
  cudaFree(c->k_cache); cudaFree(c->v_cache); cudaFree(c->lens_dev); cudaFree(c->lens_prev_dev);
  cudaFree(c->pq); cudaFree(c->po);
  c->lens_prev_dev = nullptr; c->pq = c->po = nullptr; c->p_cap = 0;
  cudaFree(c->q_buf); cudaFree(c->o_buf); cudaFree(c->new_k); cudaFree(c->new_v);
  c->k_cache = c->v_cache = nullptr; c->lens_dev = nullptr;
  c->q_buf = c->o_buf = c->new_k = c->new_v = nullptr;
  c->new_cap = 0;
}

void ctx_free_dense(lara_ctx* c) {
  cudaFree(c->dq); cudaFree(c->dk); cudaFree(c->dv); cudaFree(c->dout);
  c->dq = c->dk = c->dv = c->dout = nullptr;
  c->dense_cap = 0;
}

int ctx_ensure_ws(lara_ctx* c, size_t need) {
  if (c->ws && c->ws_bytes >= need) return LARA_OK;
  if (c->ws) { LARA_CUDA(cudaStreamSynchronize(c->stream)); cudaFree(c->ws); c->ws = nullptr; c->ws_bytes = 0; }
  LARA_CUDA(cudaMalloc(&c->ws, need));
  c->ws_bytes = need;
  LARA_CUDA(cudaMemsetAsync(c->ws, 0, need, c->stream));
  return LARA_OK;
}

// Device address of page-locked host memory the GPU can address directly
// (cudaHostAlloc / cudaHostRegister memory under unified addressing), or
// nullptr for pageable memory.  Kernels read such inputs and write such
// outputs over the interconnect themselves, so no staging copy is needed.
const void* mapped_host_ptr(const void* p, size_t align) {
  if (!aligned(p, align)) return nullptr;
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return (at.type == cudaMemoryTypeHost && at.devicePointer) ? at.devicePointer : nullptr;
}

cudaMemcpyKind in_kind(int on_device) { return on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice; }
cudaMemcpyKind out_kind(int on_device) { return on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost; }

// Wait for the stream, then turn the device status word into a return code.
int ctx_finish(lara_ctx* c) {
  LARA_CUDA(cudaMemcpyAsync(c->status_host, c->ws, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  const int bits = *c->status_host;
  if (bits) {
    LARA_CUDA(cudaMemsetAsync(c->ws, 0, sizeof(int), c->stream));
    LARA_CUDA(cudaStreamSynchronize(c->stream));
    const int code = (bits & lara::kDevWaitTimeout) ? LARA_ERR_TIMEOUT : LARA_ERR_DEVICE;
    return fail(code, "device status 0x%x:%s", bits, describe_status(bits).c_str());
  }
  return LARA_OK;
}

// The device times of the last transaction are read from its events when
// lara_read_perf asks (the events stay recorded until the next transaction).
void ctx_record_perf(lara_ctx* c) {
  c->perf_pending = true;
  c->have_perf = true;
}

void ctx_resolve_perf(lara_ctx* c) {
  if (!c->perf_pending) return;
  float total = 0.f, mac = 0.f;
  cudaEventElapsedTime(&total, c->ev[0], c->ev[3]);
  cudaEventElapsedTime(&mac, c->ev[1], c->ev[2]);
  c->perf.cycles = (uint64_t)llround((double)total * 1e6);
  c->perf.mac_cycles = (uint64_t)llround((double)mac * 1e6);
  if (c->perf.mac_cycles > c->perf.cycles) c->perf.mac_cycles = c->perf.cycles;
  c->perf.stall_cycles = c->perf.cycles - c->perf.mac_cycles;
  c->perf.clock_mhz = 1000.0;
  c->perf_pending = false;
}

int ctx_alloc(lara_ctx* c) {
  ctx_free_cache(c);
  const size_t cache_elems = (size_t)c->batch * c->hkv * c->lmax * c->d;
  LARA_CUDA(cudaMalloc(&c->k_cache, cache_elems * 2));
  LARA_CUDA(cudaMalloc(&c->v_cache, cache_elems * 2));
  LARA_CUDA(cudaMalloc(&c->lens_dev, sizeof(int32_t) * c->batch));
  LARA_CUDA(cudaMalloc(&c->lens_prev_dev, sizeof(int32_t) * c->batch));
  LARA_CUDA(cudaMemsetAsync(c->lens_dev, 0, sizeof(int32_t) * c->batch, c->stream));
  LARA_CUDA(cudaMalloc(&c->q_buf, (size_t)c->batch * c->hq * c->d * 2));
  LARA_CUDA(cudaMalloc(&c->o_buf, (size_t)c->batch * c->hq * c->d * 2));
  c->lens_host.assign(c->batch, 0);
  c->plan_valid = false;
  int ns = 0, ch = 0;
  lara::decode_plan(c->batch, c->hkv, c->hq, c->d, c->lmax, nullptr, &ns, &ch);
  int rc = ctx_ensure_ws(c, lara::decode_workspace_layout(c->batch, c->hq, c->hkv, c->d, ns).total);
  if (rc) return rc;
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  return LARA_OK;
}

int ctx_check(lara_ctx* c) {
  if (!c) return fail(LARA_ERR_BUSY_START, "attention accelerator context is closed");
  return LARA_OK;
}

// The copy streams and per-sequence events of the pipelined host-buffer
// prefill, created on first use.
int ctx_pipeline_ready(lara_ctx* c, int nseq) {
  if (!c->copy_in) LARA_CUDA(cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking));
  if (!c->copy_out) LARA_CUDA(cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking));
  while ((int)c->seq_ev.size() < 2 * nseq) {
    cudaEvent_t ev = nullptr;
    LARA_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    c->seq_ev.push_back(ev);
  }
  return LARA_OK;
}

// lara_run_prefill_chunk on host buffers, pipelined by sequence: sequence b's
// rows of q, k_new and v_new are contiguous (batch is the outer dimension), so
// its copies in run on copy_in while the main stream appends and attends
// sequence b - 1 and copy_out returns the output of the sequence before.  Each
// tensor-core prefill tile belongs to one (sequence, head), so the per-sequence
// launches write the same words as one launch over the batch.
int prefill_chunk_pipelined_issue(lara_ctx* c, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                                  uint16_t* o, int n_new, int causal);

int prefill_chunk_pipelined(lara_ctx* c, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                            uint16_t* o, int n_new, int causal) {
  int rc = ctx_pipeline_ready(c, c->batch);
  if (rc) return rc;
  rc = prefill_chunk_pipelined_issue(c, q, k_new, v_new, o, n_new, causal);
  if (rc) {
    // a failed issue may leave copies in flight on the caller's buffers: drain
    // every stream before returning the error
    cudaStreamSynchronize(c->copy_in);
    cudaStreamSynchronize(c->stream);
    cudaStreamSynchronize(c->copy_out);
    return rc;
  }
  for (auto& l : c->lens_host) l += n_new;
  c->plan_valid = false;
  rc = ctx_finish(c);
  if (rc) return rc;
  ctx_record_perf(c);
  return LARA_OK;
}

int prefill_chunk_pipelined_issue(lara_ctx* c, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                                  uint16_t* o, int n_new, int causal) {
  int rc = LARA_OK;
  const size_t q_seq = (size_t)n_new * c->hq * c->d;     // elements of one sequence's q (and o)
  const size_t kv_seq = (size_t)c->hkv * n_new * c->d;   // of its k_new (and v_new)
  const size_t cache_seq = (size_t)c->hkv * c->lmax * c->d;
  if (c->new_cap < kv_seq * c->batch * 2) {
    cudaFree(c->new_k); cudaFree(c->new_v);
    c->new_k = c->new_v = nullptr; c->new_cap = 0;
    LARA_CUDA(cudaMalloc(&c->new_k, kv_seq * c->batch * 2));
    LARA_CUDA(cudaMalloc(&c->new_v, kv_seq * c->batch * 2));
    c->new_cap = kv_seq * c->batch * 2;
  }
  cudaEvent_t* in_ev = c->seq_ev.data();
  cudaEvent_t* out_ev = in_ev + c->batch;
  LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
  LARA_CUDA(cudaMemcpyAsync(c->lens_prev_dev, c->lens_dev, sizeof(int32_t) * c->batch, cudaMemcpyDeviceToDevice,
                            c->stream));
  LARA_CUDA(cudaStreamWaitEvent(c->copy_in, c->ev[0], 0));
  for (int b = 0; b < c->batch; ++b) {
    LARA_CUDA(cudaMemcpyAsync(c->pq + b * q_seq, q + b * q_seq, q_seq * 2, cudaMemcpyHostToDevice, c->copy_in));
    LARA_CUDA(cudaMemcpyAsync(c->new_k + b * kv_seq, k_new + b * kv_seq, kv_seq * 2, cudaMemcpyHostToDevice,
                              c->copy_in));
    LARA_CUDA(cudaMemcpyAsync(c->new_v + b * kv_seq, v_new + b * kv_seq, kv_seq * 2, cudaMemcpyHostToDevice,
                              c->copy_in));
    LARA_CUDA(cudaEventRecord(in_ev[b], c->copy_in));
  }
  const float scale = 1.0f / std::sqrt((float)c->d);
  for (int b = 0; b < c->batch; ++b) {
    LARA_CUDA(cudaStreamWaitEvent(c->stream, in_ev[b], 0));
    if (b == 0) LARA_CUDA(cudaEventRecord(c->ev[1], c->stream));
    cudaError_t e = lara::kv_append_launch(c->k_cache + b * cache_seq, c->v_cache + b * cache_seq, c->lens_dev + b,
                                           c->new_k + b * kv_seq, c->new_v + b * kv_seq, 1, c->hkv, c->d, c->lmax,
                                           n_new, static_cast<int*>(c->ws), c->stream);
    if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
    rc = prefill_common(c->pq + b * q_seq, c->k_cache + b * cache_seq, c->v_cache + b * cache_seq,
                        c->lens_prev_dev + b, c->po + b * q_seq, 1, n_new, c->hq, c->hkv, c->d, c->lmax, causal, scale,
                        c->ws, c->ws_bytes, c->stream);
    if (rc) return rc;
    LARA_CUDA(cudaEventRecord(out_ev[b], c->stream));
    LARA_CUDA(cudaStreamWaitEvent(c->copy_out, out_ev[b], 0));
    LARA_CUDA(cudaMemcpyAsync(o + b * q_seq, c->po + b * q_seq, q_seq * 2, cudaMemcpyDeviceToHost, c->copy_out));
  }
  LARA_CUDA(cudaEventRecord(c->ev[2], c->stream));
  // join: the main stream waits for the last copy out (in_ev[0] is free again:
  // its wait is already enqueued)
  LARA_CUDA(cudaEventRecord(in_ev[0], c->copy_out));
  LARA_CUDA(cudaStreamWaitEvent(c->stream, in_ev[0], 0));
  LARA_CUDA(cudaEventRecord(c->ev[3], c->stream));
  return rc;
}

}  // namespace

extern "C" {

int lara_create(int device, lara_ctx** out) {
  if (!out) return fail(LARA_ERR_STREAM_DEST, "null output pointer");
  *out = nullptr;
  int n = 0;
  LARA_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return fail(LARA_ERR_BAD_CFG, "device %d not present (%d devices)", device, n);
  DeviceGuard g(device);
  int major = 0, minor = 0;
  LARA_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  LARA_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0)
    return fail(LARA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, major,
                minor);
  lara_ctx* c = new lara_ctx();
  c->device = device;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  for (int i = 0; i < 5 && e == cudaSuccess; ++i) e = cudaEventCreate(&c->ev[i]);
  if (e == cudaSuccess) e = cudaMallocHost(&c->status_host, sizeof(int));
  if (e != cudaSuccess) {
    lara_destroy(c);
    return cuda_fail(e, "context creation");
  }
  int rc = ctx_alloc(c);
  if (rc) {
    lara_destroy(c);
    return rc;
  }
  *out = c;
  return LARA_OK;
}

int lara_destroy(lara_ctx* c) {
  if (!c) return LARA_OK;
  DeviceGuard g(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  ctx_free_cache(c);
  ctx_free_dense(c);
  cudaFree(c->ws);
  cudaFree(c->lx); cudaFree(c->lw); cudaFree(c->lg); cudaFree(c->lws);
  if (c->status_host) cudaFreeHost(c->status_host);
  for (auto& ev : c->ev)
    if (ev) cudaEventDestroy(ev);
  for (auto& ev : c->seq_ev) cudaEventDestroy(ev);
  if (c->copy_in) {
    cudaStreamSynchronize(c->copy_in);
    cudaStreamDestroy(c->copy_in);
  }
  if (c->copy_out) {
    cudaStreamSynchronize(c->copy_out);
    cudaStreamDestroy(c->copy_out);
  }
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return LARA_OK;
}

int lara_ctx_device(lara_ctx* c) { return c ? c->device : -1; }

int lara_set_arithmetic(lara_ctx* c, int mode) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (mode != LARA_ARITH_IEEE && mode != LARA_ARITH_BOARD) return fail(LARA_ERR_BAD_CFG, "unknown arithmetic mode");
  if (mode == LARA_ARITH_BOARD && c->d != 128)
    return fail(LARA_ERR_UNSUPPORTED, "board arithmetic is defined for head_dim 128 only");
  c->arithmetic = mode;
  return LARA_OK;
}

int lara_get_arithmetic(lara_ctx* c) { return c ? c->arithmetic : -1; }

int lara_configure_heads(lara_ctx* c, int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len) {
  int rc = ctx_check(c);
  if (rc) return rc;
  rc = check_geometry(batch, n_q_heads, n_kv_heads, head_dim, max_seq_len);
  if (rc) return rc;
  DeviceGuard g(c->device);
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  c->batch = batch; c->hq = n_q_heads; c->hkv = n_kv_heads; c->d = head_dim; c->lmax = max_seq_len;
  ctx_free_dense(c);
  return ctx_alloc(c);
}

int lara_configure(lara_ctx* c, int seq_len, int q_pos_base, int kv_pos_base, int causal) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (seq_len < 1 || seq_len > c->lmax)
    return fail(LARA_ERR_BAD_CFG, "seq_len must be in 1..%d, got %d", c->lmax, seq_len);
  if (q_pos_base < 0 || kv_pos_base < 0 || q_pos_base + seq_len > (1 << 16) || kv_pos_base + seq_len > (1 << 16))
    return fail(LARA_ERR_BAD_CFG, "absolute position base + seq_len exceeds 16-bit range");
  c->seq_len = seq_len; c->q_pos_base = q_pos_base; c->kv_pos_base = kv_pos_base; c->causal = causal ? 1 : 0;
  return LARA_OK;
}

int lara_kv_load(lara_ctx* c, const uint16_t* k, const uint16_t* v, const int32_t* lens, int src_len, int on_device) {
  LARA_NVTX("lara_kv_load");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!k || !v || !lens) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (src_len < 0 || src_len > c->lmax) return fail(LARA_ERR_STREAM_LEN, "src_len %d outside 0..%d", src_len, c->lmax);
  for (int b = 0; b < c->batch; ++b)
    if (lens[b] < 0 || lens[b] > src_len)
      return fail(LARA_ERR_STREAM_LEN, "lens[%d]=%d outside 0..%d", b, lens[b], src_len);
  DeviceGuard g(c->device);
  if (src_len > 0) {
    const size_t row = (size_t)c->d * 2;
    // [B*Hkv][src_len][D] -> [B*Hkv][lmax][D]: one strided 2-D copy per tensor.
    LARA_CUDA(cudaMemcpy2DAsync(c->k_cache, row * c->lmax, k, row * src_len, row * src_len,
                                (size_t)c->batch * c->hkv, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpy2DAsync(c->v_cache, row * c->lmax, v, row * src_len, row * src_len,
                                (size_t)c->batch * c->hkv, in_kind(on_device), c->stream));
  }
  c->lens_host.assign(lens, lens + c->batch);
  LARA_CUDA(cudaMemcpyAsync(c->lens_dev, c->lens_host.data(), sizeof(int32_t) * c->batch, cudaMemcpyHostToDevice,
                            c->stream));
  c->plan_valid = false;
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  return LARA_OK;
}

int lara_kv_append_ctx(lara_ctx* c, const uint16_t* k_new, const uint16_t* v_new, int n_new, int on_device) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!k_new || !v_new) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (n_new < 0) return fail(LARA_ERR_STREAM_LEN, "n_new must be >= 0");
  for (int b = 0; b < c->batch; ++b)
    if (c->lens_host[b] + n_new > c->lmax)
      return fail(LARA_ERR_STREAM_LEN, "append of %d tokens overflows sequence %d (len %d, capacity %d)", n_new, b,
                  c->lens_host[b], c->lmax);
  if (n_new == 0) return LARA_OK;
  DeviceGuard g(c->device);
  const size_t bytes = (size_t)c->batch * c->hkv * n_new * c->d * 2;
  const uint16_t* kd = k_new;
  const uint16_t* vd = v_new;
  if (!on_device || !aligned(k_new, 16) || !aligned(v_new, 16)) {
    if (c->new_cap < bytes) {
      cudaFree(c->new_k); cudaFree(c->new_v);
      c->new_k = c->new_v = nullptr; c->new_cap = 0;
      LARA_CUDA(cudaMalloc(&c->new_k, bytes));
      LARA_CUDA(cudaMalloc(&c->new_v, bytes));
      c->new_cap = bytes;
    }
    LARA_CUDA(cudaMemcpyAsync(c->new_k, k_new, bytes, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpyAsync(c->new_v, v_new, bytes, in_kind(on_device), c->stream));
    kd = c->new_k;
    vd = c->new_v;
  }
  cudaError_t e = lara::kv_append_launch(c->k_cache, c->v_cache, c->lens_dev, kd, vd, c->batch, c->hkv, c->d,
                                         c->lmax, n_new, static_cast<int*>(c->ws), c->stream);
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  for (auto& l : c->lens_host) l += n_new;
  c->plan_valid = false;
  return ctx_finish(c);
}

int lara_run_prefill_chunk(lara_ctx* c, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new, uint16_t* o,
                           int n_new, int causal, int on_device) {
  LARA_NVTX("lara_run_prefill_chunk");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!q || !k_new || !v_new || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (n_new < 1) return fail(LARA_ERR_STREAM_LEN, "n_new must be >= 1");
  for (int b = 0; b < c->batch; ++b)
    if (c->lens_host[b] + n_new > c->lmax)
      return fail(LARA_ERR_STREAM_LEN, "prefill of %d tokens overflows sequence %d (len %d, capacity %d)", n_new, b,
                  c->lens_host[b], c->lmax);
  DeviceGuard g(c->device);
  int ns = 0, ch = 0;
  const size_t need = prefill_ws_bytes(c->batch, n_new, c->hq, c->hkv, c->d, c->lmax, &ns, &ch);
  if (need == 0 || (long long)c->batch * n_new > 65535)
    return fail(LARA_ERR_BAD_CFG, "batch*n_new (%lld) exceeds 65535 query rows", (long long)c->batch * n_new);
  rc = ctx_ensure_ws(c, need);
  if (rc) return rc;
  const size_t qbytes = (size_t)c->batch * n_new * c->hq * c->d * 2;
  if (c->p_cap < qbytes) {
    cudaFree(c->pq); cudaFree(c->po);
    c->pq = c->po = nullptr; c->p_cap = 0;
    LARA_CUDA(cudaMalloc(&c->pq, qbytes));
    LARA_CUDA(cudaMalloc(&c->po, qbytes));
    c->p_cap = qbytes;
  }
  // host buffers on the tensor-core prefill: pipelined by sequence
  if (!on_device && c->batch > 1 && attn_path_override() != AttnPath::kStream &&
      lara::prefill_tc_supported(c->d, c->hq, c->hkv))
    return prefill_chunk_pipelined(c, q, k_new, v_new, o, n_new, causal);
  LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
  LARA_CUDA(cudaMemcpyAsync(c->lens_prev_dev, c->lens_dev, sizeof(int32_t) * c->batch, cudaMemcpyDeviceToDevice,
                            c->stream));
  const uint16_t* qd = q;
  if (!on_device || !aligned(q, 16)) {
    LARA_CUDA(cudaMemcpyAsync(c->pq, q, qbytes, in_kind(on_device), c->stream));
    qd = c->pq;
  }
  const size_t kvbytes = (size_t)c->batch * c->hkv * n_new * c->d * 2;
  const uint16_t* kd = k_new;
  const uint16_t* vd = v_new;
  if (!on_device || !aligned(k_new, 16) || !aligned(v_new, 16)) {
    if (c->new_cap < kvbytes) {
      cudaFree(c->new_k); cudaFree(c->new_v);
      c->new_k = c->new_v = nullptr; c->new_cap = 0;
      LARA_CUDA(cudaMalloc(&c->new_k, kvbytes));
      LARA_CUDA(cudaMalloc(&c->new_v, kvbytes));
      c->new_cap = kvbytes;
    }
    LARA_CUDA(cudaMemcpyAsync(c->new_k, k_new, kvbytes, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpyAsync(c->new_v, v_new, kvbytes, in_kind(on_device), c->stream));
    kd = c->new_k;
    vd = c->new_v;
  }
  uint16_t* od = (on_device && aligned(o, 4)) ? o : c->po;
  LARA_CUDA(cudaEventRecord(c->ev[1], c->stream));
  cudaError_t e = lara::kv_append_launch(c->k_cache, c->v_cache, c->lens_dev, kd, vd, c->batch, c->hkv, c->d,
                                         c->lmax, n_new, static_cast<int*>(c->ws), c->stream);
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  rc = prefill_common(qd, c->k_cache, c->v_cache, c->lens_prev_dev, od, c->batch, n_new, c->hq, c->hkv, c->d,
                      c->lmax, causal, 1.0f / std::sqrt((float)c->d), c->ws, c->ws_bytes, c->stream);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], c->stream));
  if (od != o) LARA_CUDA(cudaMemcpyAsync(o, od, qbytes, out_kind(on_device), c->stream));
  LARA_CUDA(cudaEventRecord(c->ev[3], c->stream));
  for (auto& l : c->lens_host) l += n_new;
  c->plan_valid = false;
  rc = ctx_finish(c);
  if (rc) return rc;
  ctx_record_perf(c);
  return LARA_OK;
}

int lara_kv_read(lara_ctx* c, uint16_t* k, uint16_t* v, int32_t* lens_out, int dst_len, int on_device) {
  LARA_NVTX("lara_kv_read");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!k || !v || !lens_out) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (dst_len < 1 || dst_len > c->lmax) return fail(LARA_ERR_BAD_CFG, "dst_len must be in [1, max_seq_len]");
  DeviceGuard g(c->device);
  const size_t row = (size_t)c->d * 2;
  const size_t rows = (size_t)c->batch * c->hkv;
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  // each (sequence, kv head) row: its first dst_len tokens
  LARA_CUDA(cudaMemcpy2DAsync(k, (size_t)dst_len * row, c->k_cache, (size_t)c->lmax * row, (size_t)dst_len * row,
                              rows, kind, c->stream));
  LARA_CUDA(cudaMemcpy2DAsync(v, (size_t)dst_len * row, c->v_cache, (size_t)c->lmax * row, (size_t)dst_len * row,
                              rows, kind, c->stream));
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  for (int b = 0; b < c->batch; ++b) lens_out[b] = c->lens_host[b];
  return LARA_OK;
}

int lara_kv_truncate(lara_ctx* c, const int32_t* lens) {
  LARA_NVTX("lara_kv_truncate");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!lens) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  for (int b = 0; b < c->batch; ++b)
    if (lens[b] < 0 || lens[b] > c->lens_host[b])
      return fail(LARA_ERR_STREAM_LEN, "lens[%d]=%d outside 0..%d (a truncation only shortens)", b, lens[b],
                  c->lens_host[b]);
  DeviceGuard g(c->device);
  c->lens_host.assign(lens, lens + c->batch);
  LARA_CUDA(cudaMemcpyAsync(c->lens_dev, c->lens_host.data(), sizeof(int32_t) * c->batch, cudaMemcpyHostToDevice,
                            c->stream));
  c->plan_valid = false;
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  return LARA_OK;
}

int lara_get_seq_lens(lara_ctx* c, int32_t* lens_out) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!lens_out) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  std::memcpy(lens_out, c->lens_host.data(), sizeof(int32_t) * c->batch);
  return LARA_OK;
}

int lara_run_query(lara_ctx* c, const uint16_t* q, uint16_t* o, int on_device) {
  LARA_NVTX("lara_run_query");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!q || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  DeviceGuard g(c->device);
  if (!c->plan_valid) {
    c->plan_split = 0;
    c->plan_chunk = 0;
    lara::decode_plan(c->batch, c->hkv, c->hq, c->d, c->lmax, c->lens_host.data(), &c->plan_split, &c->plan_chunk);
    rc = ctx_ensure_ws(c, lara::decode_workspace_layout(c->batch, c->hq, c->hkv, c->d, c->plan_split).total);
    if (rc) return rc;
    c->plan_valid = true;
  }
  const size_t qbytes = (size_t)c->batch * c->hq * c->d * 2;
  LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
  // Pinned host q / o are read and written by the kernel in place; other
  // host memory is staged through device buffers.
  const uint16_t* qd = q;
  uint16_t* od = o;
  if (!on_device) {
    qd = static_cast<const uint16_t*>(mapped_host_ptr(q, 16));
    od = static_cast<uint16_t*>(const_cast<void*>(mapped_host_ptr(o, 4)));
  }
  if (!qd || !aligned(qd, 16)) {
    LARA_CUDA(cudaMemcpyAsync(c->q_buf, q, qbytes, in_kind(on_device), c->stream));
    qd = c->q_buf;
  }
  if (!od || !aligned(od, 4)) od = c->o_buf;
  LARA_CUDA(cudaEventRecord(c->ev[1], c->stream));
  rc = decode_common(qd, c->k_cache, c->v_cache, c->lens_dev, od, nullptr, nullptr, c->batch, c->hq, c->hkv, c->d,
                     c->lmax, 1.0f / std::sqrt((float)c->d), c->plan_split, c->plan_chunk, c->ws, c->ws_bytes,
                     c->stream);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], c->stream));
  if (od == c->o_buf) LARA_CUDA(cudaMemcpyAsync(o, od, qbytes, out_kind(on_device), c->stream));
  LARA_CUDA(cudaEventRecord(c->ev[3], c->stream));
  rc = ctx_finish(c);
  if (rc) return rc;
  ctx_record_perf(c);
  return LARA_OK;
}

int lara_run_attention(lara_ctx* c, const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                       int on_device) {
  LARA_NVTX("lara_run_attention");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!q || !k || !v || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  DeviceGuard g(c->device);
  const int L = c->seq_len;
  if (c->dense_cap < L) {
    ctx_free_dense(c);
    LARA_CUDA(cudaMalloc(&c->dq, (size_t)c->hq * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dout, (size_t)c->hq * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dk, (size_t)c->hkv * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dv, (size_t)c->hkv * L * c->d * 2));
    c->dense_cap = L;
  }
  const bool board = c->arithmetic == LARA_ARITH_BOARD;
  if (!board) {
    int ns = 0, ch = 0;
    rc = ctx_ensure_ws(c, dense_ws_bytes(c->hq, c->hkv, c->d, L, &ns, &ch));
    if (rc) return rc;
  }
  const size_t qb = (size_t)c->hq * L * c->d * 2, kb = (size_t)c->hkv * L * c->d * 2;
  LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
  const uint16_t *qd = q, *kd = k, *vd = v;
  if (!on_device || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16)) {
    LARA_CUDA(cudaMemcpyAsync(c->dq, q, qb, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpyAsync(c->dk, k, kb, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpyAsync(c->dv, v, kb, in_kind(on_device), c->stream));
    qd = c->dq; kd = c->dk; vd = c->dv;
  }
  uint16_t* od = (on_device && aligned(o, 4)) ? o : c->dout;
  LARA_CUDA(cudaEventRecord(c->ev[1], c->stream));
  if (board)
    rc = lara_attention_dense_board(qd, kd, vd, od, c->hq, c->hkv, c->d, L, c->causal, c->q_pos_base,
                                    c->kv_pos_base, c->stream);
  else
    rc = dense_common(qd, kd, vd, od, c->hq, c->hkv, c->d, L, c->q_pos_base, c->kv_pos_base, c->causal,
                      1.0f / std::sqrt((float)c->d), c->ws, c->ws_bytes, c->stream);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], c->stream));
  if (od != o) LARA_CUDA(cudaMemcpyAsync(o, od, qb, out_kind(on_device), c->stream));
  LARA_CUDA(cudaEventRecord(c->ev[3], c->stream));
  rc = ctx_finish(c);
  if (rc) return rc;
  ctx_record_perf(c);
  return LARA_OK;
}

namespace {
// grow-only device buffer
int ensure_buf(void** p, size_t* cap, size_t need) {
  if (*cap >= need) return LARA_OK;
  cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  const cudaError_t e = cudaMalloc(p, need);
  if (e != cudaSuccess) return lara::set_last_error(LARA_ERR_CUDA, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  *cap = need;
  return LARA_OK;
}
}  // namespace

int lara_run_layer(lara_ctx* c, const uint16_t* x, const uint16_t* w_qkv, const uint16_t* rms_weight, int hidden,
                   uint16_t* o, float rms_eps, float rope_base, int on_device) {
  LARA_NVTX("lara_run_layer");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!x || !w_qkv || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (hidden < 64 || hidden % 64) return fail(LARA_ERR_BAD_CFG, "hidden must be a positive multiple of 64");
  if (c->d != 128) return fail(LARA_ERR_UNSUPPORTED, "run_layer's fused projection is built for head_dim 128");
  DeviceGuard g(c->device);
  const int L = c->seq_len;
  const size_t n_total = (size_t)(c->hq + 2 * c->hkv) * c->d;
  if (c->dense_cap < L) {
    ctx_free_dense(c);
    LARA_CUDA(cudaMalloc(&c->dq, (size_t)c->hq * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dout, (size_t)c->hq * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dk, (size_t)c->hkv * L * c->d * 2));
    LARA_CUDA(cudaMalloc(&c->dv, (size_t)c->hkv * L * c->d * 2));
    c->dense_cap = L;
  }
  const bool board = c->arithmetic == LARA_ARITH_BOARD;
  if (!board) {
    int ns = 0, ch = 0;
    rc = ctx_ensure_ws(c, dense_ws_bytes(c->hq, c->hkv, c->d, L, &ns, &ch));
    if (rc) return rc;
  }
  const size_t xb = (size_t)L * hidden * 2, wb = (size_t)hidden * n_total * 2, gb = (size_t)hidden * 2;
  const size_t need_ws = lara_layer_prologue_workspace_bytes(1, L, hidden);
  if (c->lws_bytes < need_ws) {
    rc = ensure_buf(&c->lws, &c->lws_bytes, need_ws);
    if (rc) return rc;
    LARA_CUDA(cudaMemsetAsync(c->lws, 0, c->lws_bytes, c->stream));
  }
  const bool dev_ok = on_device && aligned(x, 16) && aligned(w_qkv, 16) && (!rms_weight || aligned(rms_weight, 16));
  if (!dev_ok) {
    rc = ensure_buf(reinterpret_cast<void**>(&c->lx), &c->lx_cap, xb);
    if (!rc) rc = ensure_buf(reinterpret_cast<void**>(&c->lw), &c->lw_cap, wb);
    if (!rc && rms_weight) rc = ensure_buf(reinterpret_cast<void**>(&c->lg), &c->lg_cap, gb);
    if (rc) return rc;
  }
  LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
  const uint16_t *xd = x, *wd = w_qkv, *gd = rms_weight;
  if (!dev_ok) {
    LARA_CUDA(cudaMemcpyAsync(c->lx, x, xb, in_kind(on_device), c->stream));
    LARA_CUDA(cudaMemcpyAsync(c->lw, w_qkv, wb, in_kind(on_device), c->stream));
    if (rms_weight) LARA_CUDA(cudaMemcpyAsync(c->lg, rms_weight, gb, in_kind(on_device), c->stream));
    xd = c->lx;
    wd = c->lw;
    gd = rms_weight ? c->lg : nullptr;
  }
  LARA_CUDA(cudaEventRecord(c->ev[1], c->stream));
  rc = lara_layer_prologue(xd, gd, wd, c->dq, c->dk, c->dv, 1, L, hidden, c->hq, c->hkv, c->d, c->q_pos_base,
                           c->kv_pos_base, rms_eps, rope_base, c->lws, c->lws_bytes, c->stream);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[4], c->stream));
  uint16_t* od = (on_device && aligned(o, 4)) ? o : c->dout;
  if (board)
    rc = lara_attention_dense_board(c->dq, c->dk, c->dv, od, c->hq, c->hkv, c->d, L, c->causal, c->q_pos_base,
                                    c->kv_pos_base, c->stream);
  else
    rc = dense_common(c->dq, c->dk, c->dv, od, c->hq, c->hkv, c->d, L, c->q_pos_base, c->kv_pos_base, c->causal,
                      1.0f / std::sqrt((float)c->d), c->ws, c->ws_bytes, c->stream);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], c->stream));
  if (od != o) LARA_CUDA(cudaMemcpyAsync(o, od, (size_t)c->hq * L * c->d * 2, out_kind(on_device), c->stream));
  LARA_CUDA(cudaEventRecord(c->ev[3], c->stream));
  // prologue status word, then the attention workspace's
  LARA_CUDA(cudaMemcpyAsync(c->status_host, c->lws, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  LARA_CUDA(cudaStreamSynchronize(c->stream));
  if (*c->status_host) {
    const int bits = *c->status_host;
    LARA_CUDA(cudaMemsetAsync(c->lws, 0, sizeof(int), c->stream));
    LARA_CUDA(cudaStreamSynchronize(c->stream));
    return fail((bits & lara::kDevWaitTimeout) ? LARA_ERR_TIMEOUT : LARA_ERR_DEVICE, "prologue device status 0x%x",
                bits);
  }
  rc = ctx_finish(c);
  if (rc) return rc;
  ctx_record_perf(c);
  float pro = 0.f, att = 0.f;
  cudaEventElapsedTime(&pro, c->ev[1], c->ev[4]);
  cudaEventElapsedTime(&att, c->ev[4], c->ev[2]);
  c->layer_prologue_ns = (uint64_t)llround((double)pro * 1e6);
  c->layer_attention_ns = (uint64_t)llround((double)att * 1e6);
  return LARA_OK;
}

int lara_read_layer_perf(lara_ctx* c, uint64_t* prologue_ns, uint64_t* attention_ns) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!prologue_ns || !attention_ns) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  *prologue_ns = c->layer_prologue_ns;
  *attention_ns = c->layer_attention_ns;
  return LARA_OK;
}

int lara_ctx_selftest_timeout(lara_ctx* c, int limit_us) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (limit_us < 1 || limit_us > 2000000) return fail(LARA_ERR_BAD_CFG, "limit_us must be in [1, 2e6]");
  DeviceGuard g(c->device);
  LARA_CUDA(lara::selftest_wait_launch(static_cast<int*>(c->ws), limit_us, c->stream));
  return ctx_finish(c);  // LARA_ERR_TIMEOUT, and the status word is cleared for the next call
}

int lara_read_perf(lara_ctx* c, lara_perf* out) {
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!out) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (c->have_perf) {
    DeviceGuard g(c->device);
    ctx_resolve_perf(c);
    *out = c->perf;
  } else {
    *out = lara_perf{0, 0, 0, 1000.0};
  }
  return LARA_OK;
}

int lara_sync(lara_ctx* c, int timeout_ms) {
  int rc = ctx_check(c);
  if (rc) return rc;
  DeviceGuard g(c->device);
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    // the last asynchronous call (lara_decode / lara_prefill) ends with ev[3]
    // on its stream; synchronous calls leave both already complete
    cudaError_t e = c->async_pending ? cudaEventQuery(c->ev[3]) : cudaStreamQuery(c->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(e, "stream query");
    if (timeout_ms >= 0 &&
        std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return fail(LARA_ERR_TIMEOUT, "attention accelerator timed out after %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  c->async_pending = false;
  return ctx_finish(c);  // device status word of the work just completed
}

int lara_decode(lara_ctx* c, const uint16_t* q, uint16_t* o, int splits, void* stream) {
  LARA_NVTX("lara_decode");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!q || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  DeviceGuard g(c->device);
  const cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  int ns = 0, ch = 0;
  if (splits > 0) {
    const int tile = lara::decode_chunk_granule(c->d, c->hq / c->hkv);
    ch = ((c->lmax + splits - 1) / splits + tile - 1) / tile * tile;
    ns = (c->lmax + ch - 1) / ch;
  } else {
    if (!c->plan_valid) {
      c->plan_split = 0;
      c->plan_chunk = 0;
      lara::decode_plan(c->batch, c->hkv, c->hq, c->d, c->lmax, c->lens_host.data(), &c->plan_split,
                        &c->plan_chunk);
      c->plan_valid = true;
    }
    ns = c->plan_split;
    ch = c->plan_chunk;
  }
  rc = ctx_ensure_ws(c, lara::decode_workspace_layout(c->batch, c->hq, c->hkv, c->d, ns).total);
  if (rc) return rc;
  // the context's buffers are ordered on its stream; make the caller's stream wait for them
  if (st != c->stream) {
    LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
    LARA_CUDA(cudaStreamWaitEvent(st, c->ev[0], 0));
  }
  LARA_CUDA(cudaEventRecord(c->ev[0], st));
  LARA_CUDA(cudaEventRecord(c->ev[1], st));
  rc = decode_common(q, c->k_cache, c->v_cache, c->lens_dev, o, nullptr, nullptr, c->batch, c->hq, c->hkv, c->d,
                     c->lmax, 1.0f / std::sqrt((float)c->d), ns, ch, c->ws, c->ws_bytes, st);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], st));
  LARA_CUDA(cudaEventRecord(c->ev[3], st));
  if (st != c->stream) LARA_CUDA(cudaStreamWaitEvent(c->stream, c->ev[3], 0));
  c->async_pending = true;
  ctx_record_perf(c);
  return LARA_OK;
}

int lara_prefill(lara_ctx* c, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new, uint16_t* o,
                 int n_new, int causal, void* stream) {
  LARA_NVTX("lara_prefill");
  int rc = ctx_check(c);
  if (rc) return rc;
  if (!q || !k_new || !v_new || !o) return fail(LARA_ERR_STREAM_DEST, "null pointer");
  if (!aligned(q, 16) || !aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(o, 4))
    return fail(LARA_ERR_STREAM_DEST, "q/k/v must be 16-byte aligned device buffers, o 4-byte");
  if (n_new < 1) return fail(LARA_ERR_STREAM_LEN, "n_new must be >= 1");
  for (int b = 0; b < c->batch; ++b)
    if (c->lens_host[b] + n_new > c->lmax)
      return fail(LARA_ERR_STREAM_LEN, "prefill of %d tokens overflows sequence %d (len %d, capacity %d)", n_new, b,
                  c->lens_host[b], c->lmax);
  DeviceGuard g(c->device);
  const cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  int ns = 0, ch = 0;
  const size_t need = prefill_ws_bytes(c->batch, n_new, c->hq, c->hkv, c->d, c->lmax, &ns, &ch);
  if (need == 0 || (long long)c->batch * n_new > 65535)
    return fail(LARA_ERR_BAD_CFG, "batch*n_new (%lld) exceeds 65535 query rows", (long long)c->batch * n_new);
  rc = ctx_ensure_ws(c, need);
  if (rc) return rc;
  if (st != c->stream) {
    LARA_CUDA(cudaEventRecord(c->ev[0], c->stream));
    LARA_CUDA(cudaStreamWaitEvent(st, c->ev[0], 0));
  }
  LARA_CUDA(cudaEventRecord(c->ev[0], st));
  LARA_CUDA(cudaMemcpyAsync(c->lens_prev_dev, c->lens_dev, sizeof(int32_t) * c->batch, cudaMemcpyDeviceToDevice,
                            st));
  LARA_CUDA(cudaEventRecord(c->ev[1], st));
  cudaError_t e = lara::kv_append_launch(c->k_cache, c->v_cache, c->lens_dev, k_new, v_new, c->batch, c->hkv, c->d,
                                         c->lmax, n_new, static_cast<int*>(c->ws), st);
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  rc = prefill_common(q, c->k_cache, c->v_cache, c->lens_prev_dev, o, c->batch, n_new, c->hq, c->hkv, c->d, c->lmax,
                      causal, 1.0f / std::sqrt((float)c->d), c->ws, c->ws_bytes, st);
  if (rc) return rc;
  LARA_CUDA(cudaEventRecord(c->ev[2], st));
  LARA_CUDA(cudaEventRecord(c->ev[3], st));
  if (st != c->stream) LARA_CUDA(cudaStreamWaitEvent(c->stream, c->ev[3], 0));
  for (auto& l : c->lens_host) l += n_new;
  c->plan_valid = false;
  c->async_pending = true;
  ctx_record_perf(c);
  return LARA_OK;
}

}  // extern "C"
