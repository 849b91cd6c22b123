// Internal (C++) interfaces shared by the CUDA translation units of
// liblara_b200.so.  Nothing here is part of the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

// Named NVTX range around a C-ABI entry point, so profiler timelines show the
// library's calls (NVTX v3 is header-only; without an attached tool a range
// costs a null check).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};
#define LARA_NVTX(name) NvtxRange lara_nvtx_range_(name)

namespace lara {

// Device status word bits (atomicOr'd into the first word of a workspace).
enum DeviceStatus : int {
  kDevOk = 0,
  kDevWaitTimeout = 1 << 0,    // a bounded mbarrier wait gave up
  kDevBadLength = 1 << 1,      // a sequence length was outside [0, max_seq_len]
  kDevAppendOverflow = 1 << 2, // an appended row would pass max_seq_len
  kDevBadPage = 1 << 3,        // a block-table entry was outside [0, num_pages)
};

// One decode launch: queries of `batch` sequences (or of `batch` query rows
// that share one K/V stream, for the dense transaction) against a bf16 KV
// cache.  All strides are in elements; rows of K/V are `head_dim` contiguous
// bf16 words, tokens of one (sequence, kv head) are contiguous.
struct DecodeParams {
  const uint16_t* q;   // q[b * q_sb + h * q_sh + d]
  long long q_sb, q_sh;
  const uint16_t* k;   // k[b * kv_sb + kvh * kv_sh + tok * D + d]
  const uint16_t* v;
  long long kv_sb, kv_sh;
  uint16_t* o;         // o[b * o_sb + h * o_sh + d] (bf16), unused in partial mode
  long long o_sb, o_sh;
  // Rows: blockIdx.z = r is a query row; its K/V stream is sequence
  // r / rows_per_seq, and it sees the first
  //   clamp((lens ? lens[r / rows_per_seq] : 0) + len_c0 + len_c1 * (r % rows_per_seq), 0, max_seq_len)
  // tokens.  Decode: rows_per_seq = 1, c0 = c1 = 0.  Dense transaction: one
  // shared K/V (kv_sb = 0), rows_per_seq = L, c0/c1 from the causal rule.
  // Chunked prefill: rows_per_seq = n new tokens, lens = cached lengths.
  const int32_t* lens;
  int len_c0, len_c1;
  int rows_per_seq;
  int max_seq_len;     // tokens allocated per (sequence, kv head) row
  int batch;           // query rows (grid.z)
  int n_q_heads, n_kv_heads, head_dim;
  float scale_log2;    // softmax scale * log2(e)
  int chunk;           // tokens per CTA (multiple of the kernel's tile)
  int chunk0;          // tokens of split 0 (0: = chunk); splits s >= 1 start at chunk0 + (s-1)*chunk
  int nsplit;          // grid.z; partial slots per row in the workspace
  // workspace (see decode_workspace_layout)
  int* status;
  int* counters;       // [batch * n_kv_heads] (rows), zero between launches
  float* part_ml;      // [batch * n_q_heads * nsplit * 2]
  float* part_acc;     // [batch * n_q_heads * nsplit * head_dim]
  // partial-output mode (split-KV across GPUs): when out_acc != nullptr the
  // kernel writes unnormalised (m (log2 domain), l, acc[D]) per (b, h) row
  // instead of bf16 output.
  float* out_ml;       // [batch * n_q_heads * 2]
  float* out_acc;      // [batch * n_q_heads * head_dim]
  // Paged cache (when block_table != nullptr): k/v are page pools
  // [num_pages][n_kv_heads][1 << page_log2][head_dim]; token t of sequence s
  // lives in page block_table[s * pages_per_seq + (t >> page_log2)] at row
  // t & ((1 << page_log2) - 1); kv_sb / kv_sh are unused.
  const int32_t* block_table;
  int page_log2, pages_per_seq, num_pages;
  // Set by decode_launch: prefetch the CTA's first ring tiles into L2 before
  // the dependency wait (contiguous decode rows only).
  int l2_prefetch;
};

struct WorkspaceLayout {
  size_t status_off, counters_off, ml_off, acc_off, total;
};

WorkspaceLayout decode_workspace_layout(int batch, int n_q_heads, int n_kv_heads, int head_dim, int nsplit);

// Chooses the split count for a (batch, kv heads, max tokens) workload on the
// current device.  `lens_host` (optional, [batch]) are the actual lengths; a
// ragged batch is planned by token count instead of by waves.  Returns the
// number of splits (grid.z) and the chunk in tokens; when nsplit*chunk < max_tokens
// split 0 takes the rest (decode_first_chunk).
void decode_plan(int batch, int n_kv_heads, int n_q_heads, int head_dim, int max_tokens, const int32_t* lens_host,
                 int* nsplit, int* chunk);

// Tile size (tokens per pipeline stage) of the compiled kernel for a head
// geometry, or 0 when no kernel is compiled for it.
int decode_tile_tokens(int head_dim, int group);

// Granule of a caller-chosen chunk: the CUDA-core tile, or 128 tokens for a
// geometry only the tensor-core kernel runs (group 16); 0 = unsupported.
int decode_chunk_granule(int head_dim, int group);

// Tokens of the first split for a (nsplit, chunk) plan over `units` (query
// row, kv head) pairs, or 0 for equal splits.  A plan whose splits do not
// cover max_seq_len (nsplit * chunk < max_seq_len) gives split 0 the rest,
// max_seq_len - (nsplit - 1) * chunk rounded up to 128 tokens: long
// first items, then short ones that even out the tail of the tensor-core
// decode's list schedule.  Otherwise, with two splits the first
// covers 7/8 of the span: all first chunks launch before any second chunk, so
// the short second chunks fill the last wave (measured on B200: +1.2 to
// +3.8 % GB/s on 64 x 4096, 64 x 8192 and 96 x 4096 decodes).  It applies
// only when the first chunks alone occupy every SM: with fewer units, SMs
// holding a long first chunk stream it alone while others finish early (8 x
// 4096 ran at 0.26-0.35 of HBM, 16 x 4096 at 0.50-0.66).
int decode_first_chunk(int nsplit, int chunk, int group, int head_dim, long long units, int max_seq_len);

cudaError_t decode_launch(const DecodeParams& p, cudaStream_t stream);

// Tensor-core decode (decode_tc.cu): whether a (head_dim, group) geometry runs
// on it (LARA_DECODE_PATH=simt|tc overrides the default, groups >= 8), its
// split plan (any chunk works; the plan uses multiples of its 128-token tile),
// and its launch.  The launch returns cudaErrorNotSupported when the tensors
// cannot be described by tensor maps (alignment, paged cache); the caller then
// runs the CUDA-core kernel.  The kernel keeps a work ticket and a finished-CTA
// count in words 32 and 33 of the workspace's status block (zero between
// launches; the last CTA resets them).
bool decode_tc_selected(int head_dim, int group);
void decode_tc_plan(int batch, int n_kv_heads, int max_tokens, const int32_t* lens_host, int* nsplit, int* chunk);
cudaError_t decode_tc_launch(const DecodeParams& p, cudaStream_t stream);

// Failure-detection self test: a bounded wait on a phase nothing completes;
// sets kDevWaitTimeout in *status after limit_us.
cudaError_t selftest_wait_launch(int* status, int limit_us, cudaStream_t stream);

// Tensor-core (tcgen05/TMEM) attention of n_q query rows per sequence over a
// bf16 KV cache [batch][Hkv][kv_rows][128].  Sequence b has
// kv_len = base + kv_add keys (base = base_lens[b] or 0) and query row i sees
// keys j <= base + q_add + i when causal.
struct PrefillTcParams {
  const uint16_t* q;           // q[b * q_sb + i * q_sr + h * q_sh + d]
  long long q_sb, q_sr, q_sh;
  const uint16_t* k;
  const uint16_t* v;
  int kv_rows;
  uint16_t* o;                 // same indexing as q with o_* strides
  long long o_sb, o_sr, o_sh;
  int batch, n_q, n_q_heads, n_kv_heads, head_dim;
  const int32_t* base_lens;
  int kv_add, q_add;
  int causal;
  float scale_log2;
  int* status;
  int split_p;                 // 1: P = P_hi + P_lo (two bf16 MMA passes); 0: P in one bf16
};

bool prefill_tc_supported(int head_dim, int n_q_heads, int n_kv_heads);
cudaError_t prefill_tc_launch(const PrefillTcParams& p, cudaStream_t stream);

// Merge `num_parts` partial states of `rows` rows; part i's (m, l) pairs start
// at part_ml + i * ml_stride, its acc rows at part_acc + i * acc_stride
// (floats).  Writes bf16 `o` if non-null, else the merged (m, l, acc).
cudaError_t lse_combine_launch(const float* part_ml, long long ml_stride, const float* part_acc, long long acc_stride,
                               int num_parts, int rows, int head_dim, uint16_t* o, float* out_ml, float* out_acc,
                               cudaStream_t stream);

cudaError_t kv_append_launch(uint16_t* k_cache, uint16_t* v_cache, int32_t* lens, const uint16_t* k_new,
                             const uint16_t* v_new, int batch, int n_kv_heads, int head_dim, int max_seq_len,
                             int n_new, int* status, cudaStream_t stream);

cudaError_t kv_append_paged_launch(uint16_t* k_pages, uint16_t* v_pages, const int32_t* block_table, int32_t* lens,
                                   const uint16_t* k_new, const uint16_t* v_new, int batch, int n_kv_heads,
                                   int head_dim, int page_log2, int pages_per_seq, int num_pages, int n_new,
                                   int* status, cudaStream_t stream);
cudaError_t pack_bf16_launch(const float* src, uint16_t* dst, size_t n, cudaStream_t stream);

int device_sm_count();

// Launch `fn` with programmatic stream serialization, so its CTAs may be
// scheduled while the previous kernel in the stream finishes (the kernel must
// call grid_dependency_wait() before touching global memory).  LARA_PDL=0
// launches it the ordinary way.
cudaError_t launch_with_pdl(const void* fn, dim3 grid, dim3 block, void** args, size_t smem, cudaStream_t stream);

// Record the calling thread's last error message (lara_last_error_string)
// and return `code`.
int set_last_error(int code, const std::string& message);

}  // namespace lara
