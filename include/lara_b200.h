/*
 * lara_b200.h -- C ABI of liblara_b200.so, the B200 (sm_100a) implementation
 * of LARA's grouped-query streaming-attention path.
 *
 * The reference drives its FPGA through a Python/PYNQ driver
 * (sw/attn_driver.py): MMIO writes to CSRs, DMA of K/V per GQA group and of
 * padded Q tiles, a host poll loop, and a DMA read of O.  This library replaces
 * that MMIO/DMA layer and the RTL datapath behind it.  Every entry point below
 * names the reference interface it replaces.
 *
 * Conventions
 *  - bf16 tensors are passed as raw uint16_t words (IEEE bf16 upper halves),
 *    exactly as the reference passes them (sw/attn_driver.py:88-103).
 *  - Layouts: decode queries q[B][Hq][D]; KV cache [B][Hkv][Lmax][D]; the
 *    dense transaction keeps the reference's head-major q[Hq][L][D],
 *    k/v[Hkv][L][D], o[Hq][L][D] (sw/attn_driver.py:487-490).
 *  - Query head h belongs to KV group h / (Hq/Hkv)
 *    (sw/board_performance.py:182-184).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream).  Stateless kernels are asynchronous and stream-ordered.
 *  - Every function returns a status code (LARA_OK on success).  The text of
 *    the most recent failure on the calling thread is returned by
 *    lara_last_error_string().
 *  - A context is not thread-safe; use one context per device per thread.
 */
#ifndef LARA_B200_H
#define LARA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LARA_API __attribute__((visibility("default")))
#else
#define LARA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  0x00-0x12 mirror the accelerator's ERROR_CODE CSR values
 * (sw/attn_driver.py:80-85, hw/rtl/pkg/attn_pkg.sv:279-286). */
#define LARA_OK 0x00              /* ERR_NONE */
#define LARA_ERR_BAD_CFG 0x01     /* ERR_BAD_CFG: geometry / length / position out of range */
#define LARA_ERR_BUSY_START 0x02  /* ERR_BUSY_START: context closed or busy */
#define LARA_ERR_STREAM_LEN 0x10  /* ERR_STREAM_LEN: a tensor size does not match the configuration */
#define LARA_ERR_STREAM_DEST 0x11 /* ERR_STREAM_DEST: null or misaligned buffer */
#define LARA_ERR_RESULT_LEN 0x12  /* ERR_RESULT_LEN: output buffer too small */
#define LARA_ERR_CUDA 0x20        /* a CUDA runtime call failed */
#define LARA_ERR_TIMEOUT 0x21     /* a bounded device wait or lara_sync timed out */
#define LARA_ERR_UNSUPPORTED 0x22 /* no kernel compiled for this head geometry */
#define LARA_ERR_DEVICE 0x23      /* the kernel reported a device-side error status */

#define LARA_ABI_VERSION 1

LARA_API int lara_abi_version(void);
LARA_API const char* lara_last_error_string(void);
LARA_API const char* lara_status_name(int status);

/* Device facts for the deployment report.  Replaces the board readiness
 * checks of sw/clear_pynq_cache.py:190-310 (`xbutil examine` must report a
 * ready KV260): here the device must be visible and this library's sm_100a
 * image must load on it (kernel_image_ok). */
typedef struct lara_device_info {
  char name[256];
  char pci_bus_id[32];
  int cc_major;
  int cc_minor;
  int sm_count;
  int kernel_image_ok; /* 1 when the library's sm_100a code loads on this device */
  int driver_version;  /* cudaDriverGetVersion, e.g. 12090 */
  int runtime_version; /* the statically linked CUDA runtime */
  unsigned long long total_mem_bytes;
} lara_device_info;

LARA_API int lara_device_count(int* count);
LARA_API int lara_device_query(int device, lara_device_info* out);

/* ------------------------------------------------------------------------ */
/* Stateless kernels: caller-owned device memory (e.g. torch tensors).       */
/* ------------------------------------------------------------------------ */

/* Split plan for a decode workload on the current device.  lens_host may be
 * NULL (every sequence is max_seq_len long) or point to B host int32 lengths.
 * Writes the split count and the tokens of splits 1..num_splits-1.  When
 * num_splits * chunk_tokens < max_seq_len, split 0 takes the rest,
 * max_seq_len - (num_splits - 1) * chunk_tokens rounded up to 128 tokens (the
 * tensor-core decode's plans use this: long first items, short later ones). */
LARA_API int lara_decode_plan(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len,
                     const int32_t* lens_host, int* num_splits, int* chunk_tokens);

/* Which decode kernel a geometry runs on: LARA_DECODE_KERNEL_TENSOR (the
 * tcgen05 kernel: head_dim 128, groups of 8 or 16 query heads) or
 * LARA_DECODE_KERNEL_CUDA_CORE.  The environment variable
 * LARA_DECODE_PATH=simt|tc overrides the choice (tc also takes groups of 1, 2
 * and 4).  The tensor-core kernel needs 16-byte aligned q/k/v rows and, for a
 * paged cache, splits on 128-token boundaries (the planner's always are);
 * otherwise the CUDA-core kernel runs.  Both give results within the parity
 * bound of the same oracle, and a paged decode gives the same words as a
 * contiguous one on the same kernel. */
#define LARA_DECODE_KERNEL_CUDA_CORE 0
#define LARA_DECODE_KERNEL_TENSOR 1
LARA_API int lara_decode_kernel(int n_q_heads, int n_kv_heads, int head_dim);

/* Bytes of device workspace a decode with `num_splits` splits needs. */
LARA_API size_t lara_decode_workspace_bytes(int batch, int n_q_heads, int n_kv_heads, int head_dim, int num_splits);

/* Zero a workspace (once, before its first use; kernels leave it reusable). */
LARA_API int lara_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Read and clear the device status word of a workspace (synchronises the
 * stream).  *device_status receives the raw bits (0 = no error). */
LARA_API int lara_workspace_status(void* workspace, void* stream, int* device_status);

/* One decode step: for every sequence b and query head h,
 *   o[b,h,:] = softmax(scale * q[b,h,:] . K[b,h/G,:len_b,:]^T) . V[b,h/G,:len_b,:]
 * bf16 in, exact products, fp32 accumulation and online softmax, bf16 RNE out.
 * seq_lens: device int32[B], each in [0, max_seq_len]; a sequence of length 0
 * gives a zero output.  num_splits/chunk_tokens come from lara_decode_plan
 * (any num_splits >= 1 and chunk_tokens a multiple of the kernel tile; splits
 * that do not cover max_seq_len leave the rest to split 0, as documented at
 * lara_decode_plan); pass 0/0 to plan here.
 * Replaces: AttentionAccelerator.run_attention (sw/attn_driver.py:469-550)
 * and the datapath it drives (hw/rtl/attn_top.sv:301-625) for one query token
 * per sequence over a resident cache. */
LARA_API int lara_gqa_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* seq_lens,
                    uint16_t* o, int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len,
                    float scale, int num_splits, int chunk_tokens, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Same as lara_gqa_decode but writes the unnormalised partial state of every
 * (b, h) row instead of bf16 output: part_ml[(b*Hq+h)*2 + {0,1}] = {m, l}
 * (m is the running max of scale*log2(e)*q.k, l the sum of 2^(s-m)) and
 * part_acc[(b*Hq+h)*D + d] = sum 2^(s-m) v.  Used when a sequence is split
 * across GPUs; lara_lse_combine merges the partials.  (The reference has a
 * single device and no counterpart; this is the per-device half of
 * split-KV decode.) */
LARA_API int lara_gqa_decode_partial(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            const int32_t* seq_lens, float* part_ml, float* part_acc, int batch, int n_q_heads,
                            int n_kv_heads, int head_dim, int max_seq_len, float scale, int num_splits,
                            int chunk_tokens, void* workspace, size_t workspace_bytes, void* stream);

/* Merge num_parts partial states of `rows` query rows:
 * part_ml[(i*rows + r)*2 + {0,1}], part_acc[(i*rows + r)*D + d] -> o[r*D + d]
 * (bf16 RNE; a row whose l sums to 0 gives zeros).
 * Replaces: the O normalise + writeback of hw/rtl/mem/output_buffer.sv:271-286
 * for state that was accumulated on several devices. */
LARA_API int lara_lse_combine(const float* part_ml, const float* part_acc, int num_parts, int rows, int head_dim,
                     uint16_t* o, void* stream);

/* lara_lse_combine with explicit per-part strides (in floats): part i's (m, l)
 * pairs start at part_ml + i*ml_part_stride and its acc rows at
 * part_acc + i*acc_part_stride.  Lets each device keep its partial state
 * packed as [rows*2 (m,l) | rows*D acc] so one all-gather moves it.
 * Replaces: as lara_lse_combine (hw/rtl/mem/output_buffer.sv:271-286). */
LARA_API int lara_lse_combine_strided(const float* part_ml, long long ml_part_stride, const float* part_acc,
                                      long long acc_part_stride, int num_parts, int rows, int head_dim, uint16_t* o,
                                      void* stream);

/* Append n_new tokens per sequence: k_new/v_new[B][Hkv][n_new][D] are written
 * at positions seq_lens[b] .. seq_lens[b]+n_new-1 of the cache, then
 * seq_lens[b] += n_new.  Rows that would pass max_seq_len are dropped and
 * flag LARA_ERR_DEVICE in the workspace status (if workspace != NULL).
 * Replaces: the K/V cache loads of sw/attn_driver.py:418-422 into
 * hw/rtl/mem/kv_cache_ram.sv:45-91. */
LARA_API int lara_kv_append(uint16_t* k_cache, uint16_t* v_cache, int32_t* seq_lens, const uint16_t* k_new,
                   const uint16_t* v_new, int batch, int n_kv_heads, int head_dim, int max_seq_len, int n_new,
                   void* workspace, void* stream);

/* fp32 -> bf16 RNE words with the integer steps of the reference packer, so
 * results (NaN and Inf patterns included) are bit-identical to it.
 * src 16-byte aligned, dst 8-byte aligned.
 * Replaces: fp32_to_bf16_u16 (sw/attn_driver.py:88-98). */
LARA_API int lara_pack_bf16(const float* src, uint16_t* dst, size_t n, void* stream);

/* Chunked prefill over the cache ("cache + self"): the n_new new tokens of
 * every sequence are already appended (lara_kv_append) at positions
 * cached_lens[b] .. cached_lens[b]+n_new-1, where cached_lens[b] (device
 * int32[B]) is the length BEFORE the append.  q/o are token-major
 * [B][n_new][Hq][D].  Query i of sequence b sits at position cached_lens[b]+i;
 * with causal != 0 it sees tokens 0..cached_lens[b]+i (kv_pos <= q_pos,
 * sw/board_performance.py:174-177), otherwise all cached_lens[b]+n_new.
 * Workspace: lara_prefill_workspace_bytes.
 * Replaces: run_attention's causal Q-tile x KV-tile traversal with causal tile
 * skipping (hw/rtl/core/attn_core.sv:107-154) over a resident cache. */
LARA_API size_t lara_prefill_workspace_bytes(int batch, int n_new, int n_q_heads, int n_kv_heads, int head_dim,
                                             int max_seq_len);
LARA_API int lara_gqa_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                              const int32_t* cached_lens, uint16_t* o, int batch, int n_new, int n_q_heads,
                              int n_kv_heads, int head_dim, int max_seq_len, int causal, float scale,
                              void* workspace, size_t workspace_bytes, void* stream);

/* One dense attention transaction, the semantics of run_attention with
 * Lq == Lkv == seq_len: q[Hq][L][D], k/v[Hkv][L][D], o[Hq][L][D] (device
 * pointers).  Query i has position q_pos_base+i, key j kv_pos_base+j; with
 * causal != 0 a key is visible when kv_pos <= q_pos
 * (sw/board_performance.py:174-177).  A query row with no visible key gives
 * zeros.  Workspace: lara_dense_workspace_bytes.
 * Replaces: AttentionAccelerator.run_attention (sw/attn_driver.py:469-550). */
LARA_API size_t lara_dense_workspace_bytes(int n_q_heads, int n_kv_heads, int head_dim, int seq_len);
LARA_API int lara_attention_dense(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int n_q_heads,
                         int n_kv_heads, int head_dim, int seq_len, int q_pos_base, int kv_pos_base, int causal,
                         float scale, void* workspace, size_t workspace_bytes, void* stream);

/* The same transaction in board arithmetic: the output words of LARA's FPGA
 * datapath, bit for bit, for boards' expected_o comparisons
 * (sw/board_matrix.py:118-156).  The FPGA's own fp32 adder and multiplier
 * (hw/rtl/pkg/attn_pkg.sv:404-597), score accumulation sequential over the
 * 128 dims, scale by fp32 0x3DB504F3, exp by a 1024-entry table with linear
 * interpolation (hw/rtl/core/softmax_engine.sv:570-705), P truncated to bf16
 * for P.V (hw/rtl/attn_top.sv:652-659), the O correction per 16-token block
 * and a 256-entry reciprocal table for the normalisation
 * (hw/rtl/mem/output_buffer.sv:199-286).  head_dim must be 128 (the scale is
 * the RTL's constant); Hq % Hkv == 0; 0 <= pos_base, pos_base + seq_len <=
 * 65536.  No workspace.  Stream-ordered; the first call on a device uploads
 * the lookup tables and synchronises the stream. */
LARA_API int lara_attention_dense_board(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                                        int n_q_heads, int n_kv_heads, int head_dim, int seq_len, int causal,
                                        int q_pos_base, int kv_pos_base, void* stream);

/* Paged KV cache: K/V live in page pools k_pages/v_pages
 * [num_pages][Hkv][page_size][D] (bf16; the rows of one (page, kv head) are
 * contiguous) and block_table[b * pages_per_seq + j] (device int32) names the
 * page holding tokens j*page_size .. (j+1)*page_size-1 of sequence b.  Pages
 * may be shared between sequences (a common prefix) and appear in any order.
 * page_size is a power of two in [16, 65536]; a sequence holds at most
 * pages_per_seq * page_size tokens, which is the max_seq_len of
 * lara_decode_plan / lara_decode_workspace_bytes.  A block-table entry outside
 * [0, num_pages) is reported through the workspace status word (the access
 * reads page 0 instead).  Otherwise identical to lara_gqa_decode: same
 * arithmetic, same results bit for bit as a contiguous cache holding the
 * same tokens.  (The reference keeps one sequence per transaction in BRAM,
 * hw/rtl/mem/kv_cache_ram.sv; there is no counterpart of a page pool.) */
LARA_API int lara_gqa_decode_paged(const uint16_t* q, const uint16_t* k_pages, const uint16_t* v_pages,
                                   const int32_t* block_table, const int32_t* seq_lens, uint16_t* o, int batch,
                                   int n_q_heads, int n_kv_heads, int head_dim, int page_size, int pages_per_seq,
                                   int num_pages, float scale, int num_splits, int chunk_tokens, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Append n_new tokens per sequence (k/v_new[B][Hkv][n_new][D]) into a paged
 * cache at positions seq_lens[b] .. seq_lens[b]+n_new-1, then advance
 * seq_lens.  The pages those positions fall in must already be in the block
 * table (the caller's page allocator assigns them).  Rows past the capacity or
 * naming a bad page are dropped and flagged in the workspace status word
 * (workspace may be NULL: no status).  Replaces: the K/V cache write of
 * hw/rtl/mem/kv_cache_ram.sv:45-91 for a paged cache. */
LARA_API int lara_kv_append_paged(uint16_t* k_pages, uint16_t* v_pages, const int32_t* block_table,
                                  int32_t* seq_lens, const uint16_t* k_new, const uint16_t* v_new, int batch,
                                  int n_kv_heads, int head_dim, int page_size, int pages_per_seq, int num_pages,
                                  int n_new, void* workspace, void* stream);

/* Layer prologue: the host half of AttentionAccelerator.run_layer
 * (sw/attn_driver.py:552-586) on the GPU, writing the run_attention layout.
 *   x_n = rms_weight ? bf16(fp32(fp32(x * inv) * rms_weight)) : x, with
 *         inv = fp32(1 / sqrt(mean(x^2) + rms_eps)) from an fp64 mean
 *         (hw/rtl/ext/rms_norm/rms_norm.sv:7)
 *   [q | k | v] = x_n @ w_qkv with w_qkv = [Wq | Wk | Wv] stored
 *         [hidden][(Hq + 2*Hkv) * D] (the [IN_DIM][OUT_DIM] weight stream of
 *         hw/rtl/ext/qkv_projection/qkv_projection.sv), fp32 accumulation on
 *         the tensor cores
 *   RoPE on q at positions q_pos_base + t and on k at kv_pos_base + t:
 *         dims (2i, 2i+1) rotate by pos * rope_base^(-2i/D)
 *         (hw/rtl/core/rope_engine.sv:1-11), fp32
 *   q[B][Hq][L][D], k[B][Hkv][L][D], v[B][Hkv][L][D] in bf16 (round to
 *         nearest even); B = batch sequences of seq_len tokens each, every
 *         sequence at the same position bases (B = 1 is run_layer's case).
 * x[B][L][hidden], rms_weight[hidden] (NULL: no normalisation) and w_qkv are
 * bf16 device buffers; all pointers 16-byte aligned.  head_dim must be 128,
 * hidden a multiple of 64, positions below 2^24.  Workspace:
 * lara_layer_prologue_workspace_bytes (its first word is the status word,
 * read by lara_workspace_status). */
LARA_API size_t lara_layer_prologue_workspace_bytes(int batch, int seq_len, int hidden);
LARA_API int lara_layer_prologue(const uint16_t* x, const uint16_t* rms_weight, const uint16_t* w_qkv, uint16_t* q,
                                 uint16_t* k, uint16_t* v, int batch, int seq_len, int hidden, int n_q_heads,
                                 int n_kv_heads, int head_dim, int q_pos_base, int kv_pos_base, float rms_eps,
                                 float rope_base, void* workspace, size_t workspace_bytes, void* stream);

/* Decode with no allocation by the caller or the library.  Same arguments,
 * semantics and results as lara_gqa_decode, minus the workspace: the split
 * partials, arrival counters and status word live in a fixed array of
 * LARA_NOALLOC_SCRATCH_BYTES in the library's own device memory, reserved on
 * every GPU that loads the library until the process exits.  For callers that
 * cannot allocate device memory where they run attention (a plugin inside a
 * framework that owns all device allocations, a serving loop that may not pay
 * cudaMalloc's implicit synchronisation, a binding that can pass only the
 * operation's tensors).  No cudaMalloc, cudaFree or other allocating routine
 * is called.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before any stream capture.  The address is cached per device together
 *    with the unique id of the CUDA context it belongs to, and looked up again
 *    when a call runs under another context (after cudaDeviceReset, or under
 *    a context a driver-API caller made current).
 *  - Device-side status flags are not reported: the kernels' status word
 *    lives in the shared array, which the caller cannot address and the next
 *    call clears.  A seq_lens entry outside [0, max_seq_len] is clamped to
 *    that range without an error, and a bounded wait that times out leaves
 *    the output undefined without an error.  Callers that need those reports
 *    use lara_gqa_decode with a workspace and lara_workspace_status.
 *  - num_splits/chunk_tokens = 0/0 plans automatically and reduces the split
 *    count until the partials fit; explicit values, or a batch whose minimum
 *    scratch exceeds the array, are rejected with LARA_ERR_RESULT_LEN and a
 *    message naming the limit.
 *  - Every call shares the one array: the status word and counters are zeroed
 *    at the start of each call (stream-ordered), and calls that overlap on the
 *    GPU (different streams, or concurrent host threads) race on it.
 * No counterpart in the reference (the FPGA owns fixed on-chip buffers). */
#define LARA_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)
LARA_API int lara_gqa_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                     const int32_t* seq_lens, uint16_t* o, int batch, int n_q_heads,
                                     int n_kv_heads, int head_dim, int max_seq_len, float scale, int num_splits,
                                     int chunk_tokens, void* stream);

/* ------------------------------------------------------------------------ */
/* Context API: the backing of the Python AttentionAccelerator.  The context */
/* owns the HBM KV cache, device I/O buffers, a stream and timing events.   */
/* Tensor pointers are host memory unless on_device != 0.                    */
/* ------------------------------------------------------------------------ */

typedef struct lara_ctx lara_ctx;

typedef struct lara_perf {
  /* Device time of the last transaction in ns (clock_mhz = 1000, so these
   * are "cycles" of a 1 GHz clock): total = first H2D copy to last D2H copy,
   * mac = attention kernels, stall = host<->device copies. */
  uint64_t cycles;
  uint64_t mac_cycles;
  uint64_t stall_cycles;
  double clock_mhz;
} lara_perf;

/* Replaces: AttentionAccelerator.__init__ (Overlay load, buffer allocation;
 * sw/attn_driver.py:251-288). */
LARA_API int lara_create(int device, lara_ctx** out);

/* Replaces: AttentionAccelerator.close (sw/attn_driver.py:324-331).  Frees
 * every device and pinned buffer; NULL is accepted. */
LARA_API int lara_destroy(lara_ctx* ctx);

/* Head geometry and cache capacity; (re)allocates the KV cache and buffers,
 * and empties the cache.  Defaults after lara_create: batch 1, 32/8 heads,
 * head_dim 128, max_seq_len 512 (hw/rtl/pkg/attn_pkg.sv:172-176).
 * Extension of the reference call surface (no CSR counterpart: the RTL
 * geometry is fixed at synthesis). */
LARA_API int lara_configure_heads(lara_ctx* ctx, int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_seq_len);

/* Transaction registers of the dense path.  Replaces: configure
 * (sw/attn_driver.py:364-376: SEQ_LEN, Q/KV_POS_BASE, CFG.causal) with its
 * validation (1 <= seq_len <= max_seq_len, positions + seq_len <= 2^16). */
LARA_API int lara_configure(lara_ctx* ctx, int seq_len, int q_pos_base, int kv_pos_base, int causal);

/* Load the cache: k/v[B][Hkv][src_len][D], lens[B] (host int32, each <=
 * src_len and <= max_seq_len).  Replaces: the KV_LOAD_REQ service of
 * sw/attn_driver.py:418-422. */
LARA_API int lara_kv_load(lara_ctx* ctx, const uint16_t* k, const uint16_t* v, const int32_t* lens, int src_len,
                 int on_device);

/* Append one chunk of n_new tokens per sequence (k/v[B][Hkv][n_new][D]). */
LARA_API int lara_kv_append_ctx(lara_ctx* ctx, const uint16_t* k_new, const uint16_t* v_new, int n_new, int on_device);

/* Chunked prefill: append k/v_new[B][Hkv][n_new][D], then attend
 * q[B][n_new][Hq][D] -> o[B][n_new][Hq][D] over cache + self (see
 * lara_gqa_prefill); synchronous.  With host buffers (on_device = 0), B > 1
 * and the tensor-core kernel, the call is pipelined by sequence: the copies of
 * one sequence overlap the kernels of the previous one and the copy back of
 * the one before (page-locked host buffers let the copies run asynchronously).
 * The output words are those of the single-launch path. */
LARA_API int lara_run_prefill_chunk(lara_ctx* ctx, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                                    uint16_t* o, int n_new, int causal, int on_device);

/* Read the cache back: the first dst_len tokens of every (sequence, kv head)
 * row into k/v[B][Hkv][dst_len][D] and the lengths into lens_out (host
 * int32[B]); synchronous.  With lara_kv_load this saves and restores a cache
 * (AttentionAccelerator.save_kv / restore_kv).  No reference counterpart: the
 * FPGA's BRAM cache does not outlive a transaction. */
LARA_API int lara_kv_read(lara_ctx* ctx, uint16_t* k, uint16_t* v, int32_t* lens_out, int dst_len, int on_device);

/* Copy the current lengths (host int32[B]). */
LARA_API int lara_get_seq_lens(lara_ctx* ctx, int32_t* lens_out);

/* Shorten the sequences to lens[B] (host int32, each <= its current length):
 * the rows past the new length are dropped and later appends overwrite them
 * (rewinding a prefill chunk or rejected speculative tokens); synchronous.
 * LARA_ERR_STREAM_LEN if a length would grow.  No reference counterpart: the
 * FPGA reloads its KV RAM on every transaction (sw/attn_driver.py:418-422), so
 * it has no resident lengths to rewind. */
LARA_API int lara_kv_truncate(lara_ctx* ctx, const int32_t* lens);

/* Decode: q[B][Hq][D] -> o[B][Hq][D] over the resident cache; synchronous
 * (returns after o is written).  Page-locked host q / o (cudaHostAlloc,
 * cudaHostRegister, torch pin_memory) are read and written by the kernel in
 * place over the interconnect; pageable host memory is staged.  Replaces: run_attention's request service and
 * readback (sw/attn_driver.py:418-464) for one query token per sequence. */
LARA_API int lara_run_query(lara_ctx* ctx, const uint16_t* q, uint16_t* o, int on_device);

/* Arithmetic of the context's dense transactions (lara_run_attention):
 * LARA_ARITH_IEEE (default; fp32 with a true exp, within 2 bf16 ulp of the
 * reference's CPU golden model) or LARA_ARITH_BOARD (the FPGA's output words
 * bit for bit, see lara_attention_dense_board; head_dim 128 only).  Decode and
 * prefill always use IEEE arithmetic. */
#define LARA_ARITH_IEEE 0
#define LARA_ARITH_BOARD 1
LARA_API int lara_set_arithmetic(lara_ctx* ctx, int mode);
LARA_API int lara_get_arithmetic(lara_ctx* ctx);

/* Dense transaction with the configure()d registers: q[Hq][L][D],
 * k/v[Hkv][L][D] -> o[Hq][L][D]; synchronous.  Replaces: run_attention
 * (sw/attn_driver.py:469-550). */
LARA_API int lara_run_attention(lara_ctx* ctx, const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o,
                       int on_device);

/* One layer: lara_layer_prologue on x[L][hidden] with w_qkv / rms_weight
 * (rms_weight may be NULL), then the dense transaction of lara_run_attention
 * on the produced q/k/v with the configure()d registers and the context's
 * arithmetic -> o[Hq][L][D]; synchronous.  Pointers are host memory unless
 * on_device != 0.  Replaces: run_layer (sw/attn_driver.py:552-586), whose
 * RMSNorm / projection / RoPE ran on the host CPU.  lara_read_perf then covers
 * the whole call; lara_read_layer_perf splits the device time into the
 * prologue kernels and the attention kernels. */
LARA_API int lara_run_layer(lara_ctx* ctx, const uint16_t* x, const uint16_t* w_qkv, const uint16_t* rms_weight,
                            int hidden, uint16_t* o, float rms_eps, float rope_base, int on_device);
LARA_API int lara_read_layer_perf(lara_ctx* ctx, uint64_t* prologue_ns, uint64_t* attention_ns);

/* Failure-detection self tests (no reference counterpart; the RTL reports
 * timeouts through ERROR_CODE / STATUS_ERROR, sw/attn_driver.py:446-454).
 * A kernel waits, with the bounded wait every pipeline wait uses, on an
 * mbarrier phase that nothing completes; after limit_us (1 .. 2e6) it gives up
 * and sets the timeout bit of the status word -- no fault, no hang.
 * lara_selftest_wait_timeout writes the word at workspace[0] (read it with
 * lara_workspace_status); lara_ctx_selftest_timeout runs it on the context's
 * stream and returns LARA_ERR_TIMEOUT, after which the context is usable. */
LARA_API int lara_selftest_wait_timeout(void* workspace, int limit_us, void* stream);
LARA_API int lara_ctx_selftest_timeout(lara_ctx* ctx, int limit_us);

/* Asynchronous, stream-ordered forms on device buffers (the reference's
 * start() / wait_done() split, sw/attn_driver.py:361-464): they return once
 * the work is queued on `stream` (NULL: the context's stream); lara_sync then
 * waits for it and reports the device status word.  All calls on one context
 * must be ordered (one stream, or synchronised); they are ordered after the
 * context's earlier work automatically.
 * lara_decode: q[B][Hq][D] -> o[B][Hq][D] over the resident cache; splits = 0
 * uses the planner.  lara_prefill: lara_run_prefill_chunk on device buffers. */
LARA_API int lara_decode(lara_ctx* ctx, const uint16_t* q, uint16_t* o, int splits, void* stream);
LARA_API int lara_prefill(lara_ctx* ctx, const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new, uint16_t* o,
                          int n_new, int causal, void* stream);

/* Replaces: read_perf (sw/attn_driver.py:466-467, CSRs 0x100/0x108/0x10C). */
LARA_API int lara_read_perf(lara_ctx* ctx, lara_perf* out);

/* Wait for the context's stream; LARA_ERR_TIMEOUT after timeout_ms (< 0:
 * no limit).  Replaces: wait_done's deadline (sw/attn_driver.py:442-454). */
LARA_API int lara_sync(lara_ctx* ctx, int timeout_ms);

/* Device the context was created on. */
LARA_API int lara_ctx_device(lara_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* LARA_B200_H */
