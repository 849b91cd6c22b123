// Decode entry point for callers that cannot allocate device memory.
//
// lara_gqa_decode needs a device workspace (split-KV partial results, the
// per-(sequence, kv head) arrival counters of the in-kernel merge, and a
// status word) that the caller allocates.  Some callers cannot do that at
// the point where they run attention: a plugin hosted by another framework
// that owns every device allocation and forbids side allocations, a serving
// loop that may not pay cudaMalloc's implicit device synchronisation or its
// unbounded latency, or a foreign-language binding that can hand over only
// the operation's own tensors.  lara_gqa_decode_noalloc serves them: its
// scratch is a fixed-size array in the library's own device memory
// (LARA_NOALLOC_SCRATCH_BYTES, reserved on every GPU that loads the library
// until the process exits), and it calls no cudaMalloc, cudaFree or other
// allocating routine.
//
// In host code the array's name is only a host-side stand-in, never a device
// address; its device address is looked up with cudaGetSymbolAddress (with
// that device current) on the entry point's first call on that device, and
// cached.  The array exists once per CUDA context, so the cache remembers the
// unique id of the context it was looked up in (cuCtxGetId) and looks the
// address up again when a call runs under another context: after
// cudaDeviceReset re-creates the primary context, or when a driver-API caller
// makes its own context current.
#include <cuda.h>  // CUcontext / CUresult types; the entry points are fetched at run time

#include <mutex>

#include "../../include/lara_b200.h"
#include "lara_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[LARA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct ScratchSlot {
  unsigned long long context_id = 0;  // 0: unknown, look the address up on every call
  void* addr = nullptr;
};

std::mutex g_scratch_mutex;
ScratchSlot g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the context current on this thread; 0 when none is current yet
// or the driver does not export the calls.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of g_decode_scratch in the context current on device `dev`.
int scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long id = current_context_id();
  if (slot.addr == nullptr || id == 0 || id != slot.context_id) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return lara::set_last_error(LARA_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc decode scratch failed: " +
                                                     std::string(cudaGetErrorString(e)));
    slot.addr = p;
    // the lookup makes the device's primary context current if none was
    slot.context_id = id != 0 ? id : current_context_id();
  }
  *out = slot.addr;
  return LARA_OK;
}

}  // namespace

extern "C" int lara_gqa_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                       const int32_t* seq_lens, uint16_t* o, int batch, int n_q_heads,
                                       int n_kv_heads, int head_dim, int max_seq_len, float scale, int num_splits,
                                       int chunk_tokens, void* stream) {
  LARA_NVTX("lara_gqa_decode_noalloc");
  const size_t cap = LARA_NOALLOC_SCRATCH_BYTES;
  if (batch < 1 || n_q_heads < 1 || n_kv_heads < 1 || head_dim < 1 || max_seq_len < 1 ||
      n_q_heads % n_kv_heads != 0)
    return lara::set_last_error(LARA_ERR_BAD_CFG, "bad decode geometry");
  const int tile = lara::decode_chunk_granule(head_dim, n_q_heads / n_kv_heads);
  if (tile == 0) return lara::set_last_error(LARA_ERR_UNSUPPORTED, "no kernel compiled for this head geometry");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return lara::set_last_error(LARA_ERR_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return lara::set_last_error(LARA_ERR_BAD_CFG, "device index out of range");
  void* scratch = nullptr;
  int rc = scratch_address(dev, &scratch);
  if (rc) return rc;

  // Split plan: the caller's, or the planner's reduced until the partial
  // results fit the fixed scratch.
  int splits = num_splits, chunk = chunk_tokens;
  if (splits <= 0 || chunk <= 0) {
    lara::decode_plan(batch, n_kv_heads, n_q_heads, head_dim, max_seq_len, nullptr, &splits, &chunk);
    while (splits > 1 && lara::decode_workspace_layout(batch, n_q_heads, n_kv_heads, head_dim, splits).total > cap) {
      --splits;
      const int tiles = (max_seq_len + tile * splits - 1) / (tile * splits);
      chunk = tiles * tile;
      splits = (max_seq_len + chunk - 1) / chunk;
    }
  }
  const lara::WorkspaceLayout w = lara::decode_workspace_layout(batch, n_q_heads, n_kv_heads, head_dim, splits);
  if (w.total > cap)
    return lara::set_last_error(
        LARA_ERR_RESULT_LEN,
        "lara_gqa_decode_noalloc: this decode needs " + std::to_string(w.total) + " bytes of scratch (" +
            std::to_string(splits) + " splits) but the fixed no-alloc scratch holds " + std::to_string(cap) +
            " bytes; use fewer splits, a smaller batch, or lara_gqa_decode with a caller workspace");

  // Every call shares the scratch, which keeps the previous call's contents:
  // the status word and the arrival counters must start at zero.
  e = cudaMemsetAsync(scratch, 0, w.ml_off, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return lara::set_last_error(LARA_ERR_CUDA, "clearing the no-alloc scratch failed");
  return lara_gqa_decode(q, k_cache, v_cache, seq_lens, o, batch, n_q_heads, n_kv_heads, head_dim, max_seq_len,
                         scale, splits, chunk, scratch, cap, stream);
}
