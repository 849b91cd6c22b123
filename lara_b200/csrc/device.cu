// Device and build facts for deployment reports.
//
// The reference's board bring-up (sw/clear_pynq_cache.py:190-310) checks that
// the FPGA is present and ready (`xbutil examine`) before any harness runs.
// On B200 the equivalent facts are the CUDA device's identity and whether
// this library's sm_100a code can be loaded on it.
#include <cstring>

#include "../../include/lara_b200.h"
#include "common.cuh"
#include "lara_internal.h"

namespace {

// Present only so that cudaFuncGetAttributes can tell whether the library's
// sm_100a image loads on a device; it is never launched.
__global__ void image_probe_kernel(int* p) {
  if (p) *p = 0;
}

// Failure-detection self test: every thread waits, with the same bounded wait
// the attention kernels use, on an mbarrier phase that nothing completes.  The
// wait gives up after limit_ns and the kernel reports kDevWaitTimeout in the
// status word -- the path a stuck pipeline takes -- without faulting.
__global__ void selftest_wait_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    lara::mbar_init(&bar, 1);
    lara::mbar_fence_init();
  }
  __syncthreads();
  const bool ok = lara::mbar_wait_bounded(&bar, 0, limit_ns);
  if (!__syncthreads_and(ok) && threadIdx.x == 0) atomicOr(status, lara::kDevWaitTimeout);
}

}  // namespace

namespace lara {
cudaError_t selftest_wait_launch(int* status, int limit_us, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 64, 0, stream>>>(status, (unsigned long long)limit_us * 1000ull);
  return cudaGetLastError();
}
}  // namespace lara

extern "C" int lara_selftest_wait_timeout(void* workspace, int limit_us, void* stream) {
  if (!workspace) return lara::set_last_error(LARA_ERR_STREAM_DEST, "null workspace");
  if (limit_us < 1 || limit_us > 2000000) return lara::set_last_error(LARA_ERR_BAD_CFG, "limit_us must be in [1, 2e6]");
  const cudaError_t e = lara::selftest_wait_launch(static_cast<int*>(workspace), limit_us,
                                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return lara::set_last_error(LARA_ERR_CUDA, std::string("self-test launch: ") + cudaGetErrorString(e));
  return LARA_OK;
}

extern "C" int lara_device_count(int* count) {
  if (!count) return lara::set_last_error(LARA_ERR_STREAM_DEST, "null output pointer");
  *count = 0;
  const cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return lara::set_last_error(LARA_ERR_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  }
  return LARA_OK;
}

extern "C" int lara_device_query(int device, lara_device_info* out) {
  if (!out) return lara::set_last_error(LARA_ERR_STREAM_DEST, "null output pointer");
  std::memset(out, 0, sizeof(*out));
  cudaRuntimeGetVersion(&out->runtime_version);
  cudaDriverGetVersion(&out->driver_version);
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess)
    return lara::set_last_error(LARA_ERR_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  if (device < 0 || device >= n)
    return lara::set_last_error(LARA_ERR_BAD_CFG, "device " + std::to_string(device) + " out of range (" +
                                                      std::to_string(n) + " visible)");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess)
    return lara::set_last_error(LARA_ERR_CUDA, std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e));
  std::strncpy(out->name, prop.name, sizeof(out->name) - 1);
  out->cc_major = prop.major;
  out->cc_minor = prop.minor;
  out->sm_count = prop.multiProcessorCount;
  out->total_mem_bytes = prop.totalGlobalMem;
  std::snprintf(out->pci_bus_id, sizeof(out->pci_bus_id), "%04x:%02x:%02x.0", prop.pciDomainID, prop.pciBusID,
                prop.pciDeviceID);

  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  cudaFuncAttributes attr;
  e = cudaFuncGetAttributes(&attr, image_probe_kernel);
  out->kernel_image_ok = (e == cudaSuccess && attr.binaryVersion == 100) ? 1 : 0;
  if (e != cudaSuccess) cudaGetLastError();  // a missing image is a fact to report, not a sticky error
  if (prev >= 0) cudaSetDevice(prev);
  return LARA_OK;
}
