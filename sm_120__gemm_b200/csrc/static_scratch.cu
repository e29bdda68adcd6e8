// Fixed split-K scratch for callers that cannot allocate device memory.
//
// The array lives in its own translation unit, hence its own CUDA module:
// with lazy module loading (the CUDA 12 default) a device pays for its
// footprint only once i4g_gemm_static_scratch has been called on it.
#include "gemm_tc.h"

#include <cuda_runtime.h>

#include <mutex>

namespace i4g {
namespace {

// Holds the split-K workspace of every tcgen05 shape on a device with up to
// 160 SMs: a plan stores at most 2 * sm_count - 2 partial tiles of 256 x 128
// FP32 (128 KiB each) after tc::kTicketBytes (4 KiB) of arrival counters,
// i.e. (2 * 160 - 2) * 128 KiB + 4 KiB < 40 MiB. Static device storage is
// zero-initialised when the module loads.
constexpr size_t kStaticScratchBytes = size_t(40) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

}  // namespace

size_t static_scratch_bytes() { return kStaticScratchBytes; }

// Device address of the scratch on the current device. The host-side name
// g_static_scratch is only a stand-in for the array, never a device address:
// the address is looked up with cudaGetSymbolAddress, with the device
// current, once per device (set-up; it also loads the module there), and
// kept for the life of the process. A cudaDeviceReset unloads the module, so
// the kept address is not valid after one: the entry point is not for use
// across a device reset.
cudaError_t static_scratch(void** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return cudaSuccess;
}

}  // namespace i4g
