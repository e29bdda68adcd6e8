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

// Holds the split-K workspace of every shape on a device with up to 160 SMs:
// a plan stores at most 2 * sm_count - 1 partial tiles of 256 x 128 FP32
// (128 KiB) plus 1 KiB of arrival counters. Static device storage is
// zero-initialised when the module loads.
constexpr size_t kStaticScratchBytes = size_t(40) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

}  // namespace

size_t static_scratch_bytes() { return kStaticScratchBytes; }

// Device address of the scratch on `device`, which must be the current
// device. The first call per device loads the module (set-up).
cudaError_t static_scratch(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return cudaSuccess;
}

}  // namespace i4g
