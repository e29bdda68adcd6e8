// Test infrastructure only: a C entry to the reference's own GPU quantizer
// (src/quantize.cu, launch_quantize), built with the reference's
// --use_fast_math flag (Makefile:18) so its divisions behave as they do in
// the reference binary. Used to count where it differs from quantize_cpu
// (src/reference.cu:6-26).
#include "quant.cuh"

extern "C" int i4r_gpu_quantize(const void* b, uint8_t* packed, void* scales, int K, int N,
                                int group, void* stream) {
  try {
    int4gemm::launch_quantize(static_cast<const half*>(b), packed, static_cast<half*>(scales), K,
                              N, group, static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return -1;
  }
}
