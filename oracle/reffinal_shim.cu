// Test and baseline infrastructure only: a C entry to the reference's own
// final GEMM, kernels/gemm_v17_instruction.cu compiled unmodified for sm_100a
// with the reference's flags (Makefile:18, --use_fast_math). The group
// dispatch is the one of kernels/gemm_final.cu:5-13 (g32: V18a, compact
// registers + pair fragments; g64: V17b, ldmatrix; g128: V18b, compact
// registers + full/empty barriers), written here so the rest of that file
// (every earlier kernel generation) need not be compiled. Inputs are the
// reference's layouts: launch_repack_mma_pair_128x32 for g32 and g128,
// launch_repack_mma_128x32 for g64, launch_repack_scales_128 for the scales
// (src/main.cu:322-329). Its mbarrier waits are unbounded
// (gemm_v17_instruction.cu:25-38), so callers run it under a host timeout.
#include "kernels.cuh"

extern "C" int i4r_launch_final(const void* a, const uint8_t* b, const void* scales, void* c,
                                int M, int N, int K, int group, void* stream) {
  try {
    const half* ha = static_cast<const half*>(a);
    const half* hs = static_cast<const half*>(scales);
    half* hc = static_cast<half*>(c);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (group == 32)
      int4gemm::launch_v18a_tma_compact_pair(ha, b, hs, hc, M, N, K, group, s);
    else if (group == 64)
      int4gemm::launch_v17b_tma_ldmatrix(ha, b, hs, hc, M, N, K, group, s);
    else
      int4gemm::launch_v18b_tma_compact_full_empty(ha, b, hs, hc, M, N, K, group, s);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  } catch (...) {
    return -2;
  }
}
