// C++ host API with the reference's exact signatures, over the C ABI of i4g.h.
//
// A caller of zichaowen8-prog/SM_120__GEMM's include/quant.cuh (lines 6-21)
// and include/kernels.cuh (lines 24-25, 81-83) keeps its calls; each wrapper
// forwards to the matching i4g_* entry point and throws std::runtime_error on
// a non-zero status, as the reference's CUDA_CHECK does (common.cuh:17-19).
//
// One contract differs, as documented in i4g.h: launch_final consumes the
// tile layout written by launch_repack_umma (not the mma.sync lane-native
// layouts), with scales from launch_repack_scales_128.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "i4g.h"

namespace int4gemm {

inline void i4g_throw_if(int status, const char* what) {
  if (status != I4G_OK)
    throw std::runtime_error(std::string(what) + " failed: " + i4g_status_string(status) +
                             ": " + i4g_last_error());
}

using KernelLaunch = void (*)(const half*, const uint8_t*, const half*, half*, int, int, int,
                              int, cudaStream_t);

inline void launch_quantize(const half* b, uint8_t* packed, half* scales, int K, int N,
                            int group_size, cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_quantize(b, packed, scales, K, N, group_size, stream), "launch_quantize");
}

inline void launch_dequantize(const uint8_t* packed, const half* scales, half* b, int K, int N,
                              int group_size, cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_dequantize(packed, scales, b, K, N, group_size, stream), "launch_dequantize");
}

inline void launch_repack_128x32(const uint8_t* packed, const half* scales, uint8_t* repacked,
                                 half* repacked_scales, int K, int N, int group_size,
                                 cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_repack_128x32(packed, scales, repacked, repacked_scales, K, N, group_size,
                                 stream),
               "launch_repack_128x32");
}

inline void launch_inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed, int K, int N,
                                         cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_inverse_repack_128x32(repacked, packed, K, N, stream),
               "launch_inverse_repack_128x32");
}

inline void launch_repack_mma_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                                     cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_repack_mma_128x32(packed, repacked, K, N, stream), "launch_repack_mma_128x32");
}

inline void launch_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                                          cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_repack_mma_pair_128x32(packed, repacked, K, N, stream),
               "launch_repack_mma_pair_128x32");
}

inline void launch_repack_scales_128(const half* scales, half* repacked_scales, int K, int N,
                                     int group_size, cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_repack_scales_128(scales, repacked_scales, K, N, group_size, stream),
               "launch_repack_scales_128");
}

// New: the weight layout launch_final consumes.
inline void launch_repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N,
                               cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_repack_umma(packed, tiles, K, N, stream), "launch_repack_umma");
}

// New: launch_quantize + launch_repack_umma + launch_repack_scales_128 in one
// pass over B (the one-shot path of src/main.cu:320-331).
inline void launch_quantize_repack(const half* b, uint8_t* tiles, half* repacked_scales, int K,
                                   int N, int group_size, cudaStream_t stream = nullptr) {
  i4g_throw_if(i4g_quantize_repack(b, tiles, repacked_scales, K, N, group_size, stream),
               "launch_quantize_repack");
}

// New: launch_final / launch_final_fp32 with a split-K workspace (zeroed
// once; size from i4g_gemm_workspace_size), for shapes whose last wave of
// output tiles is partial.
inline void launch_final_ws(const half* a, const uint8_t* b, const half* s, half* c, int M,
                            int N, int K, int group, void* workspace, size_t workspace_bytes,
                            cudaStream_t stream) {
  i4g_throw_if(i4g_gemm_ws(a, b, s, c, M, N, K, group, workspace, workspace_bytes, stream),
               "launch_final_ws");
}
inline void launch_final_fp32_ws(const half* a, const uint8_t* b, const half* s, float* c, int M,
                                 int N, int K, int group, void* workspace,
                                 size_t workspace_bytes, cudaStream_t stream) {
  i4g_throw_if(
      i4g_gemm_fp32_ws(a, b, s, c, M, N, K, group, workspace, workspace_bytes, stream),
      "launch_final_fp32_ws");
}

inline void launch_final(const half* a, const uint8_t* b, const half* s, half* c, int M, int N,
                         int K, int group, cudaStream_t stream) {
  i4g_throw_if(i4g_gemm(a, b, s, c, M, N, K, group, stream), "launch_final");
}

inline void launch_final_fp32(const half* a, const uint8_t* b, const half* s, float* c, int M,
                              int N, int K, int group, cudaStream_t stream) {
  i4g_throw_if(i4g_gemm_fp32(a, b, s, c, M, N, K, group, stream), "launch_final_fp32");
}

}  // namespace int4gemm
