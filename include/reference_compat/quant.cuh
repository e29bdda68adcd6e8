// Stand-in for the reference's include/quant.cuh when its harness
// (src/main.cu) is built against this library: the GPU preprocessing
// launchers (launch_quantize, launch_dequantize and the repacks) come from
// int4gemm.hpp. The harness's CPU checker (quantize_cpu, dequantize_cpu,
// compare_half, cpu_gemm_fp32) stays the reference's own src/reference.cu,
// linked into the harness; its declarations (include/quant.cuh:23-30) are
// repeated here because that file is replaced.
#pragma once

#include <vector>

#include "common.cuh"

#include "../int4gemm.hpp"

namespace int4gemm {

void quantize_cpu(const std::vector<half>& b, std::vector<uint8_t>& packed,
                  std::vector<half>& scales, int K, int N, int group_size);
void dequantize_cpu(const std::vector<uint8_t>& packed, const std::vector<half>& scales,
                    std::vector<half>& b, int K, int N, int group_size);
ErrorMetrics compare_half(const std::vector<half>& got, const std::vector<half>& ref);
void cpu_gemm_fp32(const std::vector<half>& a, const std::vector<half>& b,
                   std::vector<float>& c, int M, int N, int K);

}  // namespace int4gemm
