// Stand-in for the reference's include/kernels.cuh when its harness
// (src/main.cu) is built against this library instead of the reference's
// kernels: launch_final / launch_final_fp32, KernelLaunch, KernelMetadata,
// KernelResources, kernel_registry() and query_resources() all come from
// int4gemm.hpp (over libi4g.so). Put this directory ahead of the reference's
// include/ on the include path; the harness's own utilities (common.cuh,
// benchmark.cuh, layout.cuh) still come from there.
#pragma once

#include "common.cuh"

#include "../int4gemm.hpp"
