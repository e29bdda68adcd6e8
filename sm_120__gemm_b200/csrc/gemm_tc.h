// Host-side interface of the kernels (not part of the public C ABI).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdlib>
#include <cstdint>

namespace i4g {

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per device: the attribute belongs to the kernel's instance on
// each device, so a process that drives several GPUs sets it on every one.
// `done` is the kernel's bitmask of devices already set (thread-safe;
// setting the attribute twice is harmless).
template <typename Kernel>
cudaError_t ensure_dynamic_smem(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t{1} << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// The GEMM kernels are launched as programmatic dependents of the kernel
// before them on the stream (they may start while it runs, and wait for it
// before touching A, C or a workspace), unless I4G_PDL=0 (read once).
inline bool pdl_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("I4G_PDL");
    return !(e && e[0] == '0' && e[1] == 0);
  }();
  return v;
}

// Where a launch writes C: `count` copies (this GPU's, then peers' through
// peer-mapped pointers), each a row-major [M][ldc] matrix of which the launch
// fills columns [col0, col0 + N). count == 1, ldc == N, col0 == 0 is the plain
// GEMM.
constexpr int kMaxOutputs = 8;
struct Outputs {
  void* dst[kMaxOutputs];
  int count;
  int ldc;
  int col0;
};

// Static configuration and device resources of one kernel instance, for the
// registry queries of the C ABI (i4g_kernel_config / i4g_kernel_resources).
struct KernelConfig {
  int rows, cols, bk;        // activation rows, weight columns, k per stage
  int mma_m, mma_n;          // tensor-core instruction shape (weights x rows)
  int stages, threads, dynamic_smem;
};
struct KernelResources {
  int registers, static_smem, max_threads, active_per_sm;
};

namespace tc {
// Arrival counters (tickets) at the start of a split-K workspace, then the
// FP32 partials; the decode kernel's stream-K schedule uses the same layout.
constexpr size_t kTicketBytes = 4096;

// Work schedule of one launch (device-visible): `full_tiles` whole tiles,
// then the tail. chunks == 0: each of the following tiles split `split` ways
// along K (items = full_tiles + tail * split). chunks > 0 (stream-K): the
// `tail_tiles` tiles' blocks cut into `chunks` equal shares, one per CTA.
// promo > 0: an item's accumulation is cut into segments of `promo` 64-k
// blocks, each promoted into an FP32 running sum by the epilogue (0: none).
struct Sched {
  int full_tiles, split, items, chunks, tail_tiles, promo;
};

// 64-k blocks per promotion segment of the tcgen05 kernel (default 32, i.e.
// 2048 k; I4G_PROMOTE_BLOCKS overrides it, 0 switches promotion off).
int promote_blocks();

struct Plan {
  Sched sched;
  int grid;                // CTAs
  int cg;                  // CTAs per tile: 1, or 2 (a CTA pair, cluster of two)
  size_t workspace_bytes;  // 0 when nothing is split
};
// CTAs per tile the plan for these sizes uses (activation rows per CTA: tile_m / cg).
int choose_cg(int tile_m, int N, int sm_count);
// The schedule for a workspace of `budget` bytes (0: none): stream-K when it
// fits (and allow_stream_k), else equal splits when they fit, else whole tiles.
// pairs: CTA pairs resident at once on the device (max_pairs; 0: sm_count / 2).
Plan make_plan(int tile_m, int M, int N, int K, int sm_count, size_t budget,
               bool allow_stream_k, int pairs = 0);
// CTA pairs of the paired kernel that fit on the current device at once.
int max_pairs(int sm_count);

// TILE_M (activation rows per tile, the MMA-N) for a problem on sm_count SMs.
int choose_tile_m(int M, int N, int sm_count);
// The FP16-C instance for tile_m (128 or 256) and group (32, 64, 128);
// resources() needs a current device.
bool config(int tile_m, int group, KernelConfig* out);
cudaError_t resources(int tile_m, int group, KernelResources* out);
cudaError_t launch(const CUtensorMap& act_map, int tile_m, const uint8_t* tiles,
                   const __half* scales, const Outputs& out, bool fp32_out, int M, int N, int K,
                   int group, const Plan& plan, void* workspace, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream);
}  // namespace tc

namespace dec {
constexpr int MAX_M = 16;
// Whether the decode kernel serves this M, K, group.
bool supported(int M, int K, int group);
// Rows of the activation box the decode kernel's tensor map must use.
int rows_for(int M);
// Stream-K schedule of the decode kernel for a workspace (grid 0: not
// possible); `preferred` when its busiest SM does less work than under the
// cluster schedule.
struct SkPlan {
  int grid;
  size_t workspace_bytes;
  bool preferred;
};
SkPlan sk_plan(int M, int N, int K, int sm_count);
// Cluster size of the cluster schedule (K split of each column tile).
int choose_cluster(int N, int K, int sm_count);
// The cluster-schedule instance for rows (8: M <= 8, 16: M <= 16) and group.
bool config(int rows, int group, KernelConfig* out);
cudaError_t resources(int rows, int group, KernelResources* out);
constexpr int kScheduleAuto = 0, kScheduleCluster = 1, kScheduleStreamK = 2, kScheduleSlices = 3;
// The slice schedule: CTA c of `slice_grid` owns 16-column slices
// [c*S/G, (c+1)*S/G) of the S = N/16 slices over all of K (no reduction
// across CTAs). Possible when every CTA owns at most kSliceMax slices.
constexpr int kSliceMax = 8;
int slice_grid(int N, int sm_count);  // 0: not possible
// The schedule launch() runs for this shape (given a workspace of
// workspace_bytes), under the current set_schedule choice.
int pick_schedule(int M, int N, int K, int sm_count, size_t workspace_bytes);
void set_schedule(int mode);
// Launches the stream-K schedule when `workspace` holds sk_plan's bytes and
// it is preferred, else the cluster schedule (no workspace).
// A: the activation rows (read directly by the slice schedule; the others
// read them through act_map).
cudaError_t launch(const CUtensorMap& act_map, const __half* A, const uint8_t* tiles,
                   const __half* scales, const Outputs& out, int M, int N, int K, int group,
                   int sm_count, void* workspace, size_t workspace_bytes, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream);
}  // namespace dec

namespace prep {
// quantize + repack_umma + repack_scales_128 in one pass over B.
// K % max(64, group) == 0, N % 128 == 0.
cudaError_t quantize_repack(const __half* b, uint8_t* tiles, __half* rscales, int K, int N,
                            int group, cudaStream_t stream);
cudaError_t quantize(const __half* b, uint8_t* packed, __half* scales, int K, int N, int group,
                     cudaStream_t stream);
cudaError_t dequantize(const uint8_t* packed, const __half* scales, __half* b, int K, int N,
                       int group, cudaStream_t stream);
cudaError_t repack_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                          cudaStream_t stream);
cudaError_t inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed, int K, int N,
                                  cudaStream_t stream);
cudaError_t repack_scales_128(const __half* scales, __half* repacked, int K, int N, int group,
                              cudaStream_t stream);
cudaError_t repack_mma_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                              cudaStream_t stream);
cudaError_t repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                                   cudaStream_t stream);
cudaError_t repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N,
                        cudaStream_t stream);
cudaError_t inverse_repack_umma(const uint8_t* tiles, uint8_t* packed, int K, int N,
                                cudaStream_t stream);
}  // namespace prep

// Fixed-size split-K scratch in static device memory (static_scratch.cu):
// its size, and its device address on the current device.
size_t static_scratch_bytes();
cudaError_t static_scratch(void** out);
}  // namespace i4g
