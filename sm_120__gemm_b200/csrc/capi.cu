// The C ABI of include/i4g.h: argument checks, device checks, tensor maps
// and dispatch to the kernels. Nothing here allocates device memory.
#include "../../include/i4g.h"
#include "gemm_tc.h"
#include "ptx.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace {

// Per-device kernel status word: a bounded device-side wait that gives up
// records I4G_ERR_TIMEOUT here (see ptx.cuh, mbar_wait).
__device__ int g_status_word;

constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;  // 2 s

thread_local char t_last_error[512] = "";

struct DeviceInfo {
  bool ready = false;
  int status = I4G_OK;  // I4G_OK or I4G_ERR_DEVICE
  int sm_count = 0;
  int* status_word = nullptr;
};
DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

int record_cuda(cudaError_t e, const char* what) {
  std::snprintf(t_last_error, sizeof(t_last_error), "%s: %s (%s)", what, cudaGetErrorName(e),
                cudaGetErrorString(e));
  return I4G_ERR_CUDA;
}

// Checks the current device once (compute capability 10.0, the sm_100a
// target this library is built for) and caches its SM count and the device
// address of its status word.
int current_device(DeviceInfo** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    std::snprintf(t_last_error, sizeof(t_last_error), "device ordinal %d out of range", dev);
    return I4G_ERR_DEVICE;
  }
  DeviceInfo& info = g_devices[dev];
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (!info.ready) {
    int major = 0, minor = 0, sms = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return record_cuda(e, "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0) {
      std::snprintf(t_last_error, sizeof(t_last_error),
                    "device %d is sm_%d%d; this library is built for sm_100a only", dev, major,
                    minor);
      info.status = I4G_ERR_DEVICE;
    } else {
      void* p = nullptr;
      if ((e = cudaGetSymbolAddress(&p, g_status_word)) != cudaSuccess)
        return record_cuda(e, "cudaGetSymbolAddress(status word)");
      info.status_word = static_cast<int*>(p);
      info.sm_count = sms;
      info.status = I4G_OK;
    }
    info.ready = true;
  }
  if (info.status != I4G_OK) return info.status;
  *out = &info;
  return I4G_OK;
}

int fail(int code, const char* fmt, int a = 0, int b = 0, int c = 0) {
  std::snprintf(t_last_error, sizeof(t_last_error), fmt, a, b, c);
  return code;
}

bool aligned(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

int check_group(int K, int group, bool require_divisible) {
  if (group != 32 && group != 64 && group != 128)
    return fail(I4G_ERR_GROUP, "group %d is not 32, 64 or 128", group);
  if (require_divisible && K % group != 0)
    return fail(I4G_ERR_GROUP, "K=%d is not a multiple of group %d", K, group);
  return I4G_OK;
}

int finish(cudaError_t e, const char* what) {
  return e == cudaSuccess ? I4G_OK : record_cuda(e, what);
}

// ---------------------------------------------------------- tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) {
    if (err != cudaSuccess) return record_cuda(err, "cudaGetDriverEntryPoint");
    return fail(I4G_ERR_DRIVER, "cuTensorMapEncodeTiled is unavailable");
  }
  *out = fn;
  return I4G_OK;
}

// Activation map of A [M][K] fp16, 128-byte swizzle, zero fill past M:
// rows > 0 gives the 2-D box 64 (K) x rows (M) of the tcgen05 kernel; rows < 0
// the 3-D box of four consecutive 64-k blocks x -rows rows of the decode
// kernel. A few recent maps are cached per host thread, keyed by pointer and
// shape, as the reference caches its maps
// (kernels/gemm_v17_instruction.cu:214-228).
struct ActMapEntry {
  int device = -1;
  const void* a = nullptr;
  int M = 0, K = 0, rows = 0;
  unsigned long long used = 0;
  CUtensorMap map;
};

int act_map(const void* A, int M, int K, int rows, const CUtensorMap** out) {
  constexpr int kEntries = 8;
  thread_local ActMapEntry cache[kEntries];
  thread_local unsigned long long clock = 0;
  int dev = -1;
  cudaGetDevice(&dev);
  ++clock;
  ActMapEntry* victim = &cache[0];
  for (ActMapEntry& e : cache) {
    if (e.device == dev && e.a == A && e.M == M && e.K == K && e.rows == rows) {
      e.used = clock;
      *out = &e.map;
      return I4G_OK;
    }
    if (e.used < victim->used) victim = &e;
  }
  EncodeTiledFn encode = nullptr;
  int st = encode_fn(&encode);
  if (st != I4G_OK) return st;
  CUresult r;
  if (rows > 0) {
    // 2-D view [M][K]: box of 64 k x `rows` rows
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(rows)};
    const cuuint32_t estr[2] = {1, 1};
    r = encode(&victim->map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(A), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // 3-D view {64 k, M rows, K/64 blocks}: box of 64 k x -rows rows x 4 blocks
    const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(K / 64)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K) * 2, 128};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(-rows), 4};
    const cuuint32_t estr[3] = {1, 1, 1};
    r = encode(&victim->map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(A), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) {
    victim->device = -1;
    victim->used = 0;
    return fail(I4G_ERR_DRIVER, "cuTensorMapEncodeTiled failed with CUresult %d", int(r));
  }
  victim->device = dev;
  victim->a = A;
  victim->M = M;
  victim->K = K;
  victim->rows = rows;
  victim->used = clock;
  *out = &victim->map;
  return I4G_OK;
}

unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;

using MemRangeFn = int (*)(unsigned long long*, size_t*, unsigned long long);

// Tuning override for the tcgen05 kernel's activation tile (128 or 256
// rows), read once from I4G_TILE_M; 0 means the shape-based choice.
int tile_m_override() {
  static const int v = [] {
    const char* e = std::getenv("I4G_TILE_M");
    const int t = e ? std::atoi(e) : 0;
    return (t == 128 || t == 256) ? t : 0;
  }();
  return v;
}

int check_shape(int M, int N, int K) {
  if (M < 1 || N < 128 || K < 64 || N % 128 != 0 || K % 64 != 0)
    return fail(I4G_ERR_SHAPE,
                "shape M=%d N=%d K=%d: need M >= 1, N %% 128 == 0, K %% 64 == 0", M, N, K);
  if (static_cast<long long>(M) * K >= (1ll << 40) || static_cast<long long>(M) * N >= (1ll << 40))
    return fail(I4G_ERR_SHAPE, "shape M=%d N=%d K=%d too large", M, N, K);
  return I4G_OK;
}

int tc_tile_m(int M, int N, const DeviceInfo* dev) {
  return tile_m_override() ? tile_m_override() : i4g::tc::choose_tile_m(M, N, dev->sm_count);
}

i4g::Outputs single_output(void* C, int N) {
  i4g::Outputs o{};
  o.dst[0] = C;
  o.count = 1;
  o.ldc = N;
  o.col0 = 0;
  return o;
}

// `workspace` (nullable) enables the split-K schedule of the tcgen05 kernel
// when it holds at least the plan's bytes; otherwise the launch is unsplit.
int gemm_common(const void* A, const uint8_t* tiles, const void* scales, const i4g::Outputs& out,
                bool fp32_out, int M, int N, int K, int group, int variant, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (!A || !tiles || !scales) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (out.count < 1 || out.count > i4g::kMaxOutputs)
    return fail(I4G_ERR_SHAPE, "between 1 and %d output copies (got %d)", i4g::kMaxOutputs,
                out.count);
  for (int d = 0; d < out.count; ++d) {
    if (!out.dst[d]) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
    if (!aligned(out.dst[d], fp32_out ? 4 : 2))
      return fail(I4G_ERR_ALIGNMENT, "C must be aligned to its element size");
  }
  if (out.col0 < 0 || out.ldc < out.col0 + N)
    return fail(I4G_ERR_SHAPE, "columns [%d, %d) do not fit rows of %d", out.col0, out.col0 + N,
                out.ldc);
  if (out.count > 1) {
    // peer copies move in 16-byte pieces: every copy, its row stride and the
    // column offset must keep 16-byte alignment
    if (out.ldc % 8 != 0 || out.col0 % 8 != 0)
      return fail(I4G_ERR_ALIGNMENT, "ldc (%d) and col0 (%d) must be multiples of 8 with copies",
                  out.ldc, out.col0);
    for (int d = 0; d < out.count; ++d)
      if (!aligned(out.dst[d], 16))
        return fail(I4G_ERR_ALIGNMENT, "C copies must be 16-byte aligned");
  }
  int st = check_shape(M, N, K);
  if (st != I4G_OK) return st;
  st = check_group(K, group, true);
  if (st != I4G_OK) return st;
  if (!aligned(A, 16) || !aligned(tiles, 16) || !aligned(scales, 16))
    return fail(I4G_ERR_ALIGNMENT, "A, tiles and scales must be 16-byte aligned");
  if (workspace && !aligned(workspace, 256))
    return fail(I4G_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  if (variant != I4G_VARIANT_AUTO && variant != I4G_VARIANT_TC && variant != I4G_VARIANT_DECODE)
    return fail(I4G_ERR_VARIANT, "unknown variant %d", variant);
  if (variant == I4G_VARIANT_AUTO)
    variant = (!fp32_out && i4g::dec::supported(M, K, group)) ? I4G_VARIANT_DECODE
                                                              : I4G_VARIANT_TC;
  if (variant == I4G_VARIANT_DECODE && (fp32_out || M > i4g::dec::MAX_M))
    return fail(I4G_ERR_VARIANT, "decode variant needs M <= %d and an FP16 C (M=%d)",
                i4g::dec::MAX_M, M);
  if (variant == I4G_VARIANT_DECODE && !i4g::dec::supported(M, K, group))
    return fail(I4G_ERR_SHAPE, "decode variant: K=%d too large for its shared memory", K);
  DeviceInfo* dev = nullptr;
  st = current_device(&dev);
  if (st != I4G_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* sc = static_cast<const __half*>(scales);
  if (variant == I4G_VARIANT_DECODE) {
    const CUtensorMap* dmap = nullptr;
    st = act_map(A, M, K, -i4g::dec::rows_for(M), &dmap);
    if (st != I4G_OK) return st;
    return finish(i4g::dec::launch(*dmap, static_cast<const __half*>(A), tiles, sc, out, M, N, K,
                                   group, dev->sm_count,
                                   workspace, workspace ? workspace_bytes : 0,
                                   dev->status_word, g_wait_limit_ns, s),
                  "decode kernel launch");
  }
  const int tile_m = tc_tile_m(M, N, dev);
  const i4g::tc::Plan plan = i4g::tc::make_plan(tile_m, M, N, K, dev->sm_count,
                                                workspace ? workspace_bytes : 0, true,
                                                i4g::tc::max_pairs(dev->sm_count));
  const CUtensorMap* map = nullptr;
  // each CTA of a pair loads half of the tile's activation rows
  st = act_map(A, M, K, tile_m / plan.cg, &map);
  if (st != I4G_OK) return st;
  return finish(i4g::tc::launch(*map, tile_m, tiles, sc, out, fp32_out, M, N, K, group, plan,
                                plan.workspace_bytes > 0 ? workspace : nullptr,
                                dev->status_word, g_wait_limit_ns, s),
                "tcgen05 kernel launch");
}

// A kernel that waits on an mbarrier nothing will complete, through the same
// bounded wait the GEMM kernels use; it must give up and report a timeout.
__global__ void wait_timeout_selftest_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    i4g::mbar_init(i4g::smem_u32(&bar), 1);
    abort_flag = 0;
    i4g::fence_mbarrier_init();
  }
  __syncthreads();
  i4g::mbar_wait(i4g::smem_u32(&bar), 0, reinterpret_cast<volatile int*>(&abort_flag), status,
                 limit_ns);
  __syncthreads();
}

// Cross-GPU barrier over peer-mapped flag arrays (one 64-bit flag per rank in
// every rank's array). Thread t < world (t != rank) stores `epoch` into rank
// t's flag for this rank with release semantics at system scope, then waits
// (acquire, system scope) until this rank's flag for rank t reaches `epoch`.
// The stores a previous kernel on this stream made to peers (fenced at
// system scope by that kernel) are therefore visible to a peer that has
// seen the flag. Every wait is bounded by `limit_ns`; on timeout the status
// word records it and the kernel returns.
struct PeerFlagPtrs {
  unsigned long long* p[i4g::kMaxOutputs];
};

__global__ void peer_barrier_kernel(unsigned long long* local, const __grid_constant__ PeerFlagPtrs peers, int world,
                                    int rank, unsigned long long epoch, int* status,
                                    unsigned long long limit_ns) {
  const int t = static_cast<int>(threadIdx.x);
  if (t >= world || t == rank) return;
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(peers.p[t] + rank), "l"(epoch)
               : "memory");
  const uint64_t t0 = i4g::global_timer_ns();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(local + t) : "memory");
    if (v >= epoch) return;
    if (i4g::global_timer_ns() - t0 > limit_ns) {
      atomicExch(status, i4g::kStatusTimeout);
      return;
    }
    __nanosleep(64);
  }
}

}  // namespace

extern "C" {

const char* i4g_status_string(int status) {
  switch (status) {
    case I4G_OK: return "ok";
    case I4G_ERR_NULL_POINTER: return "null pointer argument";
    case I4G_ERR_SHAPE: return "unsupported shape";
    case I4G_ERR_GROUP: return "unsupported group size";
    case I4G_ERR_ALIGNMENT: return "misaligned pointer";
    case I4G_ERR_CUDA: return "CUDA runtime error";
    case I4G_ERR_DRIVER: return "CUDA driver (tensor map) error";
    case I4G_ERR_DEVICE: return "unsupported device (needs sm_100)";
    case I4G_ERR_TIMEOUT: return "device-side wait timed out";
    case I4G_ERR_VARIANT: return "unsupported kernel variant";
    default: return "unknown status";
  }
}

const char* i4g_last_error(void) { return t_last_error; }

int i4g_layout_version(void) { return 1; }

int i4g_quantize(const void* b, uint8_t* packed, void* scales, int K, int N, int group,
                 void* stream) {
  if (!b || !packed || !scales) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (K < 1 || N < 2 || N % 2 != 0)
    return fail(I4G_ERR_SHAPE, "quantize needs K >= 1 and an even N (K=%d N=%d)", K, N);
  int st = check_group(K, group, false);
  if (st != I4G_OK) return st;
  if (!aligned(b, 4) || !aligned(scales, 2))
    return fail(I4G_ERR_ALIGNMENT, "b must be 4-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::quantize(static_cast<const __half*>(b), packed,
                                    static_cast<__half*>(scales), K, N, group,
                                    static_cast<cudaStream_t>(stream)),
                "quantize launch");
}

int i4g_quantize_repack(const void* b, uint8_t* tiles, void* scales_repacked, int K, int N,
                        int group, void* stream) {
  if (!b || !tiles || !scales_repacked) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  int st = check_group(K, group, true);
  if (st != I4G_OK) return st;
  const int kc = group > 64 ? group : 64;
  if (K < kc || N < 128 || K % kc != 0 || N % 128 != 0)
    return fail(I4G_ERR_SHAPE, "quantize_repack needs K %% %d == 0 and N %% 128 == 0 (K=%d N=%d)",
                kc, K, N);
  if (!aligned(b, 16) || !aligned(tiles, 16) || !aligned(scales_repacked, 2))
    return fail(I4G_ERR_ALIGNMENT, "b and tiles must be 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::quantize_repack(static_cast<const __half*>(b), tiles,
                                           static_cast<__half*>(scales_repacked), K, N, group,
                                           static_cast<cudaStream_t>(stream)),
                "quantize_repack launch");
}

int i4g_dequantize(const uint8_t* packed, const void* scales, void* b, int K, int N, int group,
                   void* stream) {
  if (!b || !packed || !scales) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (K < 1 || N < 2 || N % 2 != 0)
    return fail(I4G_ERR_SHAPE, "dequantize needs K >= 1 and an even N (K=%d N=%d)", K, N);
  int st = check_group(K, group, false);
  if (st != I4G_OK) return st;
  if (N % 8 == 0 && (!aligned(packed, 4) || !aligned(b, 16)))
    return fail(I4G_ERR_ALIGNMENT, "packed must be 4-byte and b 16-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::dequantize(packed, static_cast<const __half*>(scales),
                                      static_cast<__half*>(b), K, N, group,
                                      static_cast<cudaStream_t>(stream)),
                "dequantize launch");
}

static int check_128x32(const void* a, const void* b, int K, int N) {
  if (!a || !b) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (K < 32 || N < 128 || K % 32 != 0 || N % 128 != 0)
    return fail(I4G_ERR_SHAPE, "repack requires K%%32==0 and N%%128==0 (K=%d N=%d)", K, N);
  return I4G_OK;
}

int i4g_repack_128x32(const uint8_t* packed, const void* scales, uint8_t* repacked,
                      void* repacked_scales, int K, int N, int group, void* stream) {
  int st = check_128x32(packed, repacked, K, N);
  if (st != I4G_OK) return st;
  if (!scales || !repacked_scales) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if ((st = check_group(K, group, true)) != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = i4g::prep::repack_128x32(packed, repacked, K, N, s);
  if (e == cudaSuccess)
    e = i4g::prep::repack_scales_128(static_cast<const __half*>(scales),
                                     static_cast<__half*>(repacked_scales), K, N, group, s);
  return finish(e, "repack launch");
}

int i4g_inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed, int K, int N,
                              void* stream) {
  int st = check_128x32(repacked, packed, K, N);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::inverse_repack_128x32(repacked, packed, K, N,
                                                 static_cast<cudaStream_t>(stream)),
                "inverse repack launch");
}

int i4g_repack_mma_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N, void* stream) {
  int st = check_128x32(packed, repacked, K, N);
  if (st != I4G_OK) return st;
  if (!aligned(repacked, 2)) return fail(I4G_ERR_ALIGNMENT, "repacked must be 2-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::repack_mma_128x32(packed, repacked, K, N,
                                             static_cast<cudaStream_t>(stream)),
                "mma repack launch");
}

int i4g_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                               void* stream) {
  int st = check_128x32(packed, repacked, K, N);
  if (st != I4G_OK) return st;
  if (!aligned(repacked, 4)) return fail(I4G_ERR_ALIGNMENT, "repacked must be 4-byte aligned");
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::repack_mma_pair_128x32(packed, repacked, K, N,
                                                  static_cast<cudaStream_t>(stream)),
                "mma pair repack launch");
}

int i4g_repack_scales_128(const void* scales, void* repacked_scales, int K, int N, int group,
                          void* stream) {
  if (!scales || !repacked_scales) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (N < 128 || N % 128 != 0 || K < 1)
    return fail(I4G_ERR_SHAPE, "scale repack requires N%%128==0 (K=%d N=%d)", K, N);
  int st = check_group(K, group, true);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::repack_scales_128(static_cast<const __half*>(scales),
                                             static_cast<__half*>(repacked_scales), K, N, group,
                                             static_cast<cudaStream_t>(stream)),
                "scale repack launch");
}

static int check_umma(const void* a, const void* b, int K, int N) {
  if (!a || !b) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (K < 64 || N < 128 || K % 64 != 0 || N % 128 != 0)
    return fail(I4G_ERR_SHAPE, "tile layout requires K%%64==0 and N%%128==0 (K=%d N=%d)", K, N);
  if (!aligned(a, 16) || !aligned(b, 16))
    return fail(I4G_ERR_ALIGNMENT, "tile layout buffers must be 16-byte aligned");
  return I4G_OK;
}

int i4g_repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N, void* stream) {
  int st = check_umma(packed, tiles, K, N);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::repack_umma(packed, tiles, K, N, static_cast<cudaStream_t>(stream)),
                "tile repack launch");
}

int i4g_inverse_repack_umma(const uint8_t* tiles, uint8_t* packed, int K, int N, void* stream) {
  int st = check_umma(tiles, packed, K, N);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  return finish(i4g::prep::inverse_repack_umma(tiles, packed, K, N,
                                               static_cast<cudaStream_t>(stream)),
                "inverse tile repack launch");
}

int i4g_gemm(const void* A, const uint8_t* tiles, const void* scales, void* C, int M, int N,
             int K, int group, void* stream) {
  return gemm_common(A, tiles, scales, single_output(C, N), false, M, N, K, group,
                     I4G_VARIANT_AUTO, nullptr, 0, stream);
}

int i4g_gemm_fp32(const void* A, const uint8_t* tiles, const void* scales, float* C, int M,
                  int N, int K, int group, void* stream) {
  return gemm_common(A, tiles, scales, single_output(C, N), true, M, N, K, group,
                     I4G_VARIANT_TC, nullptr, 0, stream);
}

int i4g_gemm_variant(const void* A, const uint8_t* tiles, const void* scales, void* C, int M,
                     int N, int K, int group, int variant, void* stream) {
  return gemm_common(A, tiles, scales, single_output(C, N), false, M, N, K, group, variant,
                     nullptr, 0, stream);
}

int i4g_gemm_workspace_size(int M, int N, int K, size_t* bytes) {
  if (!bytes) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  *bytes = 0;
  int st = check_shape(M, N, K);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  *bytes = i4g::tc::make_plan(tc_tile_m(M, N, dev), M, N, K, dev->sm_count, SIZE_MAX, true,
                              i4g::tc::max_pairs(dev->sm_count))
               .workspace_bytes;
  if (i4g::dec::supported(M, K, 32) &&  // FP16 C at these M runs the decode kernel
      i4g::dec::pick_schedule(M, N, K, dev->sm_count, SIZE_MAX) == i4g::dec::kScheduleStreamK) {
    const i4g::dec::SkPlan sk = i4g::dec::sk_plan(M, N, K, dev->sm_count);
    if (sk.workspace_bytes > *bytes) *bytes = sk.workspace_bytes;
  }
  return I4G_OK;
}

int i4g_gemm_ws(const void* A, const uint8_t* tiles, const void* scales, void* C, int M, int N,
                int K, int group, void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_common(A, tiles, scales, single_output(C, N), false, M, N, K, group,
                     I4G_VARIANT_AUTO, workspace, workspace_bytes, stream);
}

int i4g_gemm_fp32_ws(const void* A, const uint8_t* tiles, const void* scales, float* C, int M,
                     int N, int K, int group, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return gemm_common(A, tiles, scales, single_output(C, N), true, M, N, K, group,
                     I4G_VARIANT_TC, workspace, workspace_bytes, stream);
}

int i4g_gemm_static_scratch(const void* A, const uint8_t* tiles, const void* scales, void* C,
                            int M, int N, int K, int group, void* stream) {
  int st = check_shape(M, N, K);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  size_t need = 0;
  if (!i4g::dec::supported(M, K, group)) {
    need = i4g::tc::make_plan(tc_tile_m(M, N, dev), M, N, K, dev->sm_count, SIZE_MAX, true,
                              i4g::tc::max_pairs(dev->sm_count))
               .workspace_bytes;
  } else {
    // the decode kernel's stream-K schedule when it is the one chosen and its
    // workspace fits the static scratch; the slice and cluster schedules
    // need none
    if (i4g::dec::pick_schedule(M, N, K, dev->sm_count, i4g::static_scratch_bytes()) ==
        i4g::dec::kScheduleStreamK)
      need = i4g::dec::sk_plan(M, N, K, dev->sm_count).workspace_bytes;
  }
  if (need > i4g::static_scratch_bytes()) {
    std::snprintf(t_last_error, sizeof(t_last_error),
                  "shape M=%d N=%d K=%d needs %zu bytes of split-K scratch; the static scratch "
                  "holds %zu",
                  M, N, K, need, i4g::static_scratch_bytes());
    return I4G_ERR_SHAPE;
  }
  void* scratch = nullptr;
  if (need > 0) {
    cudaError_t e = i4g::static_scratch(&scratch);
    if (e != cudaSuccess) return record_cuda(e, "cudaGetSymbolAddress(static scratch)");
    // The arrival counters must be zero when the kernel starts. Completed
    // launches leave them so; clearing them here keeps a launch that gave up
    // on a device-side wait from corrupting the next call.
    e = cudaMemsetAsync(scratch, 0, i4g::tc::kTicketBytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda(e, "clearing the static scratch counters");
  }
  return gemm_common(A, tiles, scales, single_output(C, N), false, M, N, K, group,
                     I4G_VARIANT_AUTO, scratch, need, stream);
}

int i4g_gemm_to_peers(const void* A, const uint8_t* tiles, const void* scales, void* const* dsts,
                      int ndst, int ldc, int col0, int M, int N, int K, int group,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!dsts) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (ndst < 1 || ndst > i4g::kMaxOutputs)
    return fail(I4G_ERR_SHAPE, "between 1 and %d output copies (got %d)", i4g::kMaxOutputs,
                ndst);
  i4g::Outputs out{};
  for (int d = 0; d < ndst; ++d) out.dst[d] = dsts[d];
  out.count = ndst;
  out.ldc = ldc;
  out.col0 = col0;
  return gemm_common(A, tiles, scales, out, false, M, N, K, group, I4G_VARIANT_AUTO, workspace,
                     workspace_bytes, stream);
}

int i4g_ipc_handle(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  static MemRangeFn range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range = reinterpret_cast<MemRangeFn>(p);
  });
  if (!range) return fail(I4G_ERR_DRIVER, "cuMemGetAddressRange is unavailable");
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return fail(I4G_ERR_DRIVER, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return record_cuda(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<unsigned long long>(ptr) - base;
  return I4G_OK;
}

int i4g_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? I4G_OK : record_cuda(e, "cudaIpcOpenMemHandle");
}

int i4g_ipc_close(void* base) {
  if (!base) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? I4G_OK : record_cuda(e, "cudaIpcCloseMemHandle");
}

int i4g_shard_range(int K, int N, int group, int world, int rank, size_t* tile_offset,
                    size_t* scale_offset, int* n0, int* n1) {
  if (!tile_offset || !scale_offset || !n0 || !n1)
    return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (world < 1 || rank < 0 || rank >= world)
    return fail(I4G_ERR_SHAPE, "rank %d out of range for world %d", rank, world);
  if (K < 64 || K % 64 != 0 || N < 128 || N % (128 * world) != 0)
    return fail(I4G_ERR_SHAPE, "N=%d must split into %d multiples of 128 (K=%d)", N, world, K);
  int st = check_group(K, group, true);
  if (st != I4G_OK) return st;
  const int n_local = N / world;
  *n0 = rank * n_local;
  *n1 = *n0 + n_local;
  const size_t first_tile = static_cast<size_t>(*n0 / 128);
  *tile_offset = first_tile * static_cast<size_t>(K / 64) * 4096;
  *scale_offset = first_tile * static_cast<size_t>(K / group) * 128 * 2;
  return I4G_OK;
}

int i4g_device_status(int* out, void* stream) {
  if (!out) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != I4G_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyAsync(&value, dev->status_word, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dev->status_word, 0, sizeof(int), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return record_cuda(e, "reading the device status word");
  *out = value;
  return I4G_OK;
}

int i4g_plan(int M, int N, int K, int group, int fp32_out, int sm_count,
             size_t workspace_bytes, int* kernel, int* schedule, int* param, size_t* bytes) {
  if (!kernel || !schedule || !param || !bytes)
    return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  int st = check_shape(M, N, K);
  if (st != I4G_OK) return st;
  st = check_group(K, group, true);
  if (st != I4G_OK) return st;
  if (sm_count < 1 || sm_count > 4096) return fail(I4G_ERR_SHAPE, "sm_count %d", sm_count);
  // the same choices as gemm_common and the kernels' launchers
  if (!fp32_out && i4g::dec::supported(M, K, group)) {
    *kernel = I4G_PLAN_KERNEL_DECODE;
    const i4g::dec::SkPlan sk = i4g::dec::sk_plan(M, N, K, sm_count);
    const int sched = i4g::dec::pick_schedule(M, N, K, sm_count, workspace_bytes);
    if (sched == i4g::dec::kScheduleSlices) {
      *schedule = I4G_PLAN_SLICES;
      *param = i4g::dec::slice_grid(N, sm_count);
      *bytes = 0;
    } else if (sched == i4g::dec::kScheduleStreamK) {
      *schedule = I4G_PLAN_STREAMK;
      *param = sk.grid;
      *bytes = sk.workspace_bytes;
    } else {
      *schedule = I4G_PLAN_CLUSTER;
      *param = i4g::dec::choose_cluster(N, K, sm_count);
      *bytes = 0;
    }
    return I4G_OK;
  }
  const int tile_m =
      tile_m_override() ? tile_m_override() : i4g::tc::choose_tile_m(M, N, sm_count);
  const i4g::tc::Plan plan = i4g::tc::make_plan(tile_m, M, N, K, sm_count, workspace_bytes, true);
  *kernel = tile_m == 128 ? I4G_PLAN_KERNEL_TC128 : I4G_PLAN_KERNEL_TC256;
  *bytes = plan.workspace_bytes;
  if (plan.sched.chunks > 0) {
    *schedule = I4G_PLAN_STREAMK;
    *param = plan.sched.chunks;
  } else if (plan.sched.split > 1) {
    *schedule = I4G_PLAN_SPLIT;
    *param = plan.sched.split;
  } else {
    *schedule = I4G_PLAN_WHOLE;
    *param = plan.grid;
  }
  return I4G_OK;
}

static int kernel_instance(int variant, int rows, int group) {
  int st = check_group(group, group, false);
  if (st != I4G_OK) return st;
  if (variant == I4G_VARIANT_TC && (rows == 128 || rows == 256)) return I4G_OK;
  if (variant == I4G_VARIANT_DECODE && (rows == 8 || rows == 16)) return I4G_OK;
  return fail(I4G_ERR_VARIANT, "no kernel instance for variant %d with %d rows", variant, rows);
}

int i4g_kernel_config(int variant, int rows, int group, i4g_kernel_config_t* out) {
  if (!out) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  int st = kernel_instance(variant, rows, group);
  if (st != I4G_OK) return st;
  i4g::KernelConfig c{};
  const bool ok = variant == I4G_VARIANT_TC ? i4g::tc::config(rows, group, &c)
                                            : i4g::dec::config(rows, group, &c);
  if (!ok) return fail(I4G_ERR_VARIANT, "no kernel instance for %d rows", rows);
  *out = i4g_kernel_config_t{c.rows, c.cols, c.bk, c.mma_m, c.mma_n, c.stages, c.threads,
                             c.dynamic_smem};
  return I4G_OK;
}

int i4g_kernel_resources(int variant, int rows, int group, i4g_kernel_resources_t* out) {
  if (!out) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  int st = kernel_instance(variant, rows, group);
  if (st != I4G_OK) return st;
  DeviceInfo* dev = nullptr;
  if ((st = current_device(&dev)) != I4G_OK) return st;
  i4g::KernelResources r{};
  const cudaError_t e = variant == I4G_VARIANT_TC ? i4g::tc::resources(rows, group, &r)
                                                  : i4g::dec::resources(rows, group, &r);
  if (e != cudaSuccess) return record_cuda(e, "kernel attribute query");
  *out = i4g_kernel_resources_t{r.registers, r.static_smem, r.max_threads, r.active_per_sm};
  return I4G_OK;
}

int i4g_max_pairs(int* pairs) {
  if (!pairs) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  DeviceInfo* dev = nullptr;
  const int st = current_device(&dev);
  if (st != I4G_OK) return st;
  *pairs = i4g::tc::max_pairs(dev->sm_count);
  return I4G_OK;
}

int i4g_set_decode_schedule(int schedule) {
  if (schedule != I4G_DECODE_AUTO && schedule != I4G_DECODE_CLUSTER &&
      schedule != I4G_DECODE_STREAMK && schedule != I4G_DECODE_SLICES)
    return fail(I4G_ERR_VARIANT, "unknown decode schedule %d", schedule);
  static_assert(I4G_DECODE_AUTO == i4g::dec::kScheduleAuto &&
                    I4G_DECODE_CLUSTER == i4g::dec::kScheduleCluster &&
                    I4G_DECODE_STREAMK == i4g::dec::kScheduleStreamK &&
                    I4G_DECODE_SLICES == i4g::dec::kScheduleSlices,
                "decode schedule codes");
  i4g::dec::set_schedule(schedule);
  return I4G_OK;
}

int i4g_peer_barrier(unsigned long long* local_flags, unsigned long long* const* peer_flags,
                     int world, int rank, unsigned long long epoch,
                     unsigned long long limit_ns, void* stream) {
  if (!local_flags || !peer_flags) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
  if (world < 1 || world > i4g::kMaxOutputs || rank < 0 || rank >= world)
    return fail(I4G_ERR_SHAPE, "rank %d of world %d (at most %d ranks)", rank, world,
                i4g::kMaxOutputs);
  if (epoch == 0) return fail(I4G_ERR_SHAPE, "epoch must be positive");
  if (!aligned(local_flags, 8)) return fail(I4G_ERR_ALIGNMENT, "flags must be 8-byte aligned");
  PeerFlagPtrs peers{};
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    if (!peer_flags[r]) return fail(I4G_ERR_NULL_POINTER, "null pointer argument");
    if (!aligned(peer_flags[r], 8)) return fail(I4G_ERR_ALIGNMENT, "flags must be 8-byte aligned");
    peers.p[r] = peer_flags[r];
  }
  DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != I4G_OK) return st;
  const unsigned long long limit = limit_ns ? limit_ns : g_wait_limit_ns;
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      local_flags, peers, world, rank, epoch, dev->status_word, limit);
  return finish(cudaGetLastError(), "peer barrier launch");
}

int i4g_selftest_wait_timeout(unsigned long long limit_ns, void* stream) {
  DeviceInfo* dev = nullptr;
  int st = current_device(&dev);
  if (st != I4G_OK) return st;
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(I4G_ERR_SHAPE, "limit must be in (0, 1 s]");
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status_word,
                                                                                limit_ns);
  return finish(cudaGetLastError(), "self-test launch");
}

}  // extern "C"
