// Fused W4A16 GEMM for sm_100a: tcgen05 tensor cores, TMEM accumulators,
// TMA-fed activations, INT4 weights dequantised straight into TMEM.
//
// Replaces the reference's production path launch_final -> v17_kernel
// (kernels/gemm_final.cu:5-13, kernels/gemm_v17_instruction.cu:275-555),
// which is an sm_120 mma.sync kernel. Same product: C = A x dequant(B) with
// FP32 accumulation and an FP16 (or FP32) C.
//
// Formulation (swap-AB). The MMA computes D[n][m] = sum_k W[n][k] * A[m][k]:
//   MMA-M = 128 weight columns n      operand A from TMEM (dequantised here)
//   MMA-N = TILE_M activation rows m  operand B from SMEM (TMA, 128B swizzle)
//   D     = TILE_M fp32 TMEM columns, double-buffered so the epilogue of one
//           tile overlaps the main loop of the next.
// Putting the weights on the MMA-M side means every dequantised weight is
// used by TILE_M activation rows, and the dequantised FP16 values never touch
// shared memory: each dequant thread owns one TMEM lane (one weight column)
// and writes it with tcgen05.st.
//
// Warp roles (448 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: activation box + packed weight block + scales
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warps 2-9   dequant: smem nibbles -> half(q*s) -> TMEM weight stage
//   warps 10-13 epilogue: TMEM -> registers -> FP16 -> global C
//
// Pipelines (all mbarrier based, every wait bounded):
//   full[s]/empty[s]    smem stages (activation, packed weights, scales)
//   wfull[w]/wempty[w]  TMEM weight stages (32 columns = 64 k each)
//   afull[a]/aempty[a]  TMEM accumulators
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_runtime.h>

namespace i4g {
namespace tc {

constexpr int TILE_N = 128;         // weight columns per tile (MMA-M)
constexpr int BK = 64;              // k per stage (one 128-byte swizzle row)
constexpr int W_STAGES = 4;         // TMEM weight stages
constexpr int W_COLS = 32;          // TMEM columns per weight stage (64 halves)
constexpr int NUM_DEQ_WARPS = 8;
constexpr int NUM_EPI_WARPS = 4;
constexpr int THREADS = 32 * (2 + NUM_DEQ_WARPS + NUM_EPI_WARPS);
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL0 = W_STAGES * W_COLS;  // 128
constexpr int WBLOCK_BYTES = TILE_N * BK / 2;  // 4096: one tile-layout block
constexpr int SCALE_BYTES = 512;            // up to two groups x 128 halves
constexpr int GROUP_M = 16;                 // rasterisation band (m-tiles)

template <int TILE_M>
struct Smem {
  static constexpr int ACT_BYTES = TILE_M * BK * 2;
  static constexpr int STAGES = TILE_M >= 192 ? 6 : (TILE_M >= 128 ? 8 : 10);
  static constexpr int ACT_OFF = 0;
  static constexpr int W_OFF = ACT_OFF + STAGES * ACT_BYTES;
  static constexpr int S_OFF = W_OFF + STAGES * WBLOCK_BYTES;
  static constexpr int BAR_OFF = S_OFF + STAGES * SCALE_BYTES;
  // barriers: full, empty (STAGES each), wfull, wempty (W_STAGES each),
  // afull, aempty (2 each), drain (1)
  static constexpr int NUM_BARS = 2 * STAGES + 2 * W_STAGES + 4 + 1;
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int TOTAL = MISC_OFF + 16;
  static constexpr int DYN_BYTES = TOTAL + 1024;  // slack for 1024-byte alignment
  static_assert(ACT_BYTES % 1024 == 0, "activation stage must keep 1024B alignment");
  static_assert(2 * TILE_M + ACC_COL0 <= TMEM_COLS, "TMEM budget");
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mt, int& nt) {
  // Bands of GROUP_M m-tiles, walked n-major inside a band, so that the
  // activation rows of a band and a run of weight blocks stay in L2.
  const int band_tiles = GROUP_M * num_n;
  const int band = tile / band_tiles;
  const int first_m = band * GROUP_M;
  const int band_m = min(GROUP_M, num_m - first_m);
  const int within = tile - band * band_tiles;
  mt = first_m + within % band_m;
  nt = within / band_m;
}

template <int TILE_M, int GROUP, bool FP32_OUT>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap act_map,
                   const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                   void* __restrict__ c_out, int M, int N, int K, int* status,
                   unsigned long long wait_limit_ns) {
  using L = Smem<TILE_M>;
  constexpr int STAGES = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const uint32_t act_base = smem_u32(smem + L::ACT_OFF);
  const uint32_t w_base = smem_u32(smem + L::W_OFF);
  const uint32_t s_base = smem_u32(smem + L::S_OFF);
  const uint32_t bar_base = smem_u32(smem + L::BAR_OFF);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto wfull_bar = [&](int w) { return bar_base + 8u * (2 * STAGES + w); };
  auto wempty_bar = [&](int w) { return bar_base + 8u * (2 * STAGES + W_STAGES + w); };
  auto afull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 * W_STAGES + a); };
  auto aempty_bar = [&](int a) {
    return bar_base + 8u * (2 * STAGES + 2 * W_STAGES + 2 + a);
  };
  const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 2 * W_STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + TILE_M - 1) / TILE_M;
  const int num_n = N / TILE_N;
  const int num_tiles = num_m * num_n;
  const int kblocks = K / BK;
  const int groups = K / GROUP;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1 + NUM_DEQ_WARPS);
    }
    for (int w = 0; w < W_STAGES; ++w) {
      mbar_init(wfull_bar(w), NUM_DEQ_WARPS * 32);
      mbar_init(wempty_bar(w), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(afull_bar(a), 1);
      mbar_init(aempty_bar(a), NUM_EPI_WARPS * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&act_map);
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      int last_issue[16];
      for (int s = 0; s < STAGES; ++s) last_issue[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, num_m, num_n, mt, nt);
        const uint8_t* wblk = tiles + static_cast<size_t>(nt) * kblocks * WBLOCK_BYTES;
        const __half* sblk = scales + static_cast<size_t>(nt) * groups * TILE_N;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, status, wait_limit_ns)) {
            ok = false;
            break;
          }
          int g0, sbytes;
          if (GROUP == 32) { g0 = 2 * kb; sbytes = 512; }
          else if (GROUP == 64) { g0 = kb; sbytes = 256; }
          else { g0 = kb >> 1; sbytes = 256; }
          mbar_arrive_expect_tx(full_bar(s), L::ACT_BYTES + WBLOCK_BYTES + sbytes);
          tma_load_2d(act_base + s * L::ACT_BYTES, &act_map, full_bar(s), kb * BK, mt * TILE_M);
          bulk_load(w_base + s * WBLOCK_BYTES, wblk + static_cast<size_t>(kb) * WBLOCK_BYTES,
                    WBLOCK_BYTES, full_bar(s));
          bulk_load(s_base + s * SCALE_BYTES, sblk + static_cast<size_t>(g0) * TILE_N, sbytes,
                    full_bar(s));
          last_issue[s] = static_cast<int>(it);
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (last_issue[s] >= 0) {
            volatile int never = 0;
            mbar_wait(full_bar(s), (static_cast<uint32_t>(last_issue[s]) / STAGES) & 1u, &never,
                      nullptr, 100000000ull);
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_f16_f32(TILE_N, TILE_M);
      uint32_t it = 0, t_local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t aph = (t_local >> 1) & 1u;
        if (!mbar_wait(aempty_bar(acc), aph ^ 1u, abort_flag, status, wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ACC_COL0 + acc * TILE_M;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          const int ws = it % W_STAGES;
          const uint32_t wph = (it / W_STAGES) & 1u;
          if (!mbar_wait(full_bar(s), ph, abort_flag, status, wait_limit_ns) ||
              !mbar_wait(wfull_bar(ws), wph, abort_flag, status, wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = act_base + s * L::ACT_BYTES;
#pragma unroll
          for (int k16 = 0; k16 < BK / 16; ++k16) {
            const uint32_t a_tmem = tmem_base + ws * W_COLS + k16 * 8;
            const uint64_t b_desc = smem_desc_sw128(b_addr + k16 * 32);
            mma_f16_ts(d_tmem, a_tmem, b_desc, IDESC, (kb | k16) != 0);
          }
          tc_commit(empty_bar(s));
          tc_commit(wempty_bar(ws));
        }
        if (!ok) break;
        tc_commit(afull_bar(acc));
      }
      // Drain: every MMA this thread issued has completed before TMEM is freed.
      tc_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, nullptr, 100000000ull);
    }
  } else if (warp < 2 + NUM_DEQ_WARPS) {
    // ---------------------------------------------------------------- dequant
    const int d = warp - 2;
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int h = d / 4;                   // which 32 of the 64 k in a stage
    const int row = quarter * 32 + lane;   // weight column inside the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1u;
        const int ws = it % W_STAGES;
        const uint32_t wph = (it / W_STAGES) & 1u;
        if (!mbar_wait(full_bar(s), ph, abort_flag, status, wait_limit_ns)) {
          ok = false;
          break;
        }
        uint4 codes;
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(codes.x), "=r"(codes.y), "=r"(codes.z), "=r"(codes.w)
                     : "r"(w_base + s * WBLOCK_BYTES + h * 2048 + row * 16));
        const int gl = (GROUP == 32) ? h : 0;
        uint16_t sbits;
        asm volatile("ld.shared.u16 %0, [%1];"
                     : "=h"(sbits)
                     : "r"(s_base + s * SCALE_BYTES + (gl * TILE_N + row) * 2));
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));
        const uint32_t s2 = half_bits_x2(sbits);
        uint32_t r[16];
        const uint32_t wv[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          r[4 * i + 0] = decode_pair<0>(wv[i], s2);
          r[4 * i + 1] = decode_pair<1>(wv[i], s2);
          r[4 * i + 2] = decode_pair<2>(wv[i], s2);
          r[4 * i + 3] = decode_pair<3>(wv[i], s2);
        }
        if (!mbar_wait(wempty_bar(ws), wph ^ 1u, abort_flag, status, wait_limit_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_32x32b_x16(tmem_base + lane_addr + ws * W_COLS + h * 16, r);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(wfull_bar(ws));
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t t_local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t_local) {
      int mt, nt;
      tile_coords(tile, num_m, num_n, mt, nt);
      const int acc = t_local & 1;
      const uint32_t aph = (t_local >> 1) & 1u;
      if (!mbar_wait(afull_bar(acc), aph, abort_flag, status, wait_limit_ns)) break;
      tc_fence_after();
      const int n = nt * TILE_N + row;
#pragma unroll 1
      for (int c = 0; c < TILE_M / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + ACC_COL0 + acc * TILE_M + c * 32, v);
        tmem_ld_wait(v);
        const int m0 = mt * TILE_M + c * 32;
        if constexpr (FP32_OUT) {
          float* cp = static_cast<float*>(c_out) + static_cast<size_t>(m0) * N + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (m0 + j < M) cp[static_cast<size_t>(j) * N] = __uint_as_float(v[j]);
        } else {
          __half* cp = static_cast<__half*>(c_out) + static_cast<size_t>(m0) * N + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (m0 + j < M) cp[static_cast<size_t>(j) * N] = __float2half_rn(__uint_as_float(v[j]));
        }
      }
      tc_fence_before();
      mbar_arrive(aempty_bar(acc));
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host

template <int TILE_M, int GROUP, bool FP32_OUT>
cudaError_t launch_impl(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                        void* c, int M, int N, int K, int sm_count, int* status,
                        unsigned long long wait_limit_ns, cudaStream_t stream) {
  using L = Smem<TILE_M>;
  auto kernel = gemm_tc_kernel<TILE_M, GROUP, FP32_OUT>;
  static bool configured = false;  // per instantiation; idempotent attribute
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::DYN_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int num_tiles = ((M + TILE_M - 1) / TILE_M) * (N / TILE_N);
  const int grid = num_tiles < sm_count ? num_tiles : sm_count;
  kernel<<<grid, THREADS, L::DYN_BYTES, stream>>>(act_map, tiles, scales, c, M, N, K, status,
                                                  wait_limit_ns);
  return cudaGetLastError();
}

template <int TILE_M, bool FP32_OUT>
cudaError_t launch_group(const CUtensorMap& act_map, const uint8_t* tiles,
                         const __half* scales, void* c, int M, int N, int K, int group,
                         int sm_count, int* status, unsigned long long wait_limit_ns,
                         cudaStream_t stream) {
  switch (group) {
    case 32:
      return launch_impl<TILE_M, 32, FP32_OUT>(act_map, tiles, scales, c, M, N, K, sm_count,
                                               status, wait_limit_ns, stream);
    case 64:
      return launch_impl<TILE_M, 64, FP32_OUT>(act_map, tiles, scales, c, M, N, K, sm_count,
                                               status, wait_limit_ns, stream);
    default:
      return launch_impl<TILE_M, 128, FP32_OUT>(act_map, tiles, scales, c, M, N, K, sm_count,
                                                status, wait_limit_ns, stream);
  }
}

int choose_tile_m(int M, int N, int sm_count) {
  // Estimated main-loop time ~ waves x per-tile cost; per-tile cost grows
  // with TILE_M, with a floor for the fixed dequant work of a weight block.
  static const int options[3] = {64, 128, 192};
  int best = 192;
  double best_cost = 1e30;
  for (int tm : options) {
    const long tiles = static_cast<long>((M + tm - 1) / tm) * (N / TILE_N);
    const long waves = (tiles + sm_count - 1) / sm_count;
    const double per_tile = tm > 96 ? tm : 96.0;
    const double cost = static_cast<double>(waves) * per_tile;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = tm;
    }
  }
  return best;
}

cudaError_t launch(const CUtensorMap& act_map, int tile_m, const uint8_t* tiles,
                   const __half* scales, void* c, bool fp32_out, int M, int N, int K, int group,
                   int sm_count, int* status, unsigned long long wait_limit_ns,
                   cudaStream_t stream) {
#define I4G_TC_CASE(TM)                                                                       \
  if (tile_m == TM)                                                                           \
    return fp32_out ? launch_group<TM, true>(act_map, tiles, scales, c, M, N, K, group,       \
                                             sm_count, status, wait_limit_ns, stream)         \
                    : launch_group<TM, false>(act_map, tiles, scales, c, M, N, K, group,      \
                                              sm_count, status, wait_limit_ns, stream);
  I4G_TC_CASE(64)
  I4G_TC_CASE(128)
  I4G_TC_CASE(192)
#undef I4G_TC_CASE
  return cudaErrorInvalidValue;
}

}  // namespace tc
}  // namespace i4g
