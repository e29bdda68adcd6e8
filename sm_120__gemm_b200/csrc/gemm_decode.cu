// Decode-shaped W4A16 GEMM (M <= 16): HBM-bound, tensor-core GEMV.
//
// The reference has no decode path (its kernels need M % 64 == 0,
// kernels/gemm_v17_instruction.cu:569); this kernel serves the M <= 16 shapes
// of the same product C = A x dequant(B).
//
// Swap-AB on mma.sync.m16n8k16: the 16x16 "A" fragment is a block of 16
// weight columns x 16 k, decoded in registers from the tile layout, and the
// 16x8 "B" fragment holds 8 activation rows. Inside a 64-k block the MMA's k
// order is permuted so that lane (g, t) needs activations A[m][16t..16t+15]
// and the weight nibbles of columns g and g+8 at k 16t..16t+15 (8 bytes
// each in the tile layout): MMA step j, lane slot 2t / 2t+1 / 2t+8 / 2t+9
// carries real k 16t+4j / +1 / +2 / +3. The sum over a 64-k block is the same
// set of products, accumulated in FP32.
//
// Work split: a CTA owns one 128-column tile of the layout (eight compute
// warps, 16 columns each) and a contiguous chunk of K. A producer thread
// streams the chunk through a shared-memory ring in stages of four 64-k
// blocks with exactly three copies per stage: one 16 KB bulk copy of the
// weights (four consecutive tile-layout blocks), one bulk copy of their
// scales and one 3-D TMA box of the activation rows (zero past M). Issuing a
// copy costs a few hundred cycles whatever its size, so large stages are what
// keep enough HBM traffic in flight. A thread-block cluster spans the K
// chunks of the same columns; its CTAs reduce their partial sums through
// distributed shared memory in rank order (deterministic, no global scratch).
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_runtime.h>

namespace i4g {
namespace dec {

constexpr int BK = 64;
constexpr int KPS = 4;         // 64-k blocks per ring stage
constexpr int STAGES = 2;
constexpr int MAX_CLUSTER = 8;
constexpr int NCOL = 128;
constexpr int WARPS = NCOL / 16;
constexpr int THREADS = (WARPS + 1) * 32;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int MT, int GROUP>
struct Layout {
  static constexpr int ROWS = MT * 8;
  static constexpr int ABYTES = KPS * ROWS * BK * 2;     // [KPS][ROWS][64] halves, swizzled
  static constexpr int WBYTES = KPS * 4096;              // four tile-layout blocks
  // scale groups a stage can touch (one more when a group spans two blocks
  // and the chunk starts in the middle of one)
  static constexpr int SGROUPS = KPS * BK / GROUP + (GROUP > BK ? 1 : 0);
  static constexpr int SBYTES = SGROUPS * 128 * 2;
  static constexpr int SLOT = ((ABYTES + WBYTES + SBYTES + 1023) / 1024) * 1024;
  static constexpr int BARS = STAGES * SLOT;              // full[], empty[]
  static constexpr int PARTIAL = BARS + 2 * STAGES * 8;   // fp32 partial tiles
  static constexpr int ABORT = PARTIAL + WARPS * 32 * 4 * MT * 4;
  static constexpr int DYN = ABORT + 16 + 1024;           // + slack for 1024B alignment
};

template <int MT, int GROUP>
__global__ void __launch_bounds__(THREADS, 2)
    decode_kernel(const __grid_constant__ CUtensorMap act_map,
                  const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                  __half* __restrict__ c, int M, int N, int K, int* status,
                  unsigned long long wait_limit_ns) {
  using L = Layout<MT, GROUP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + L::BARS;  // full[STAGES], empty[STAGES]
  float* partial = reinterpret_cast<float*>(smem + L::PARTIAL);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const int nt = blockIdx.x / csize;  // 128-column tile of the layout
  const int kblocks = K / BK;
  const int groups = K / GROUP;
  const int kb0 = static_cast<int>((static_cast<long>(crank) * kblocks) / csize);
  const int kb1 = static_cast<int>((static_cast<long>(crank + 1) * kblocks) / csize);
  const int nstages = (kb1 - kb0 + KPS - 1) / KPS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (STAGES + s), WARPS);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  if (warp == WARPS) {
    // --------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&act_map);
      const uint8_t* wsrc = tiles + static_cast<size_t>(nt) * kblocks * 4096;
      const __half* ssrc = scales + static_cast<size_t>(nt) * groups * 128;
      int issued = 0;
      for (int i = 0; i < nstages; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1u;
        if (!mbar_wait(bars + 8 * (STAGES + s), ph ^ 1u, abort_flag, status, wait_limit_ns)) break;
        issued = i + 1;
        const int kb = kb0 + i * KPS;
        const int nkb = min(KPS, kb1 - kb);
        const int g0 = kb * BK / GROUP;
        const int g1 = ((kb + nkb) * BK + GROUP - 1) / GROUP;
        const uint32_t dst = ring + s * L::SLOT;
        const uint32_t full = bars + 8 * s;
        mbar_arrive_expect_tx(full, L::ABYTES + nkb * 4096 + (g1 - g0) * 256);
        tma_load_3d(dst, &act_map, full, 0, 0, kb);
        bulk_load(dst + L::ABYTES, wsrc + static_cast<size_t>(kb) * 4096, nkb * 4096, full);
        bulk_load(dst + L::ABYTES + L::WBYTES, ssrc + static_cast<size_t>(g0) * 128,
                  (g1 - g0) * 256, full);
      }
      if (issued < nstages) {  // gave up: let the copies already issued land first
        volatile int never = 0;
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
          mbar_wait(bars + 8 * (i % STAGES), (i / STAGES) & 1u, &never, nullptr, 100000000ull);
      }
    }
  } else {
    // ---------------------------------------------------------------- compute
    const int g = lane >> 2, t = lane & 3;
    const int r0 = warp * 16 + g;  // weight column (inside the tile) of a0/a2
    float acc[MT][4];
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mb][i] = 0.0f;
    const uint32_t wofs = L::ABYTES + (t >> 1) * 2048 + r0 * 16 + (t & 1) * 8;
    // activation row (mb*8 + g) of block j: box row R = j*ROWS + mb*8 + g, and
    // R % 8 == g; 16-byte chunks 2t, 2t+1 sit at (chunk ^ g) under the swizzle
    const uint32_t aofs0 = g * 128 + (((2 * t) ^ g) << 4);
    const uint32_t aofs1 = g * 128 + (((2 * t + 1) ^ g) << 4);
    for (int i = 0; i < nstages; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1u;
      if (!mbar_wait(bars + 8 * s, ph, abort_flag, status, wait_limit_ns)) break;
      const uint32_t slot = ring + s * L::SLOT;
      const int kb = kb0 + i * KPS;
      const int nkb = min(KPS, kb1 - kb);
      const int sg0 = kb * BK / GROUP;  // first scale group held by this stage
#pragma unroll 1
      for (int j = 0; j < nkb; ++j) {
        uint32_t lo0, lo1, hi0, hi1;
        uint16_t slo, shi;
        const uint32_t wp = slot + j * 4096 + wofs;
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(lo0), "=r"(lo1) : "r"(wp));
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(hi0), "=r"(hi1) : "r"(wp + 128));
        const int grp = ((kb + j) * BK + 16 * t) / GROUP - sg0;
        const uint32_t sp = slot + L::ABYTES + L::WBYTES + (grp * 128 + r0) * 2;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(slo) : "r"(sp));
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(shi) : "r"(sp + 16));
        uint32_t av[MT][8];
#pragma unroll
        for (int mb = 0; mb < MT; ++mb) {
          const uint32_t rb = slot + (j * L::ROWS + mb * 8) * 128;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(av[mb][0]), "=r"(av[mb][1]), "=r"(av[mb][2]), "=r"(av[mb][3])
                       : "r"(rb + aofs0));
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(av[mb][4]), "=r"(av[mb][5]), "=r"(av[mb][6]), "=r"(av[mb][7])
                       : "r"(rb + aofs1));
        }
        const uint32_t slo2 = half_bits_x2(slo), shi2 = half_bits_x2(shi);
        const uint32_t lo[2] = {lo0, lo1}, hi[2] = {hi0, hi1};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t wl = lo[q >> 1], wh = hi[q >> 1];
          uint32_t a0, a1, a2, a3;
          if (q & 1) {
            a0 = decode_pair<2>(wl, slo2);
            a2 = decode_pair<3>(wl, slo2);
            a1 = decode_pair<2>(wh, shi2);
            a3 = decode_pair<3>(wh, shi2);
          } else {
            a0 = decode_pair<0>(wl, slo2);
            a2 = decode_pair<1>(wl, slo2);
            a1 = decode_pair<0>(wh, shi2);
            a3 = decode_pair<1>(wh, shi2);
          }
#pragma unroll
          for (int mb = 0; mb < MT; ++mb)
            mma_16816(acc[mb], a0, a1, a2, a3, av[mb][2 * q], av[mb][2 * q + 1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8 * (STAGES + s));
    }
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) partial[(warp * 32 + lane) * 4 * MT + 4 * mb + i] = acc[mb][i];
  }

  // Cluster reduction over the K chunks, in rank order, by rank 0. The
  // producer warp's lanes reconverge first: the cluster barrier is warp-aligned.
  __syncwarp();
  cluster_sync();
  if (crank == 0 && warp < WARPS) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = (warp * 32 + lane) * 4 * MT + 4 * mb + i;
        float sum = partial[idx];
        const uint32_t addr = smem_u32(&partial[idx]);
        for (uint32_t r = 1; r < csize; ++r) sum += ld_dsmem_f32(addr, r);
        const int col = nt * NCOL + warp * 16 + g + ((i >> 1) << 3);
        const int m = mb * 8 + 2 * t + (i & 1);
        if (m < M) c[static_cast<size_t>(m) * N + col] = __float2half_rn(sum);
      }
  }
  cluster_sync();  // every CTA's shared memory stays alive until rank 0 has read it
}

template <int MT, int GROUP>
cudaError_t launch_typed(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                         __half* c, int M, int N, int K, int cluster, int* status,
                         unsigned long long wait_limit_ns, cudaStream_t stream) {
  using L = Layout<MT, GROUP>;
  auto kernel = decode_kernel<MT, GROUP>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::DYN);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N / NCOL) * cluster);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = L::DYN;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, act_map, tiles, scales, c, M, N, K, status,
                            wait_limit_ns);
}

// Cluster size: enough CTAs for about three per SM, each streaming at least
// two ring stages.
int choose_cluster(int N, int K, int sm_count) {
  const int kblocks = K / BK;
  const int cols = N / NCOL;
  int cluster = 1;
  while (cluster < MAX_CLUSTER && cols * cluster < 3 * sm_count &&
         kblocks / (cluster * 2) >= 2 * KPS)
    cluster *= 2;
  return cluster;
}

template <int MT>
cudaError_t launch_mt(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                      __half* c, int M, int N, int K, int group, int cluster, int* status,
                      unsigned long long wait_limit_ns, cudaStream_t stream) {
  switch (group) {
    case 32:
      return launch_typed<MT, 32>(act_map, tiles, scales, c, M, N, K, cluster, status,
                                  wait_limit_ns, stream);
    case 64:
      return launch_typed<MT, 64>(act_map, tiles, scales, c, M, N, K, cluster, status,
                                  wait_limit_ns, stream);
    default:
      return launch_typed<MT, 128>(act_map, tiles, scales, c, M, N, K, cluster, status,
                                   wait_limit_ns, stream);
  }
}

int rows_for(int M) { return M <= 8 ? 8 : 16; }

cudaError_t launch(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                   __half* c, int M, int N, int K, int group, int sm_count, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream) {
  const int cluster = choose_cluster(N, K, sm_count);
  if (M <= 8)
    return launch_mt<1>(act_map, tiles, scales, c, M, N, K, group, cluster, status,
                        wait_limit_ns, stream);
  return launch_mt<2>(act_map, tiles, scales, c, M, N, K, group, cluster, status, wait_limit_ns,
                      stream);
}

}  // namespace dec
}  // namespace i4g
