// Decode-shaped W4A16 GEMM (M <= 16): HBM-bound, tensor-core GEMV.
//
// The reference has no decode path (its kernels need M % 64 == 0,
// kernels/gemm_v17_instruction.cu:569); this kernel serves the M <= 16 shapes
// of the same product C = A x dequant(B).
//
// Swap-AB on mma.sync.m16n8k16: the 16x16 "A" fragment is a block of 16
// weight columns x 16 k, decoded in registers straight from the tile layout
// (no shared memory), and the 16x8 "B" fragment holds 8 activation rows.
// Inside a 64-k block the MMA's k order is permuted so that lane (g, t)
// needs activations A[m][16t .. 16t+15] (two 16-byte loads) and the weight
// nibbles of columns g and g+8 at k 16t .. 16t+15 (two 8-byte loads from the
// tile layout): MMA step j, lane slot 2t / 2t+1 / 2t+8 / 2t+9 carries real k
// 16t+4j / +1 / +2 / +3. The sum over a 64-k block is the same set of
// products, accumulated in FP32.
//
// Work split: one thread-block cluster of C CTAs per 16 weight columns; the
// C*W warps of the cluster take contiguous K chunks. Each warp keeps four
// 64-k weight blocks in flight (registers) to cover HBM latency. Partial
// tiles are reduced first inside each CTA through shared memory, then across
// the cluster through distributed shared memory, in a fixed order, so the
// result is deterministic and no global scratch memory is used.
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_runtime.h>

namespace i4g {
namespace dec {

constexpr int BK = 64;
constexpr int WBLOCK_BYTES = 4096;
constexpr int WARPS = 4;  // per CTA
constexpr int DEPTH = 4;  // weight blocks in flight per warp

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct WUnit {
  uint2 lo, hi;    // nibbles of columns g and g+8, k 16t .. 16t+15
  uint32_t s2x;    // their scales: low half column g, high half column g+8
};

template <int MT>
struct AUnit {
  uint4 v[MT][2];  // A[mb*8+g][16t .. 16t+15]
};

struct Ctx {
  const uint8_t* wbase;    // tile-layout bytes of this lane's two columns, kb = 0
  const unsigned short* sbase;
  const __half* abase;     // A + g*K + 16t
  int K, M, g, t;
};

template <int GROUP>
__device__ __forceinline__ void load_w(WUnit& u, const Ctx& c, int kb) {
  const uint8_t* p = c.wbase + static_cast<size_t>(kb) * WBLOCK_BYTES;
  u.lo = __ldcs(reinterpret_cast<const uint2*>(p));
  u.hi = __ldcs(reinterpret_cast<const uint2*>(p + 8 * 16));
  const int grp = (kb * BK + 16 * c.t) / GROUP;
  const unsigned short* s = c.sbase + static_cast<size_t>(grp) * 128;
  u.s2x = static_cast<uint32_t>(__ldg(s)) | (static_cast<uint32_t>(__ldg(s + 8)) << 16);
}

template <int MT>
__device__ __forceinline__ void load_a(AUnit<MT>& u, const Ctx& c, int kb) {
#pragma unroll
  for (int mb = 0; mb < MT; ++mb) {
    if (mb * 8 + c.g < c.M) {
      const uint4* p = reinterpret_cast<const uint4*>(c.abase + static_cast<size_t>(mb * 8) * c.K +
                                                      kb * BK);
      u.v[mb][0] = __ldg(p);
      u.v[mb][1] = __ldg(p + 1);
    } else {
      u.v[mb][0] = make_uint4(0, 0, 0, 0);
      u.v[mb][1] = make_uint4(0, 0, 0, 0);
    }
  }
}

template <int MT>
__device__ __forceinline__ void compute(const WUnit& w, const AUnit<MT>& a, float (&acc)[MT][4]) {
  const uint32_t slo2 = __byte_perm(w.s2x, 0, 0x1010);
  const uint32_t shi2 = __byte_perm(w.s2x, 0, 0x3232);
  const uint32_t lo[2] = {w.lo.x, w.lo.y};
  const uint32_t hi[2] = {w.hi.x, w.hi.y};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t wl = lo[j >> 1], wh = hi[j >> 1];
    uint32_t a0, a1, a2, a3;
    if (j & 1) {
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
    for (int mb = 0; mb < MT; ++mb) {
      const uint32_t* av = reinterpret_cast<const uint32_t*>(&a.v[mb][0]);
      mma_16816(acc[mb], a0, a1, a2, a3, av[2 * j], av[2 * j + 1]);
    }
  }
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

__device__ __forceinline__ float ld_dsmem_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(remote)
               : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int MT, int GROUP>
__global__ void __launch_bounds__(WARPS * 32)
    decode_kernel(const __half* __restrict__ a, const uint8_t* __restrict__ tiles,
                  const __half* __restrict__ scales, __half* __restrict__ c, int M, int N,
                  int K) {
  __shared__ float red[WARPS][32][4 * MT];
  __shared__ float cta_sum[32][4 * MT];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t csize = cluster_nctarank();
  const int nb = blockIdx.x / csize;      // 16-column block of this cluster
  const int nt = nb >> 3;                  // 128-column tile of the layout
  const int g = lane >> 2, t = lane & 3;
  const int rowg = (nb & 7) * 16 + g;
  const int kblocks = K / BK;
  const int chunks = static_cast<int>(csize) * WARPS;
  const int chunk = static_cast<int>(crank) * WARPS + warp;
  const int kb0 = static_cast<int>((static_cast<long>(chunk) * kblocks) / chunks);
  const int kb1 = static_cast<int>((static_cast<long>(chunk + 1) * kblocks) / chunks);

  Ctx ctx;
  ctx.wbase = tiles + static_cast<size_t>(nt) * kblocks * WBLOCK_BYTES + (t >> 1) * 2048 +
              rowg * 16 + (t & 1) * 8;
  ctx.sbase = reinterpret_cast<const unsigned short*>(scales) +
              static_cast<size_t>(nt) * (K / GROUP) * 128 + rowg;
  ctx.abase = a + static_cast<size_t>(g) * K + 16 * t;
  ctx.K = K;
  ctx.M = M;
  ctx.g = g;
  ctx.t = t;

  float acc[MT][4];
#pragma unroll
  for (int mb = 0; mb < MT; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mb][i] = 0.0f;

  const int n = kb1 - kb0;
  WUnit w[DEPTH];
  AUnit<MT> av[2];
#pragma unroll
  for (int i = 0; i < DEPTH; ++i)
    if (i < n) load_w<GROUP>(w[i], ctx, kb0 + i);
  if (n > 0) load_a<MT>(av[0], ctx, kb0);
  for (int base = 0; base < n; base += DEPTH) {
#pragma unroll
    for (int i = 0; i < DEPTH; ++i) {
      const int u = base + i;
      if (u < n) {
        if (u + 1 < n) load_a<MT>(av[(i + 1) & 1], ctx, kb0 + u + 1);
        compute<MT>(w[i], av[i & 1], acc);
        if (u + DEPTH < n) load_w<GROUP>(w[i], ctx, kb0 + u + DEPTH);
      }
    }
  }

  // Reduce the CTA's warps (fixed order), then the cluster's CTAs.
#pragma unroll
  for (int mb = 0; mb < MT; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][lane][4 * mb + i] = acc[mb][i];
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 4 * MT; idx += blockDim.x) {
    const int l = idx / (4 * MT), e = idx % (4 * MT);
    float s = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < WARPS; ++w2) s += red[w2][l][e];
    cta_sum[l][e] = s;
  }
  cluster_sync();
  if (crank == 0) {
    for (int idx = threadIdx.x; idx < 32 * 4 * MT; idx += blockDim.x) {
      const int l = idx / (4 * MT), e = idx % (4 * MT);
      float s = cta_sum[l][e];
      for (uint32_t r = 1; r < csize; ++r) s += ld_dsmem_f32(&cta_sum[l][e], r);
      const int mb = e / 4, i = e % 4;
      const int gl = l >> 2, tl = l & 3;
      const int col = nb * 16 + gl + ((i >> 1) << 3);
      const int m = mb * 8 + 2 * tl + (i & 1);
      if (m < M) c[static_cast<size_t>(m) * N + col] = __float2half_rn(s);
    }
  }
  cluster_sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

// Cluster size: enough CTAs to cover the SMs several times over, while each
// warp still streams at least four 64-k blocks.
int choose_cluster(int N, int K, int sm_count) {
  const int nblocks = N / 16;
  const int kblocks = K / BK;
  int c = 1;
  while (c < 8 && nblocks * c < 5 * sm_count && kblocks / (2 * c * WARPS) >= DEPTH) c *= 2;
  return c;
}

template <int MT, int GROUP>
cudaError_t launch_typed(const __half* a, const uint8_t* tiles, const __half* scales, __half* c,
                         int M, int N, int K, int cluster, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N / 16) * cluster);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_kernel<MT, GROUP>, a, tiles, scales, c, M, N, K);
}

template <int MT>
cudaError_t launch_mt(const __half* a, const uint8_t* tiles, const __half* scales, __half* c,
                      int M, int N, int K, int group, int cluster, cudaStream_t stream) {
  switch (group) {
    case 32: return launch_typed<MT, 32>(a, tiles, scales, c, M, N, K, cluster, stream);
    case 64: return launch_typed<MT, 64>(a, tiles, scales, c, M, N, K, cluster, stream);
    default: return launch_typed<MT, 128>(a, tiles, scales, c, M, N, K, cluster, stream);
  }
}

cudaError_t launch(const __half* a, const uint8_t* tiles, const __half* scales, __half* c,
                   int M, int N, int K, int group, int sm_count, cudaStream_t stream) {
  const int cluster = choose_cluster(N, K, sm_count);
  if (M <= 8) return launch_mt<1>(a, tiles, scales, c, M, N, K, group, cluster, stream);
  return launch_mt<2>(a, tiles, scales, c, M, N, K, group, cluster, stream);
}

}  // namespace dec
}  // namespace i4g
