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
// Grid: one CTA per 16 weight columns; the CTA's warps split K and reduce
// their partial tiles through shared memory in a fixed order (deterministic).
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_runtime.h>

namespace i4g {
namespace dec {

constexpr int BK = 64;
constexpr int WBLOCK_BYTES = 4096;
constexpr int MAX_WARPS = 16;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int MT>
struct Unit {
  uint2 wlo, whi;       // nibbles of columns g and g+8, k 16t .. 16t+15
  uint16_t slo, shi;    // their scales
  uint4 act[MT][2];     // A[mb*8+g][16t .. 16t+15]
};

template <int MT, int GROUP>
__device__ __forceinline__ void load_unit(Unit<MT>& u, const __half* __restrict__ a,
                                          const uint8_t* __restrict__ tiles,
                                          const __half* __restrict__ scales, int M, int K,
                                          int nt, int rowg, int kb, int g, int t) {
  const int kblocks = K / BK;
  const int groups = K / GROUP;
  const uint8_t* blk = tiles + (static_cast<size_t>(nt) * kblocks + kb) * WBLOCK_BYTES +
                       (t >> 1) * 2048 + (t & 1) * 8;
  u.wlo = __ldcs(reinterpret_cast<const uint2*>(blk + rowg * 16));
  u.whi = __ldcs(reinterpret_cast<const uint2*>(blk + (rowg + 8) * 16));
  const int grp = (kb * BK + 16 * t) / GROUP;
  const unsigned short* srow = reinterpret_cast<const unsigned short*>(scales) +
                               (static_cast<size_t>(nt) * groups + grp) * 128;
  u.slo = __ldg(srow + rowg);
  u.shi = __ldg(srow + rowg + 8);
#pragma unroll
  for (int mb = 0; mb < MT; ++mb) {
    const int m = mb * 8 + g;
    if (m < M) {
      const uint4* ap = reinterpret_cast<const uint4*>(a + static_cast<size_t>(m) * K +
                                                       kb * BK + 16 * t);
      u.act[mb][0] = __ldg(ap);
      u.act[mb][1] = __ldg(ap + 1);
    } else {
      u.act[mb][0] = make_uint4(0, 0, 0, 0);
      u.act[mb][1] = make_uint4(0, 0, 0, 0);
    }
  }
}

template <int MT>
__device__ __forceinline__ void compute_unit(const Unit<MT>& u, float (&acc)[MT][4]) {
  const uint32_t slo2 = half_bits_x2(u.slo);
  const uint32_t shi2 = half_bits_x2(u.shi);
  const uint32_t lo[2] = {u.wlo.x, u.wlo.y};
  const uint32_t hi[2] = {u.whi.x, u.whi.y};
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
      const uint32_t* av = reinterpret_cast<const uint32_t*>(&u.act[mb][0]);
      mma_16816(acc[mb], a0, a1, a2, a3, av[2 * j], av[2 * j + 1]);
    }
  }
}

template <int MT, int GROUP>
__global__ void __launch_bounds__(MAX_WARPS * 32)
    decode_kernel(const __half* __restrict__ a, const uint8_t* __restrict__ tiles,
                  const __half* __restrict__ scales, __half* __restrict__ c, int M, int N,
                  int K) {
  __shared__ float red[MAX_WARPS][32][4 * MT];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int nb = blockIdx.x;          // 16-column block
  const int nt = nb >> 3;             // 128-column tile of the layout
  const int rowg = (nb & 7) * 16 + g; // column inside that tile
  const int kblocks = K / BK;
  const int kb0 = static_cast<int>((static_cast<long>(warp) * kblocks) / nwarps);
  const int kb1 = static_cast<int>((static_cast<long>(warp + 1) * kblocks) / nwarps);

  float acc[MT][4];
#pragma unroll
  for (int mb = 0; mb < MT; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mb][i] = 0.0f;

  if (kb0 < kb1) {
    Unit<MT> cur, nxt;
    load_unit<MT, GROUP>(cur, a, tiles, scales, M, K, nt, rowg, kb0, g, t);
    for (int kb = kb0; kb < kb1; ++kb) {
      if (kb + 1 < kb1) load_unit<MT, GROUP>(nxt, a, tiles, scales, M, K, nt, rowg, kb + 1, g, t);
      compute_unit<MT>(cur, acc);
      cur = nxt;
    }
  }

#pragma unroll
  for (int mb = 0; mb < MT; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][lane][4 * mb + i] = acc[mb][i];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s = 0.0f;
        for (int w = 0; w < nwarps; ++w) s += red[w][lane][4 * mb + i];
        const int n = nb * 16 + g + ((i >> 1) << 3);
        const int m = mb * 8 + 2 * t + (i & 1);
        if (m < M) c[static_cast<size_t>(m) * N + n] = __float2half_rn(s);
      }
  }
}

template <int MT>
cudaError_t launch_mt(const __half* a, const uint8_t* tiles, const __half* scales, __half* c,
                      int M, int N, int K, int group, cudaStream_t stream) {
  const int kblocks = K / BK;
  int warps = kblocks / 8;  // about eight 64-k blocks per warp
  warps = warps < 4 ? 4 : (warps > MAX_WARPS ? MAX_WARPS : warps);
  if (warps > kblocks) warps = kblocks;
  const dim3 grid(N / 16), block(warps * 32);
  switch (group) {
    case 32:
      decode_kernel<MT, 32><<<grid, block, 0, stream>>>(a, tiles, scales, c, M, N, K);
      break;
    case 64:
      decode_kernel<MT, 64><<<grid, block, 0, stream>>>(a, tiles, scales, c, M, N, K);
      break;
    default:
      decode_kernel<MT, 128><<<grid, block, 0, stream>>>(a, tiles, scales, c, M, N, K);
      break;
  }
  return cudaGetLastError();
}

cudaError_t launch(const __half* a, const uint8_t* tiles, const __half* scales, __half* c,
                   int M, int N, int K, int group, cudaStream_t stream) {
  if (M <= 8) return launch_mt<1>(a, tiles, scales, c, M, N, K, group, stream);
  return launch_mt<2>(a, tiles, scales, c, M, N, K, group, stream);
}

}  // namespace dec
}  // namespace i4g
