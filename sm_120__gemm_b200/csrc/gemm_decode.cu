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
// warps, 16 columns each) and a contiguous slice of K. A producer thread
// streams the slice through a shared-memory ring of STAGES stages, each four
// 64-k blocks fetched with three copies: one bulk copy of the weights (four
// consecutive tile-layout blocks, 16 KB), one of their scales and one 3-D TMA
// box of the activation rows (zero past M). A deep ring keeps enough weight
// bytes in flight per SM to stream HBM at full rate without holding them in
// registers. A thread-block cluster spans the K slices of one column tile;
// its CTAs reduce their partial sums through distributed shared memory, each
// CTA summing a share of the tile over the ranks in rank order
// (deterministic, no global scratch).
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_runtime.h>

#include <cstdlib>

namespace i4g {
namespace dec {

constexpr int BK = 64;
constexpr int KPS = 4;  // 64-k blocks per ring stage
constexpr int MAX_CLUSTER = 8;
constexpr int NCOL = 128;
constexpr int CWARPS = NCOL / 16;
constexpr int THREADS = (CWARPS + 1) * 32;
constexpr int CTAS_PER_SM = 2;
constexpr int SMEM_PER_SM = 227 * 1024;

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

__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// One lane's share of one 64-k block: loads its weight words (column r0 at
// wp, column r0 + 8 at wp + 128), the two columns' scales (sp, sp + 16) and
// its activation chunks, decodes the 32 weights to exact half(q * s) and
// issues the MMA steps. Decode of word w, pair p (k pair 2p, 2p+1 at bits 4p
// and 16 + 4p): pairs 0 and 2 (of w and w >> 8) XOR the masked nibbles into
// 0x6408, the half 1032 + q, then one exact subtraction of 1032; pairs 1 and 3
// into 0x6480 = 1024 + 16 (q + 8), then one exact fma by 1/16 and -72. One
// rounding multiply by the scale follows (explicit .rn: never contracted).
// X is a register-name suffix, so that two blocks can share one asm
// statement and interleave.
#define I4G_DEC_REGS(X)                                                          \
  ".reg .b32 w0" X ", w1" X ", w2" X ", w3" X ", y0" X ", y1" X ", y2" X ", y3" X \
  ", s0" X ", s1" X ";\n\t"                                                      \
  ".reg .b16 h0" X ", h1" X ";\n\t"                                              \
  ".reg .b32 p0" X ", p1" X ", p2" X ", p3" X ", p4" X ", p5" X ", p6" X ", p7" X  \
  ";\n\t"                                                                        \
  ".reg .b32 q0" X ", q1" X ", q2" X ", q3" X ", q4" X ", q5" X ", q6" X ", q7" X  \
  ";\n\t"                                                                        \
  ".reg .b32 a0" X ", a1" X ", a2" X ", a3" X ", a4" X ", a5" X ", a6" X ", a7" X  \
  ";\n\t"

#define I4G_DEC_LOADS(X, WP, WOFS, SP, AP0, AP1, AOFS)                  \
  "ld.shared.v2.b32 {w0" X ", w1" X "}, [" WP "+" WOFS "];\n\t"        \
  "ld.shared.v2.b32 {w2" X ", w3" X "}, [" WP "+" WOFS "+128];\n\t"    \
  "ld.shared.b16 h0" X ", [" SP "];\n\t"                               \
  "ld.shared.b16 h1" X ", [" SP "+16];\n\t"                            \
  "ld.shared.v4.b32 {a0" X ", a1" X ", a2" X ", a3" X "}, [" AP0 "+" AOFS "];\n\t" \
  "ld.shared.v4.b32 {a4" X ", a5" X ", a6" X ", a7" X "}, [" AP1 "+" AOFS "];\n\t" \
  "mov.b32 s0" X ", {h0" X ", h0" X "};\n\t"                            \
  "mov.b32 s1" X ", {h1" X ", h1" X "};\n\t"

#define I4G_DEC_WORD(W, T, O0, O1, O2, O3, S)                          \
  "shr.b32 " T ", " W ", 8;\n\t"                                       \
  "lop3.b32 " O0 ", " W ", 0x000F000F, 0x64086408, 0x6a;\n\t"          \
  "lop3.b32 " O1 ", " W ", 0x00F000F0, 0x64806480, 0x6a;\n\t"          \
  "lop3.b32 " O2 ", " T ", 0x000F000F, 0x64086408, 0x6a;\n\t"          \
  "lop3.b32 " O3 ", " T ", 0x00F000F0, 0x64806480, 0x6a;\n\t"          \
  "sub.rn.f16x2 " O0 ", " O0 ", kbias;\n\t"                            \
  "fma.rn.f16x2 " O1 ", " O1 ", k16th, km72;\n\t"                      \
  "sub.rn.f16x2 " O2 ", " O2 ", kbias;\n\t"                            \
  "fma.rn.f16x2 " O3 ", " O3 ", k16th, km72;\n\t"                      \
  "mul.rn.f16x2 " O0 ", " O0 ", " S ";\n\t"                            \
  "mul.rn.f16x2 " O1 ", " O1 ", " S ";\n\t"                            \
  "mul.rn.f16x2 " O2 ", " O2 ", " S ";\n\t"                            \
  "mul.rn.f16x2 " O3 ", " O3 ", " S ";\n\t"

#define I4G_DEC_DECODE(X)                                                                   \
  I4G_DEC_WORD("w0" X, "y0" X, "p0" X, "p1" X, "p2" X, "p3" X, "s0" X)                      \
  I4G_DEC_WORD("w1" X, "y1" X, "p4" X, "p5" X, "p6" X, "p7" X, "s0" X)                      \
  I4G_DEC_WORD("w2" X, "y2" X, "q0" X, "q1" X, "q2" X, "q3" X, "s1" X)                      \
  I4G_DEC_WORD("w3" X, "y3" X, "q4" X, "q5" X, "q6" X, "q7" X, "s1" X)

// The four MMA steps of a block go to four independent accumulators, so a
// warp issues them back to back instead of waiting on each result.
#define I4G_DEC_MMA1(C, X, P, Q, B0, B1)                                                      \
  "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {" C "}, {p" P X ", q" P X ", p" Q X   \
  ", q" Q X "}, {" B0 ", " B1 "}, {" C "};\n\t"
#define I4G_DEC_MMA(C0, C1, C2, C3, X, A)                                                     \
  I4G_DEC_MMA1(C0, X, "0", "1", A "0" X, A "1" X)                                             \
  I4G_DEC_MMA1(C1, X, "2", "3", A "2" X, A "3" X)                                             \
  I4G_DEC_MMA1(C2, X, "4", "5", A "4" X, A "5" X)                                             \
  I4G_DEC_MMA1(C3, X, "6", "7", A "6" X, A "7" X)

#define I4G_DEC_CONSTS                                 \
  ".reg .b32 kbias, k16th, km72;\n\t"                  \
  "mov.b32 kbias, 0x64086408;\n\t"                     \
  "mov.b32 k16th, 0x2C002C00;\n\t"                     \
  "mov.b32 km72, 0xD480D480;\n\t"

#define I4G_ACC16(A)                                                                        \
  "+f"(A[0][0]), "+f"(A[0][1]), "+f"(A[0][2]), "+f"(A[0][3]), "+f"(A[1][0]), "+f"(A[1][1]),  \
      "+f"(A[1][2]), "+f"(A[1][3]), "+f"(A[2][0]), "+f"(A[2][1]), "+f"(A[2][2]),             \
      "+f"(A[2][3]), "+f"(A[3][0]), "+f"(A[3][1]), "+f"(A[3][2]), "+f"(A[3][3])

// One block, 8 activation rows.
__device__ __forceinline__ void block_step(uint32_t wp, uint32_t sp, uint32_t ap0, uint32_t ap1,
                                           float (&acc)[1][4][4]) {
  asm volatile(
      "{\n\t" I4G_DEC_CONSTS I4G_DEC_REGS("A")
      I4G_DEC_LOADS("A", "%16", "0", "%17", "%18", "%19", "0")
      I4G_DEC_DECODE("A")
      I4G_DEC_MMA("%0, %1, %2, %3", "%4, %5, %6, %7", "%8, %9, %10, %11", "%12, %13, %14, %15",
                  "A", "a")
      "}\n"
      : I4G_ACC16(acc[0])
      : "r"(wp), "r"(sp), "r"(ap0), "r"(ap1));
}

// Two consecutive blocks (weights 4096 bytes apart, activations 8 rows x 128
// bytes apart), 8 activation rows: two independent decode streams in one
// statement, so the scheduler can overlap them.
__device__ __forceinline__ void block_step2(uint32_t wp, uint32_t sp0, uint32_t sp1, uint32_t ap0,
                                            uint32_t ap1, float (&acc)[1][4][4]) {
  asm volatile(
      "{\n\t" I4G_DEC_CONSTS I4G_DEC_REGS("A") I4G_DEC_REGS("B")
      I4G_DEC_LOADS("A", "%16", "0", "%17", "%19", "%20", "0")
      I4G_DEC_LOADS("B", "%16", "4096", "%18", "%19", "%20", "1024")
      I4G_DEC_DECODE("A")
      I4G_DEC_DECODE("B")
      I4G_DEC_MMA("%0, %1, %2, %3", "%4, %5, %6, %7", "%8, %9, %10, %11", "%12, %13, %14, %15",
                  "A", "a")
      I4G_DEC_MMA("%0, %1, %2, %3", "%4, %5, %6, %7", "%8, %9, %10, %11", "%12, %13, %14, %15",
                  "B", "a")
      "}\n"
      : I4G_ACC16(acc[0])
      : "r"(wp), "r"(sp0), "r"(sp1), "r"(ap0), "r"(ap1));
}

// One block, 16 activation rows: the second 8 rows sit 8 * 128 bytes further.
__device__ __forceinline__ void block_step(uint32_t wp, uint32_t sp, uint32_t ap0, uint32_t ap1,
                                           float (&acc)[2][4][4]) {
  asm volatile(
      "{\n\t" I4G_DEC_CONSTS I4G_DEC_REGS("A")
      ".reg .b32 a0C, a1C, a2C, a3C, a4C, a5C, a6C, a7C;\n\t"
      I4G_DEC_LOADS("A", "%32", "0", "%33", "%34", "%35", "0")
      "ld.shared.v4.b32 {a0C, a1C, a2C, a3C}, [%34+1024];\n\t"
      "ld.shared.v4.b32 {a4C, a5C, a6C, a7C}, [%35+1024];\n\t"
      I4G_DEC_DECODE("A")
      I4G_DEC_MMA("%0, %1, %2, %3", "%4, %5, %6, %7", "%8, %9, %10, %11", "%12, %13, %14, %15",
                  "A", "a")
      I4G_DEC_MMA1("%16, %17, %18, %19", "A", "0", "1", "a0C", "a1C")
      I4G_DEC_MMA1("%20, %21, %22, %23", "A", "2", "3", "a2C", "a3C")
      I4G_DEC_MMA1("%24, %25, %26, %27", "A", "4", "5", "a4C", "a5C")
      I4G_DEC_MMA1("%28, %29, %30, %31", "A", "6", "7", "a6C", "a7C")
      "}\n"
      : I4G_ACC16(acc[0]), I4G_ACC16(acc[1])
      : "r"(wp), "r"(sp), "r"(ap0), "r"(ap1));
}

#undef I4G_ACC16
#undef I4G_DEC_CONSTS
#undef I4G_DEC_MMA
#undef I4G_DEC_MMA1
#undef I4G_DEC_DECODE
#undef I4G_DEC_WORD
#undef I4G_DEC_LOADS
#undef I4G_DEC_REGS

// Byte offset, inside a stage's scales, of the group holding lane (., t)'s
// 16 k of block j; `odd` is the parity of the stage's first block (a group
// of 128 spans two blocks).
template <int GROUP>
__device__ __forceinline__ uint32_t scale_offset(int j, int t, int odd) {
  if constexpr (GROUP == 32) return static_cast<uint32_t>(2 * j + (t >> 1)) * 256u;
  if constexpr (GROUP == 64) return static_cast<uint32_t>(j) * 256u;
  return static_cast<uint32_t>((j + odd) >> 1) * 256u;
}

template <int MT, int GROUP, int STAGES>
struct Layout {
  static constexpr int ROWS = MT * 8;
  static constexpr int ABYTES = KPS * ROWS * BK * 2;  // [KPS][ROWS][64] halves, swizzled
  static constexpr int WBYTES = KPS * 4096;           // four tile-layout blocks
  // scale groups a stage can touch (one more when a group spans two blocks
  // and the slice starts in the middle of one)
  static constexpr int SGROUPS = KPS * BK / GROUP + (GROUP > BK ? 1 : 0);
  static constexpr int SBYTES = SGROUPS * 128 * 2;
  static constexpr int SLOT = ((ABYTES + WBYTES + SBYTES + 1023) / 1024) * 1024;
  static constexpr int BARS = STAGES * SLOT;             // full[], empty[]
  static constexpr int PARTIAL = BARS + 2 * STAGES * 8;  // fp32 partial tile
  static constexpr int ABORT = PARTIAL + CWARPS * 32 * 4 * MT * 4;
  static constexpr int DYN = ABORT + 16 + 1024;  // + slack for 1024-byte alignment
};

// Ring depth: as many stages as two CTAs per SM can hold, at most 6.
template <int MT, int GROUP>
constexpr int stages_for() {
  int s = 6;
  while (s > 2 && CTAS_PER_SM * (Layout<MT, GROUP, 6>::SLOT * s + 2 * s * 8 +
                                 CWARPS * 32 * 4 * MT * 4 + 16 + 1024 + 1024) > SMEM_PER_SM)
    --s;
  return s;
}

template <int MT, int GROUP, int STAGES>
__global__ void __launch_bounds__(THREADS, CTAS_PER_SM)
    decode_kernel(const __grid_constant__ CUtensorMap act_map,
                  const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                  const __grid_constant__ Outputs out, int M, int N, int K, int* status,
                  unsigned long long wait_limit_ns) {
  using L = Layout<MT, GROUP, STAGES>;
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
      mbar_init(bars + 8 * (STAGES + s), CWARPS);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  if (warp == CWARPS) {
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
        bulk_load(dst + L::ABYTES, wsrc + static_cast<size_t>(kb) * 4096, nkb * 4096, full);
        tma_load_3d(dst, &act_map, full, 0, 0, kb);
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
    float acc[MT][4][4];  // [row block][MMA step][fragment]
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mb][q][i] = 0.0f;
    const uint32_t wofs = L::ABYTES + (t >> 1) * 2048 + r0 * 16 + (t & 1) * 8;
    const uint32_t sofs = L::ABYTES + L::WBYTES + r0 * 2;
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
      const uint32_t wp = slot + wofs;
      const uint32_t sp = slot + sofs;
      const uint32_t ap0 = slot + aofs0, ap1 = slot + aofs1;
      const int odd = kb & 1;
      if (nkb == KPS) {
        if constexpr (MT == 1) {
          block_step2(wp, sp + scale_offset<GROUP>(0, t, odd), sp + scale_offset<GROUP>(1, t, odd),
                      ap0, ap1, acc);
          block_step2(wp + 2 * 4096, sp + scale_offset<GROUP>(2, t, odd),
                      sp + scale_offset<GROUP>(3, t, odd), ap0 + 2 * L::ROWS * 128,
                      ap1 + 2 * L::ROWS * 128, acc);
        } else {
#pragma unroll
          for (int j = 0; j < KPS; ++j)
            block_step(wp + j * 4096, sp + scale_offset<GROUP>(j, t, odd),
                       ap0 + j * (L::ROWS * 128), ap1 + j * (L::ROWS * 128), acc);
        }
      } else {
#pragma unroll 1
        for (int j = 0; j < nkb; ++j)
          block_step(wp + j * 4096, sp + scale_offset<GROUP>(j, t, odd),
                     ap0 + j * (L::ROWS * 128), ap1 + j * (L::ROWS * 128), acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8 * (STAGES + s));
    }
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        partial[(threadIdx.x * MT + mb) * 4 + i] =
            (acc[mb][0][i] + acc[mb][1][i]) + (acc[mb][2][i] + acc[mb][3][i]);
  }

  // Cluster reduction over the K slices: CTA `crank` sums its share of the
  // tile's partial elements over ranks 0..csize-1 in rank order. The
  // producer warp's lanes reconverge first: the cluster barrier is
  // warp-aligned.
  __syncwarp();
  cluster_sync();
  constexpr int UNITS = CWARPS * 32 * MT;  // float4 partial units of the tile
  const int x0 = static_cast<int>((crank * UNITS) / csize);
  const int x1 = static_cast<int>(((crank + 1) * UNITS) / csize);
  const uint32_t part_u32 = smem_u32(partial);
  for (int x = x0 + static_cast<int>(threadIdx.x); x < x1; x += THREADS) {
    // every rank's partial is loaded before any is added; the sum runs in
    // rank order
    float4 v[MAX_CLUSTER];
#pragma unroll
    for (int r = 0; r < MAX_CLUSTER; ++r)
      if (r < static_cast<int>(csize))
        v[r] = ld_dsmem_f32x4(part_u32 + x * 16, static_cast<uint32_t>(r));
    float4 sum = v[0];
#pragma unroll
    for (int r = 1; r < MAX_CLUSTER; ++r) {
      if (r < static_cast<int>(csize)) {
        sum.x += v[r].x;
        sum.y += v[r].y;
        sum.z += v[r].z;
        sum.w += v[r].w;
      }
    }
    const int mb = x % MT;
    const int th = x / MT;
    const int w = th >> 5, ln = th & 31;
    const int col = nt * NCOL + w * 16 + (ln >> 2);
    const int m = mb * 8 + 2 * (ln & 3);
    // fragment k: column col + 8 (k >> 1), row m + (k & 1)
    const size_t ldc = static_cast<size_t>(out.ldc);
    const size_t off = static_cast<size_t>(m) * ldc + out.col0 + col;
    const __half hx = __float2half_rn(sum.x), hy = __float2half_rn(sum.y);
    const __half hz = __float2half_rn(sum.z), hw = __float2half_rn(sum.w);
    const int copies = out.count;
#pragma unroll 1
    for (int d = 0; d < copies; ++d) {
      __half* c0 = static_cast<__half*>(d == 0 ? out.dst[0] : out.dst[d]) + off;
      if (m < M) {
        c0[0] = hx;
        c0[8] = hz;
      }
      if (m + 1 < M) {
        c0[ldc] = hy;
        c0[ldc + 8] = hw;
      }
    }
  }
  if (out.count > 1) __threadfence_system();  // peer copies are read by other GPUs
  cluster_sync();  // every CTA's shared memory stays alive until all have read it
}

template <int MT, int GROUP>
cudaError_t launch_typed(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                         const Outputs& out, int M, int N, int K, int cluster, int* status,
                         unsigned long long wait_limit_ns, cudaStream_t stream) {
  constexpr int S = stages_for<MT, GROUP>();
  using L = Layout<MT, GROUP, S>;
  auto kernel = decode_kernel<MT, GROUP, S>;
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
  return cudaLaunchKernelEx(&cfg, kernel, act_map, tiles, scales, out, M, N, K, status,
                            wait_limit_ns);
}

// Tuning override for the cluster size (1-8), read once from
// I4G_DECODE_CLUSTER; 0 means the shape-based choice.
int cluster_override() {
  static const int v = [] {
    const char* e = std::getenv("I4G_DECODE_CLUSTER");
    const int c = e ? std::atoi(e) : 0;
    return (c >= 1 && c <= MAX_CLUSTER) ? c : 0;
  }();
  return v;
}

// Cluster size: the K split that spreads the column tiles over the SMs most
// evenly in one wave of resident CTAs (the busiest SM holds ceil(ctas / sms)
// CTAs; the score is the mean over that), the larger split on ties, while
// every CTA keeps at least two ring stages of work.
int choose_cluster(int N, int K, int sm_count) {
  if (cluster_override()) return cluster_override();
  const int kblocks = K / BK;
  const int tiles = N / NCOL;
  int best = 1;
  double best_score = -1.0;
  for (int cl = 1; cl <= MAX_CLUSTER; ++cl) {
    if (cl > 1 && kblocks / cl < 2 * KPS) break;
    const long ctas = static_cast<long>(tiles) * cl;
    const long most = (ctas + sm_count - 1) / sm_count;
    if (most > CTAS_PER_SM) break;
    const double score = (static_cast<double>(ctas) / sm_count) / most;
    if (score >= best_score - 1e-9) {
      best_score = score;
      best = cl;
    }
  }
  return best;
}

template <int MT>
cudaError_t launch_mt(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                      const Outputs& out, int M, int N, int K, int group, int cluster, int* status,
                      unsigned long long wait_limit_ns, cudaStream_t stream) {
  switch (group) {
    case 32:
      return launch_typed<MT, 32>(act_map, tiles, scales, out, M, N, K, cluster, status,
                                  wait_limit_ns, stream);
    case 64:
      return launch_typed<MT, 64>(act_map, tiles, scales, out, M, N, K, cluster, status,
                                  wait_limit_ns, stream);
    default:
      return launch_typed<MT, 128>(act_map, tiles, scales, out, M, N, K, cluster, status,
                                   wait_limit_ns, stream);
  }
}

int rows_for(int M) { return M <= 8 ? 8 : 16; }

bool supported(int M, int K, int group) {
  (void)K;
  (void)group;
  return M >= 1 && M <= MAX_M;
}

cudaError_t launch(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                   const Outputs& out, int M, int N, int K, int group, int sm_count, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream) {
  const int cluster = choose_cluster(N, K, sm_count);
  if (M <= 8)
    return launch_mt<1>(act_map, tiles, scales, out, M, N, K, group, cluster, status,
                        wait_limit_ns, stream);
  return launch_mt<2>(act_map, tiles, scales, out, M, N, K, group, cluster, status, wait_limit_ns,
                      stream);
}

}  // namespace dec
}  // namespace i4g
