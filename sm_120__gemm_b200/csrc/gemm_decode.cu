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

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

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
constexpr int kDefaultPrefetchBlocks = 8;
constexpr int kPdlFreeSlots = 32;

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

// Producer side of one ring stage: 64-k blocks [kb, kb + nkb) of column
// tile nt (weights, their scale groups) and the activation box at kb.
template <int MT, int GROUP, int STAGES>
__device__ __forceinline__ void issue_stage(const CUtensorMap* act_map, const uint8_t* tiles,
                                            const __half* scales, int nt, int kb, int nkb,
                                            int kblocks, int groups, uint32_t dst,
                                            uint32_t full) {
  using L = Layout<MT, GROUP, STAGES>;
  const uint8_t* wsrc = tiles + static_cast<size_t>(nt) * kblocks * 4096;
  const __half* ssrc = scales + static_cast<size_t>(nt) * groups * 128;
  const int g0 = kb * BK / GROUP;
  const int g1 = ((kb + nkb) * BK + GROUP - 1) / GROUP;
  mbar_arrive_expect_tx(full, L::ABYTES + nkb * 4096 + (g1 - g0) * 256);
  bulk_load(dst + L::ABYTES, wsrc + static_cast<size_t>(kb) * 4096, nkb * 4096, full);
  tma_load_3d(dst, act_map, full, 0, 0, kb);
  bulk_load(dst + L::ABYTES + L::WBYTES, ssrc + static_cast<size_t>(g0) * 128, (g1 - g0) * 256,
            full);
}

// Per-lane shared-memory offsets inside a stage (see the fragment mapping at
// the top of the file).
struct LaneOffsets {
  uint32_t w, s, a0, a1;
};

template <int MT, int GROUP, int STAGES>
__device__ __forceinline__ LaneOffsets lane_offsets(int warp, int lane) {
  using L = Layout<MT, GROUP, STAGES>;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = warp * 16 + g;  // weight column (inside the tile) of a0/a2
  LaneOffsets o;
  o.w = L::ABYTES + (t >> 1) * 2048 + r0 * 16 + (t & 1) * 8;
  o.s = L::ABYTES + L::WBYTES + r0 * 2;
  // activation row (mb*8 + g) of block j: box row R = j*ROWS + mb*8 + g, and
  // R % 8 == g; 16-byte chunks 2t, 2t+1 sit at (chunk ^ g) under the swizzle
  o.a0 = g * 128 + (((2 * t) ^ g) << 4);
  o.a1 = g * 128 + (((2 * t + 1) ^ g) << 4);
  return o;
}

// Consumer side of one ring stage: nkb 64-k blocks starting at block kb.
template <int MT, int GROUP, int STAGES>
__device__ __forceinline__ void compute_stage(uint32_t slot, const LaneOffsets& o, int lane,
                                              int kb, int nkb, float (&acc)[MT][4][4]) {
  using L = Layout<MT, GROUP, STAGES>;
  const int t = lane & 3;
  const uint32_t wp = slot + o.w;
  const uint32_t sp = slot + o.s;
  const uint32_t ap0 = slot + o.a0, ap1 = slot + o.a1;
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
      block_step(wp + j * 4096, sp + scale_offset<GROUP>(j, t, odd), ap0 + j * (L::ROWS * 128),
                 ap1 + j * (L::ROWS * 128), acc);
  }
}

// Writes one lane's four sums of fragment (row block mb) to every copy of C:
// v.x at (m, col), v.y at (m + 1, col), v.z at (m, col + 8), v.w at
// (m + 1, col + 8), where col = tile column of the lane (warp w, lane ln)
// and m = mb * 8 + 2 (ln & 3).
__device__ __forceinline__ void store_fragment(const Outputs& out, int M, int nt, int w, int ln,
                                               int mb, float4 v) {
  const int col = nt * NCOL + w * 16 + (ln >> 2);
  const int m = mb * 8 + 2 * (ln & 3);
  const size_t ldc = static_cast<size_t>(out.ldc);
  const size_t off = static_cast<size_t>(m) * ldc + out.col0 + col;
  const __half hx = __float2half_rn(v.x), hy = __float2half_rn(v.y);
  const __half hz = __float2half_rn(v.z), hw = __float2half_rn(v.w);
  const int copies = out.count;
#pragma unroll 1
  for (int d = 0; d < copies; ++d) {
    __half* c0 = static_cast<__half*>(out.dst[d]) + off;
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

template <int MT, int GROUP, int STAGES>
__global__ void __launch_bounds__(THREADS, CTAS_PER_SM)
    decode_kernel(const __grid_constant__ CUtensorMap act_map,
                  const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                  const __grid_constant__ Outputs out, int M, int N, int K, int* status,
                  unsigned long long wait_limit_ns, int prefetch_blocks) {
  using L = Layout<MT, GROUP, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + L::BARS;  // full[STAGES], empty[STAGES]
  float* partial = reinterpret_cast<float*>(smem + L::PARTIAL);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);
  volatile int* never = abort_flag + 2;  // a flag nobody sets (draining waits)

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
    *never = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  // Launched as a programmatic dependent of the previous kernel on the stream,
  // this CTA may start while that kernel still runs. Until the dependency
  // wait it touches only its own shared memory and warms L2 with the first
  // `prefetch_blocks` blocks of its weight slice and their scales (a prefetch
  // never stales: see bulk_prefetch_l2), so the previous kernel's tail
  // overlaps this kernel's first HBM reads. A, the weights and C are read
  // and written only after the wait. The prefetch is kept short (two ring
  // stages by default): the copy unit serves it before the ring's first
  // copies, so a long one delays the fill when nothing runs before the kernel
  // (measured on B200 at K = 4096, N = 14336, M = 1: 12.1 us per call without
  // prefetch, 12.2 with 8 blocks, 14.6 with 64).
  if (warp == CWARPS && lane == 0) {
    prefetch_tensormap(&act_map);
    const int nkb = min(kb1 - kb0, prefetch_blocks);
    if (nkb > 0) {
      const uint8_t* wsrc = tiles + (static_cast<size_t>(nt) * kblocks + kb0) * 4096;
      const uint32_t wbytes = static_cast<uint32_t>(nkb) * 4096u;
      for (uint32_t off = 0; off < wbytes; off += 65536u)
        bulk_prefetch_l2(wsrc + off, min(65536u, wbytes - off));
      const int g0 = kb0 * BK / GROUP;
      const int g1 = ((kb0 + nkb) * BK + GROUP - 1) / GROUP;
      bulk_prefetch_l2(scales + (static_cast<size_t>(nt) * groups + g0) * 128,
                       static_cast<uint32_t>(g1 - g0) * 256u);
    }
  }
  grid_dependency_wait();
  if (threadIdx.x == 0) launch_dependents();

  if (warp == CWARPS) {
    // --------------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nstages; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1u;
        if (!mbar_wait(bars + 8 * (STAGES + s), ph ^ 1u, abort_flag, status, wait_limit_ns)) break;
        issued = i + 1;
        const int kb = kb0 + i * KPS;
        issue_stage<MT, GROUP, STAGES>(&act_map, tiles, scales, nt, kb, min(KPS, kb1 - kb),
                                       kblocks, groups, ring + s * L::SLOT, bars + 8 * s);
      }
      if (issued < nstages) {  // gave up: let the copies already issued land first
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
          mbar_wait(bars + 8 * (i % STAGES), (i / STAGES) & 1u, never, nullptr, 100000000ull);
      }
    }
  } else {
    // ---------------------------------------------------------------- compute
    float acc[MT][4][4];  // [row block][MMA step][fragment]
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mb][q][i] = 0.0f;
    const LaneOffsets o = lane_offsets<MT, GROUP, STAGES>(warp, lane);
    for (int i = 0; i < nstages; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1u;
      if (!mbar_wait(bars + 8 * s, ph, abort_flag, status, wait_limit_ns)) break;
      const int kb = kb0 + i * KPS;
      compute_stage<MT, GROUP, STAGES>(ring + s * L::SLOT, o, lane, kb, min(KPS, kb1 - kb), acc);
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
    const int th = x / MT;
    store_fragment(out, M, nt, th >> 5, th & 31, x % MT, sum);
  }
  if (out.count > 1) __threadfence_system();  // peer copies are read by other GPUs
  cluster_sync();  // every CTA's shared memory stays alive until all have read it
}

// ---------------------------------------------------------------------------
// Stream-K schedule. The product has units = (N / 128) * (K / 64) units of
// one column tile x one 64-k block; a persistent grid of G CTAs (CTAS_PER_SM
// per SM) gives CTA c the contiguous run [c*units/G, (c+1)*units/G) in
// tile-major order, so every SM streams and decodes the same number of
// weights whatever N / 128 is. A run is cut at tile edges into segments. A
// CTA whose segment covers a whole tile writes that tile of C itself;
// otherwise it stores its FP32 partial in the workspace, at slot c + tile
// (unique: each slot index counts the run and tile boundaries before the
// segment), and the last of the tile's CTAs to arrive (a ticket per tile,
// indexed by the tile's first CTA, which no other split tile shares) sums
// the tile's partials in run order, so the result does not depend on
// arrival order, and writes C.

__host__ __device__ __forceinline__ int sk_owner(long unit, int grid, long units) {
  // CTA whose run holds `unit`: the largest c with c*units/G <= unit
  return static_cast<int>(((unit + 1) * grid - 1) / units);
}

template <int MT>
constexpr size_t sk_slot_float4s() {
  return static_cast<size_t>(CWARPS) * 32 * MT;
}

template <int MT, int GROUP, int STAGES>
__global__ void __launch_bounds__(THREADS, CTAS_PER_SM)
    decode_sk_kernel(const __grid_constant__ CUtensorMap act_map,
                     const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                     const __grid_constant__ Outputs out, int M, int N, int K,
                     uint32_t* __restrict__ tickets, float4* __restrict__ partials, int* status,
                     unsigned long long wait_limit_ns, int prefetch_blocks) {
  using L = Layout<MT, GROUP, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + L::BARS;  // full[STAGES], empty[STAGES]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::ABORT);
  volatile int* never = abort_flag + 2;  // a flag nobody sets (draining waits)
  volatile int* last_flag = abort_flag + 1;  // "this CTA reduces the tile", per segment

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = K / BK;
  const int groups = K / GROUP;
  const long units = static_cast<long>(N / NCOL) * kblocks;
  const int grid = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  const long u0 = c * units / grid;
  const long u1 = (c + 1) * units / grid;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + 8 * (STAGES + s), CWARPS);
    }
    *abort_flag = 0;
    *never = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  // Programmatic dependent launch, as in decode_kernel: before the wait only
  // shared memory and an L2 warm-up of the run's first weight blocks; A, the
  // weights, C and the workspace (tickets, partials) after it.
  if (warp == CWARPS && lane == 0) {
    prefetch_tensormap(&act_map);
    const int nt = static_cast<int>(u0 / kblocks), kb = static_cast<int>(u0 % kblocks);
    const int nkb = static_cast<int>(
        min(static_cast<long>(min(kblocks - kb, prefetch_blocks)), u1 - u0));
    if (nkb > 0)
      bulk_prefetch_l2(tiles + (static_cast<size_t>(nt) * kblocks + kb) * 4096,
                       static_cast<uint32_t>(nkb) * 4096u);
  }
  grid_dependency_wait();
  if (threadIdx.x == 0) launch_dependents();

  if (warp == CWARPS) {
    // --------------------------------------------------------------- producer
    if (lane == 0) {
      int i = 0, issued = 0;
      bool ok = true;
      for (long u = u0; ok && u < u1;) {
        const int nt = static_cast<int>(u / kblocks);
        const int kb_end = static_cast<int>(min(u1 - static_cast<long>(nt) * kblocks,
                                                static_cast<long>(kblocks)));
        for (int kb = static_cast<int>(u - static_cast<long>(nt) * kblocks); kb < kb_end;
             kb += KPS, ++i) {
          const int s = i % STAGES;
          const uint32_t ph = (i / STAGES) & 1u;
          if (!mbar_wait(bars + 8 * (STAGES + s), ph ^ 1u, abort_flag, status, wait_limit_ns)) {
            ok = false;
            break;
          }
          issued = i + 1;
          issue_stage<MT, GROUP, STAGES>(&act_map, tiles, scales, nt, kb, min(KPS, kb_end - kb),
                                         kblocks, groups, ring + s * L::SLOT, bars + 8 * s);
        }
        u = static_cast<long>(nt) * kblocks + kb_end;
      }
      if (!ok) {  // gave up: let the copies already issued land first
        for (int j = (issued > STAGES ? issued - STAGES : 0); j < issued; ++j)
          mbar_wait(bars + 8 * (j % STAGES), (j / STAGES) & 1u, never, nullptr, 100000000ull);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ compute
  constexpr int CTHREADS = CWARPS * 32;
  constexpr size_t SLOT4 = sk_slot_float4s<MT>();
  float acc[MT][4][4];  // [row block][MMA step][fragment]
#pragma unroll
  for (int mb = 0; mb < MT; ++mb)
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int x = 0; x < 4; ++x) acc[mb][q][x] = 0.0f;
  const LaneOffsets o = lane_offsets<MT, GROUP, STAGES>(warp, lane);
  bool ok = true;  // false once a wait gave up: no more MMAs, C or partials
  int i = 0;
  int split0 = -1, split1 = -1;  // tiles this run shares with other CTAs
  int nsplit = 0;
  for (long u = u0; u < u1;) {
    const int nt = static_cast<int>(u / kblocks);
    const int kb_begin = static_cast<int>(u - static_cast<long>(nt) * kblocks);
    const int kb_end = static_cast<int>(min(u1 - static_cast<long>(nt) * kblocks,
                                            static_cast<long>(kblocks)));
    for (int kb = kb_begin; kb < kb_end; kb += KPS, ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1u;
      if (ok) ok = mbar_wait(bars + 8 * s, ph, abort_flag, status, wait_limit_ns);
      if (ok)
        compute_stage<MT, GROUP, STAGES>(ring + s * L::SLOT, o, lane, kb, min(KPS, kb_end - kb),
                                         acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8 * (STAGES + s));
    }
    u = static_cast<long>(nt) * kblocks + kb_end;

    float4 v[MT];
#pragma unroll
    for (int mb = 0; mb < MT; ++mb) {
      v[mb].x = (acc[mb][0][0] + acc[mb][1][0]) + (acc[mb][2][0] + acc[mb][3][0]);
      v[mb].y = (acc[mb][0][1] + acc[mb][1][1]) + (acc[mb][2][1] + acc[mb][3][1]);
      v[mb].z = (acc[mb][0][2] + acc[mb][1][2]) + (acc[mb][2][2] + acc[mb][3][2]);
      v[mb].w = (acc[mb][0][3] + acc[mb][1][3]) + (acc[mb][2][3] + acc[mb][3][3]);
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int x = 0; x < 4; ++x) acc[mb][q][x] = 0.0f;
    }
    if (kb_begin == 0 && kb_end == kblocks) {  // whole tile: this CTA writes C
      if (ok)
#pragma unroll
        for (int mb = 0; mb < MT; ++mb) store_fragment(out, M, nt, warp, lane, mb, v[mb]);
      continue;
    }
    // split tile: publish the partial now (no wait); tickets are taken once
    // the whole run is done. Only a run's first and last segments can cut a
    // tile, so there are at most two.
    float4* mine = partials + static_cast<size_t>(c + nt) * SLOT4 + threadIdx.x * MT;
#pragma unroll
    for (int mb = 0; mb < MT; ++mb) __stcg(mine + mb, v[mb]);
    if (nsplit++ == 0)
      split0 = nt;
    else
      split1 = nt;
  }
  if (nsplit == 0) {  // CTA-uniform
    if (out.count > 1) __threadfence_system();
    return;
  }
  __threadfence();
  if (!epi_bar_and(CTHREADS, ok)) return;  // also orders every partial before the tickets
  if (threadIdx.x == 0) {
    int last = 0;
    for (int j = 0; j < nsplit; ++j) {
      const long first_unit = static_cast<long>(j == 0 ? split0 : split1) * kblocks;
      const int c_first = sk_owner(first_unit, grid, units);
      const int c_last = sk_owner(first_unit + kblocks - 1, grid, units);
      if (atomicAdd(&tickets[c_first], 1u) == static_cast<uint32_t>(c_last - c_first))
        last |= 1 << j;
    }
    *last_flag = last;
  }
  epi_bar_sync(CTHREADS);
  const int last = *last_flag;
  if (last) __threadfence();
  for (int j = 0; j < nsplit; ++j) {
    if (!((last >> j) & 1)) continue;
    const int nt = j == 0 ? split0 : split1;
    const long first_unit = static_cast<long>(nt) * kblocks;
    const int c_first = sk_owner(first_unit, grid, units);
    const int nparts = sk_owner(first_unit + kblocks - 1, grid, units) - c_first + 1;
    const float4* part = partials + static_cast<size_t>(c_first + nt) * SLOT4 + threadIdx.x * MT;
    // sum the parts in run order; each batch of loads is issued before any
    // of its adds
    float4 sum[MT];
    constexpr int BATCH = 8 / MT;
#pragma unroll 1
    for (int p0 = 0; p0 < nparts; p0 += BATCH) {
      float4 q[BATCH][MT];
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
        if (p0 + b < nparts)
#pragma unroll
          for (int mb = 0; mb < MT; ++mb)
            q[b][mb] = __ldcg(part + static_cast<size_t>(p0 + b) * SLOT4 + mb);
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        if (p0 + b >= nparts) break;
#pragma unroll
        for (int mb = 0; mb < MT; ++mb) {
          if (p0 + b == 0) {
            sum[mb] = q[b][mb];
          } else {
            sum[mb].x += q[b][mb].x;
            sum[mb].y += q[b][mb].y;
            sum[mb].z += q[b][mb].z;
            sum[mb].w += q[b][mb].w;
          }
        }
      }
    }
#pragma unroll
    for (int mb = 0; mb < MT; ++mb) store_fragment(out, M, nt, warp, lane, mb, sum[mb]);
    if (threadIdx.x == 0) tickets[c_first] = 0u;  // ready for the next launch
  }
  if (out.count > 1) __threadfence_system();  // peer copies are read by other GPUs
}

// ---------------------------------------------------------------------------
// Slice schedule. The columns are cut into 16-column slices (one mma.sync
// A operand each) and CTA c (one per SM) owns the contiguous run of slices
// [c*S/G, (c+1)*S/G) over all of K, so no two CTAs share an output and
// nothing is reduced across CTAs, and every SM streams the same number of
// weight bytes to within one slice. A stage is BS 64-k blocks (BS = 16, 8
// or 4 for runs of at most 2, 4 or 8 slices, so that the run's (slice,
// block) units give each of the 16 warps one or two); unit u goes to warp
// u % 16. Every thread also fetches a share of each stage with 16-byte
// cp.async copies (the activation rows into the 128-byte-swizzled layout
// the block step reads, the run's slice-halves and the run's columns of the
// stage's scale groups) and signals the stage's barrier once they land:
// small copies through the copy engine (a 5-D tensor box of 256-byte lines,
// or 256-byte bulk copies) were served one after another, about a stage per
// half microsecond. Each warp keeps the sums of its units over all stages;
// at the end the block-parts of each slice are added in order through
// shared memory (deterministic).

constexpr int SLICE_COLS = 16;
constexpr int SL_WARPS = 16;
constexpr int SL_THREADS = SL_WARPS * 32;
constexpr int SL_MAX = 8;  // slices a CTA may own
static_assert(SL_MAX == kSliceMax, "slice bound");

// Blocks per stage for a run of at most `nsl` slices.
constexpr int slice_bs(int nsl) { return nsl <= 2 ? 16 : nsl <= 4 ? 8 : 4; }

template <int MT, int GROUP, int BS>
struct SliceLayout {
  static constexpr int ROWS = MT * 8;
  static constexpr int NSL = BS == 16 ? 2 : BS == 8 ? 4 : 8;  // slices at most
  static constexpr int ABYTES = BS * ROWS * 128;              // [block][row][64 k], swizzled
  static constexpr int WBYTES = NSL * BS * 512;               // [block][half][slice][256 B]
  static constexpr int SG = BS * BK / GROUP;                  // scale groups per stage
  static constexpr int SBYTES = SG * NSL * 32;                // [group][slice][16 columns]
  static constexpr int SLOT = ((ABYTES + WBYTES + SBYTES + 1023) / 1024) * 1024;
  static constexpr int UNITS = NSL * BS;                      // (slice, block) units, <= 32
  static_assert(UNITS <= 2 * SL_WARPS, "two units per warp at most");
  static_assert(BK * BS % GROUP == 0, "stages hold whole scale groups");
};

template <int MT, int GROUP, int BS>
constexpr int slice_stages() {
  using L = SliceLayout<MT, GROUP, BS>;
  int s = 8;
  while (s > 2 && L::SLOT * s + 2 * s * 8 + 16 + 1024 + 1024 > SMEM_PER_SM) --s;
  return s;
}

template <int MT, int GROUP, int BS, int STAGES>
struct SliceRing {
  using L = SliceLayout<MT, GROUP, BS>;
  static constexpr int BARS = STAGES * L::SLOT;  // full[STAGES]
  static constexpr int ABORT = BARS + STAGES * 8;
  static constexpr int DYN = ABORT + 16 + 1024;
  // the final cross-warp sums reuse the ring: [unit][lane][MT] float4
  static_assert(L::UNITS * 32 * MT * 16 <= BARS, "reduction scratch fits the ring");
};

// Writes one lane's four sums of the fragment of slice column base `col`
// (16 columns) and row block mb to every copy of C (as store_fragment).
__device__ __forceinline__ void store_slice_fragment(const Outputs& out, int M, int col, int ln,
                                                     int mb, float4 v) {
  const int c = col + (ln >> 2);
  const int m = mb * 8 + 2 * (ln & 3);
  const size_t ldc = static_cast<size_t>(out.ldc);
  const size_t off = static_cast<size_t>(m) * ldc + out.col0 + c;
  const __half hx = __float2half_rn(v.x), hy = __float2half_rn(v.y);
  const __half hz = __float2half_rn(v.z), hw = __float2half_rn(v.w);
#pragma unroll 1
  for (int d = 0; d < out.count; ++d) {
    __half* c0 = static_cast<__half*>(out.dst[d]) + off;
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

// Scale group, inside a stage, of lane (., t)'s 16 k of block b.
template <int GROUP>
__device__ __forceinline__ int slice_group(int b, int t) {
  if constexpr (GROUP == 32) return 2 * b + (t >> 1);
  if constexpr (GROUP == 64) return b;
  return b >> 1;
}

template <int MT, int GROUP, int BS, int STAGES>
__global__ void __launch_bounds__(SL_THREADS, 1)
    decode_slices_kernel(const __half* __restrict__ A, const uint8_t* __restrict__ tiles,
                         const __half* __restrict__ scales, const __grid_constant__ Outputs out,
                         int M, int N, int K, int* status, unsigned long long wait_limit_ns) {
  using L = SliceLayout<MT, GROUP, BS>;
  using R = SliceRing<MT, GROUP, BS, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + R::BARS;  // full[STAGES]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + R::ABORT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = K / BK;
  const int groups = K / GROUP;
  const int nslices = N / SLICE_COLS;
  const int s0 = static_cast<int>((static_cast<long>(blockIdx.x) * nslices) / gridDim.x);
  const int s1 = static_cast<int>((static_cast<long>(blockIdx.x + 1) * nslices) / gridDim.x);
  const int nsl = s1 - s0;  // 1 .. L::NSL (host-checked)
  const int nstages = (kblocks + BS - 1) / BS;

  if (threadIdx.x == 0) {
    // every thread arrives once per stage, when its copies have landed
    for (int s = 0; s < STAGES; ++s) mbar_init(bars + 8 * s, SL_THREADS);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  // This thread's copies of stage i: 16-byte pieces p = threadIdx.x + 512 n
  // of [activation: block, row, chunk][weights: block, half, slice, chunk]
  // [scales: group, slice, half-slice].
  const int apieces = BS * L::ROWS * 8;
  const size_t act_row = static_cast<size_t>(K);
  auto issue = [&](int i) {
    const uint32_t slot = ring + (i % STAGES) * L::SLOT;
    const int kb = i * BS;
    const int nkb = min(BS, kblocks - kb);
    const int wpieces = nkb * 2 * nsl * 16;
    const int spieces = (nkb * BK / GROUP) * nsl * 2;
    const int total = apieces + wpieces + spieces;
    for (int p = threadIdx.x; p < total; p += SL_THREADS) {
      if (p < apieces) {
        const int blk = p / (L::ROWS * 8), r = (p >> 3) % L::ROWS, c = p & 7;
        const bool valid = r < M && blk < nkb;
        const __half* src = valid ? A + r * act_row + (kb + blk) * BK + c * 8 : A;
        cp_async16(slot + (blk * L::ROWS + r) * 128 + ((c ^ (r & 7)) << 4), src, valid ? 16 : 0);
      } else if (p < apieces + wpieces) {
        const int q = p - apieces;
        const int c = q & 15, j = (q >> 4) % nsl, bh = (q >> 4) / nsl;  // bh = block * 2 + half
        const int sl = s0 + j;
        const uint8_t* src = tiles +
                             (static_cast<size_t>(sl >> 3) * kblocks + kb + (bh >> 1)) * 4096 +
                             (bh & 1) * 2048 + (sl & 7) * 256 + c * 16;
        cp_async16(slot + L::ABYTES + (bh * nsl + j) * 256 + c * 16, src, 16);
      } else {
        const int q = p - apieces - wpieces;
        const int h = q & 1, j = (q >> 1) % nsl, gi = (q >> 1) / nsl;
        const int sl = s0 + j;
        const __half* src = scales +
                            (static_cast<size_t>(sl >> 3) * groups + kb * BK / GROUP + gi) * 128 +
                            (sl & 7) * SLICE_COLS + h * 8;
        cp_async16(slot + L::ABYTES + L::WBYTES + (gi * nsl + j) * 32 + h * 16, src, 16);
      }
    }
    cp_async_arrive(bars + 8 * (i % STAGES));
  };
  for (int i = 0; i < STAGES && i < nstages; ++i) issue(i);

  // this warp's units: u = warp and warp + 16, u = slice * BS + block (the
  // same block for both)
  const int g = lane >> 2, t = lane & 3;
  const uint32_t a0 = g * 128 + (((2 * t) ^ g) << 4);
  const uint32_t a1 = g * 128 + (((2 * t + 1) ^ g) << 4);
  const int b = warp % BS;
  const uint32_t aoff = b * (L::ROWS * 128);
  uint32_t woff[2], soff[2];
  bool own[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int u = warp + q * SL_WARPS;
    own[q] = u < nsl * BS;
    const int j = own[q] ? u / BS : 0;
    woff[q] = L::ABYTES + ((b * 2 + (t >> 1)) * nsl + j) * 256 + g * 16 + (t & 1) * 8;
    soff[q] = L::ABYTES + L::WBYTES + (slice_group<GROUP>(b, t) * nsl + j) * 32 + g * 2;
  }
  float acc[2][MT][4][4];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int mb = 0; mb < MT; ++mb)
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[q][mb][x][y] = 0.0f;
  for (int i = 0; i < nstages; ++i) {
    const int s = i % STAGES;
    const bool ok = mbar_wait(bars + 8 * s, (i / STAGES) & 1u, abort_flag, status, wait_limit_ns);
    // uniform exit; past this barrier every thread is done with stage i - 1,
    // whose slot takes stage i - 1 + STAGES
    if (!__syncthreads_and(ok)) break;
    if (i >= 1 && i - 1 + STAGES < nstages) issue(i - 1 + STAGES);
    const uint32_t slot = ring + s * L::SLOT;
    if (b < kblocks - i * BS) {
#pragma unroll
      for (int q = 0; q < 2; ++q)
        if (own[q])
          block_step(slot + woff[q], slot + soff[q], slot + a0 + aoff, slot + a1 + aoff, acc[q]);
    }
  }
  // every copy has landed (or, after a timeout, lands now) before the ring
  // is reused
  cp_async_wait_all();
  __syncthreads();
  {
    // The block-parts of each slice, added in order through shared memory.
    float4* red = reinterpret_cast<float4*>(smem);  // [unit][lane][MT]
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (!own[q]) continue;
      const int u = warp + q * SL_WARPS;
#pragma unroll
      for (int mb = 0; mb < MT; ++mb) {
        float4 v;
        v.x = (acc[q][mb][0][0] + acc[q][mb][1][0]) + (acc[q][mb][2][0] + acc[q][mb][3][0]);
        v.y = (acc[q][mb][0][1] + acc[q][mb][1][1]) + (acc[q][mb][2][1] + acc[q][mb][3][1]);
        v.z = (acc[q][mb][0][2] + acc[q][mb][1][2]) + (acc[q][mb][2][2] + acc[q][mb][3][2]);
        v.w = (acc[q][mb][0][3] + acc[q][mb][1][3]) + (acc[q][mb][2][3] + acc[q][mb][3][3]);
        red[(u * 32 + lane) * MT + mb] = v;
      }
    }
    __syncthreads();
    // thread -> (slice j, lane ln, row block mb)
    const int idx = static_cast<int>(threadIdx.x);
    const int j = idx / (32 * MT);
    const int ln = (idx / MT) % 32;
    const int mb = idx % MT;
    if (j < nsl) {
      float4 sum = red[((j * BS) * 32 + ln) * MT + mb];
#pragma unroll
      for (int bb = 1; bb < BS; ++bb) {
        const float4 v = red[((j * BS + bb) * 32 + ln) * MT + mb];
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      store_slice_fragment(out, M, (s0 + j) * SLICE_COLS, ln, mb, sum);
    }
    if (out.count > 1) __threadfence_system();  // peer copies are read by other GPUs
  }
}

// 64-k blocks of its weight slice a cluster-schedule CTA warms L2 with
// before its dependency wait (I4G_DECODE_PREFETCH overrides; read once).
int prefetch_blocks() {
  static const int v = [] {
    const char* e = std::getenv("I4G_DECODE_PREFETCH");
    const int b = e ? std::atoi(e) : kDefaultPrefetchBlocks;
    return b < 0 ? 0 : b;
  }();
  return v;
}

template <int MT, int GROUP>
cudaError_t launch_typed(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                         const Outputs& out, int M, int N, int K, int cluster, bool pdl,
                         int* status, unsigned long long wait_limit_ns, cudaStream_t stream) {
  constexpr int S = stages_for<MT, GROUP>();
  using L = Layout<MT, GROUP, S>;
  auto kernel = decode_kernel<MT, GROUP, S>;
  static std::atomic<uint64_t> configured{0};  // devices set, per instantiation
  cudaError_t e = ensure_dynamic_smem(kernel, L::DYN, configured);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N / NCOL) * cluster);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = L::DYN;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  // the L2 warm-up only pays when it overlaps the previous kernel (without
  // PDL, K = 8192, N = 7168, g64, M = 16: 13.7 us with it, 13.1 without)
  return cudaLaunchKernelEx(&cfg, kernel, act_map, tiles, scales, out, M, N, K, status,
                            wait_limit_ns, pdl ? prefetch_blocks() : 0);
}

template <int MT, int GROUP>
cudaError_t launch_sk_typed(const CUtensorMap& act_map, const uint8_t* tiles,
                            const __half* scales, const Outputs& out, int M, int N, int K,
                            int grid, void* workspace, int* status,
                            unsigned long long wait_limit_ns, cudaStream_t stream) {
  constexpr int S = stages_for<MT, GROUP>();
  using L = Layout<MT, GROUP, S>;
  auto kernel = decode_sk_kernel<MT, GROUP, S>;
  static std::atomic<uint64_t> configured{0};  // devices set, per instantiation
  cudaError_t e = ensure_dynamic_smem(kernel, L::DYN, configured);
  if (e != cudaSuccess) return e;
  uint32_t* tickets = static_cast<uint32_t*>(workspace);
  float4* partials =
      reinterpret_cast<float4*>(static_cast<char*>(workspace) + tc::kTicketBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = L::DYN;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, act_map, tiles, scales, out, M, N, K, tickets,
                            partials, status, wait_limit_ns,
                            pdl_enabled() ? prefetch_blocks() : 0);
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

// Schedule choice: kScheduleAuto lets the model in sk_plan decide between
// stream-K and the cluster schedule (the slice schedule is slower on every
// measured shape); kScheduleSlices / kScheduleCluster / kScheduleStreamK
// force one (slices where slice_grid allows, stream-K only with a large
// enough workspace). Set by set_schedule; until then, I4G_DECODE_SCHEDULE
// ("slices", "cluster" or "streamk") gives the initial value.
std::atomic<int> g_schedule{-1};

int schedule_mode() {
  int v = g_schedule.load(std::memory_order_relaxed);
  if (v >= 0) return v;
  const char* e = std::getenv("I4G_DECODE_SCHEDULE");
  int init = kScheduleAuto;
  if (e && std::strcmp(e, "cluster") == 0) init = kScheduleCluster;
  if (e && std::strcmp(e, "streamk") == 0) init = kScheduleStreamK;
  if (e && std::strcmp(e, "slices") == 0) init = kScheduleSlices;
  int expected = -1;
  g_schedule.compare_exchange_strong(expected, init, std::memory_order_relaxed);
  return g_schedule.load(std::memory_order_relaxed);
}

void set_schedule(int mode) { g_schedule.store(mode, std::memory_order_relaxed); }

SkPlan sk_plan(int M, int N, int K, int sm_count) {
  SkPlan p{};
  const long tiles = N / NCOL;
  const long kblocks = K / BK;
  const long units = tiles * kblocks;
  const int grid = static_cast<int>(std::min<long>(units, static_cast<long>(CTAS_PER_SM) *
                                                              sm_count));
  if (grid < 1 || grid * 4 > static_cast<int>(tc::kTicketBytes)) return p;
  const size_t slots = static_cast<size_t>(grid) + tiles - 1;
  const size_t bytes = tc::kTicketBytes + slots * 16 *
                                              (M <= 8 ? sk_slot_float4s<1>() : sk_slot_float4s<2>());
  // Work of the busiest SM, in 64-k blocks of one column tile: the cluster
  // schedule puts up to CTAS_PER_SM CTAs of ceil(kblocks / cluster) blocks on
  // an SM, stream-K CTAS_PER_SM runs of ceil(units / grid) blocks. Measured
  // on B200 (M = 1, g128, back-to-back calls): a block costs ~0.13 us on the
  // busiest SM under either schedule, and stream-K's reduction through the
  // workspace (partial stores, fence, ticket, last-arriver sum) costs ~3.5 us
  // more than the cluster's reduction through distributed shared memory. So
  // stream-K pays only when it takes more than ~27 blocks off the busiest SM
  // (e.g. N = 28672, K = 8192: 256 -> 194 blocks, 36.3 -> 33.2 us; at N =
  // 14336, K = 4096 the 14 blocks it saves do not: 12.6 vs 14.8 us).
  const int cl = choose_cluster(N, K, sm_count);
  const long ctas = tiles * cl;
  const long most = (ctas + sm_count - 1) / sm_count;
  const long cluster_work = most * ((kblocks + cl - 1) / cl);
  const long per_sm = (static_cast<long>(grid) + sm_count - 1) / sm_count;
  const long sk_work = per_sm * ((units + grid - 1) / grid);
  p.grid = grid;
  p.workspace_bytes = bytes;
  const int mode = schedule_mode();
  p.preferred = mode == kScheduleStreamK ||
                (mode == kScheduleAuto && (cluster_work - sk_work) * 13 > 350);
  return p;
}

template <int MT, int GROUP, int BS>
cudaError_t launch_slices_typed(const __half* A, const uint8_t* tiles, const __half* scales,
                                const Outputs& out, int M, int N, int K, int grid, int* status,
                                unsigned long long wait_limit_ns, cudaStream_t stream) {
  constexpr int S = slice_stages<MT, GROUP, BS>();
  using R = SliceRing<MT, GROUP, BS, S>;
  auto kernel = decode_slices_kernel<MT, GROUP, BS, S>;
  static std::atomic<uint64_t> configured{0};  // devices set, per instantiation
  cudaError_t e = ensure_dynamic_smem(kernel, R::DYN, configured);
  if (e != cudaSuccess) return e;
  kernel<<<grid, SL_THREADS, R::DYN, stream>>>(A, tiles, scales, out, M, N, K, status,
                                               wait_limit_ns);
  return cudaGetLastError();
}

template <int MT, int GROUP>
cudaError_t launch_slices_bs(const __half* A, const uint8_t* tiles, const __half* scales,
                             const Outputs& out, int M, int N, int K, int grid, int* status,
                             unsigned long long wait_limit_ns, cudaStream_t stream) {
  const int slices = N / SLICE_COLS;
  const int most = (slices + grid - 1) / grid;  // slices of the longest run
  switch (slice_bs(most)) {
    case 16:
      return launch_slices_typed<MT, GROUP, 16>(A, tiles, scales, out, M, N, K, grid, status,
                                                wait_limit_ns, stream);
    case 8:
      return launch_slices_typed<MT, GROUP, 8>(A, tiles, scales, out, M, N, K, grid, status,
                                               wait_limit_ns, stream);
    default:
      return launch_slices_typed<MT, GROUP, 4>(A, tiles, scales, out, M, N, K, grid, status,
                                               wait_limit_ns, stream);
  }
}

int slice_grid(int N, int sm_count) {
  const int slices = N / SLICE_COLS;
  const int grid = slices < sm_count ? slices : sm_count;
  if (grid < 1 || (slices + grid - 1) / grid > SL_MAX) return 0;
  return grid;
}

template <int MT>
cudaError_t launch_mt(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                      const Outputs& out, int M, int N, int K, int group, int cluster, bool pdl,
                      const SkPlan* sk, void* workspace, int* status,
                      unsigned long long wait_limit_ns, cudaStream_t stream) {
#define I4G_DEC_CASE(G)                                                                     \
  if (group == G)                                                                           \
    return sk ? launch_sk_typed<MT, G>(act_map, tiles, scales, out, M, N, K, sk->grid,     \
                                       workspace, status, wait_limit_ns, stream)           \
              : launch_typed<MT, G>(act_map, tiles, scales, out, M, N, K, cluster, pdl,    \
                                    status, wait_limit_ns, stream);
  I4G_DEC_CASE(32)
  I4G_DEC_CASE(64)
  I4G_DEC_CASE(128)
#undef I4G_DEC_CASE
  return cudaErrorInvalidValue;
}

template <int MT, int GROUP>
KernelConfig config_of() {
  constexpr int S = stages_for<MT, GROUP>();
  return KernelConfig{MT * 8, NCOL, KPS * BK, 16, MT * 8, S, THREADS, Layout<MT, GROUP, S>::DYN};
}

template <int MT, int GROUP>
cudaError_t resources_of(KernelResources* out) {
  constexpr int S = stages_for<MT, GROUP>();
  using L = Layout<MT, GROUP, S>;
  auto kernel = decode_kernel<MT, GROUP, S>;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = ensure_dynamic_smem(kernel, L::DYN, configured);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes a{};
  if ((e = cudaFuncGetAttributes(&a, kernel)) != cudaSuccess) return e;
  int active = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, THREADS, L::DYN);
  if (e != cudaSuccess) return e;
  *out = KernelResources{a.numRegs, static_cast<int>(a.sharedSizeBytes), a.maxThreadsPerBlock,
                         active};
  return cudaSuccess;
}

bool config(int rows, int group, KernelConfig* out) {
#define I4G_DEC_CFG(R, G) \
  if (rows == R * 8 && group == G) { *out = config_of<R, G>(); return true; }
  I4G_DEC_CFG(1, 32) I4G_DEC_CFG(1, 64) I4G_DEC_CFG(1, 128)
  I4G_DEC_CFG(2, 32) I4G_DEC_CFG(2, 64) I4G_DEC_CFG(2, 128)
#undef I4G_DEC_CFG
  return false;
}

cudaError_t resources(int rows, int group, KernelResources* out) {
#define I4G_DEC_RES(R, G) \
  if (rows == R * 8 && group == G) return resources_of<R, G>(out);
  I4G_DEC_RES(1, 32) I4G_DEC_RES(1, 64) I4G_DEC_RES(1, 128)
  I4G_DEC_RES(2, 32) I4G_DEC_RES(2, 64) I4G_DEC_RES(2, 128)
#undef I4G_DEC_RES
  return cudaErrorInvalidValue;
}

int rows_for(int M) { return M <= 8 ? 8 : 16; }

bool supported(int M, int K, int group) {
  (void)K;
  (void)group;
  return M >= 1 && M <= MAX_M;
}

int pick_schedule(int M, int N, int K, int sm_count, size_t workspace_bytes) {
  const int mode = schedule_mode();
  if (mode == kScheduleSlices && slice_grid(N, sm_count) > 0) return kScheduleSlices;
  const SkPlan sk = sk_plan(M, N, K, sm_count);
  if (workspace_bytes > 0 && sk.preferred && workspace_bytes >= sk.workspace_bytes)
    return kScheduleStreamK;
  return kScheduleCluster;
}

cudaError_t launch(const CUtensorMap& act_map, const __half* A, const uint8_t* tiles,
                   const __half* scales, const Outputs& out, int M, int N, int K, int group,
                   int sm_count, void* workspace, size_t workspace_bytes, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream) {
  const int sched = pick_schedule(M, N, K, sm_count, workspace ? workspace_bytes : 0);
  if (sched == kScheduleSlices) {
    const int grid = slice_grid(N, sm_count);
#define I4G_SL_CASE(MT, G)                                                                   \
  if (group == G)                                                                            \
    return launch_slices_bs<MT, G>(A, tiles, scales, out, M, N, K, grid, status,             \
                                   wait_limit_ns, stream);
    if (M <= 8) {
      I4G_SL_CASE(1, 32) I4G_SL_CASE(1, 64) I4G_SL_CASE(1, 128)
    } else {
      I4G_SL_CASE(2, 32) I4G_SL_CASE(2, 64) I4G_SL_CASE(2, 128)
    }
#undef I4G_SL_CASE
    return cudaErrorInvalidValue;
  }
  const SkPlan sk = sk_plan(M, N, K, sm_count);
  const bool use_sk = sched == kScheduleStreamK;
  const int cluster = use_sk ? 1 : choose_cluster(N, K, sm_count);
  // The cluster schedule is launched as a programmatic dependent only when at
  // least kPdlFreeSlots CTA slots stay free for the next call's CTAs to start
  // early. Measured on B200 (back-to-back calls, weights larger than L2): 72
  // free slots (K = 4096, N = 14336, cluster 2) 12.1 -> 11.1 us at M = 1 and
  // 15.3 -> 13.4 at M = 16; 40 (K = 14336, N = 4096, cluster 8) 11.9 -> 10.7;
  // 16 (K = 8192, N = 7168, cluster 5) unchanged at M = 1 and 13.0 -> 15.0 at
  // M = 16.
  const int free_slots = CTAS_PER_SM * sm_count - (N / NCOL) * cluster;
  const bool pdl = pdl_enabled() && free_slots >= kPdlFreeSlots;
  if (M <= 8)
    return launch_mt<1>(act_map, tiles, scales, out, M, N, K, group, cluster, pdl,
                        use_sk ? &sk : nullptr, workspace, status, wait_limit_ns, stream);
  return launch_mt<2>(act_map, tiles, scales, out, M, N, K, group, cluster, pdl,
                      use_sk ? &sk : nullptr, workspace, status, wait_limit_ns, stream);
}

}  // namespace dec
}  // namespace i4g
