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
//   D     = TILE_M fp32 TMEM columns
// Putting the weights on the MMA-M side means every dequantised weight is
// used by TILE_M activation rows, and the dequantised FP16 values never touch
// shared memory: each dequant thread owns one TMEM lane (one weight column)
// and writes it with tcgen05.st. A tcgen05.mma of M=128, K=16 costs about the
// same issue time at any N up to 256, so the main shape uses N = 256.
//
// Warp roles (one CTA per SM, persistent over output tiles):
//   warp 0       activation producer: TMA of a 64-k x TILE_M box
//   warp 1       TMEM allocator and the single MMA-issuing thread
//   warp 2       weight producer: bulk copies of packed nibbles and scales
//   warps 3-10   dequant, two groups of four warps; group g takes the 64-k
//                blocks with index % 2 == g, each thread turning one weight
//                column's 64 nibbles into 64 halves (one tcgen05.st)
//   warps 11-26  epilogue: TMEM -> registers -> FP16 (or FP32) -> global C
//
// Pipelines (mbarriers, every wait bounded):
//   afull/aempty[A_STAGES]  activation boxes in smem (freed by MMA completion)
//   wfull/wempty[W_STAGES]  packed weight blocks in smem (freed once read)
//   tfull/tempty[T_STAGES]  dequantised weight stages in TMEM
//   dfull/dempty[ACC]       accumulators in TMEM
// The weight ring does not wait for the tensor core, so the dequant runs
// ahead of the MMA by up to T_STAGES blocks.
//
// Accumulation accuracy: the tensor core's FP32 accumulator drifts further
// from the exact sum than a sequential round-to-nearest FP32 sum as the chain
// of MMAs onto it grows. So every `promo` 64-k blocks the epilogue warps fold
// the accumulator into a running sum (promotion): S = H + D rounded once in
// FP32, a coarse H (FP8) kept in registers, and the exact remainder S - H written
// back into the accumulator, onto which the next MMAs accumulate. The tile's
// result is H + D. The chain the tensor core accumulates stays short whatever K
// is.
//
// Schedule: work items are whole tiles, round robin over the grid; then,
// when the caller provides a workspace, the tiles of the last, partial wave
// ("tail") are shared out along K so that the last wave keeps every SM busy:
// either each tail tile split into `split` equal items, or (stream-K) the
// tail's run of (tile, 64-k block) blocks cut into `chunks` equal shares, one
// per CTA, each share covering the end of one tile and the start of the
// next. A partial item writes its FP32 partial tile to a workspace slot and
// takes a ticket; the item that draws the tile's last ticket sums the tile's
// partials in slot order (deterministic) and writes C, then resets the
// ticket counter for the next launch.
#include "ptx.cuh"
#include "gemm_tc.h"

#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdlib>

namespace i4g {
namespace tc {

constexpr int TILE_N = 128;         // weight columns per tile (MMA-M)
constexpr int BK = 64;              // k per stage (one 128-byte swizzle row)
constexpr int T_COLS = 32;          // TMEM columns per dequantised weight stage (64 halves)
constexpr int T_STAGES = 8;         // TMEM weight stages
constexpr int DEQ_GROUPS = 1;       // dequant warp groups (4 warps = 128 lanes each)
constexpr int NUM_DEQ_WARPS = 4 * DEQ_GROUPS;
constexpr int NUM_EPI_WARPS = 16;   // four per TMEM lane quarter
constexpr int FIRST_DEQ_WARP = 3;
constexpr int FIRST_EPI_WARP = FIRST_DEQ_WARP + NUM_DEQ_WARPS;
constexpr int THREADS = 32 * (FIRST_EPI_WARP + NUM_EPI_WARPS);
// 23 warps (736 threads): 80 registers a thread (six warps share one SMSP's
// 16,384 registers)
static_assert(NUM_DEQ_WARPS == 4 && NUM_EPI_WARPS == 16, "each TMEM lane quarter (warp % 4) "
              "has one dequant warp and four epilogue warps");
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL0 = T_STAGES * T_COLS;    // 256
constexpr int WBLOCK_BYTES = TILE_N * BK / 2;  // 4096: one tile-layout block
constexpr int SCALE_BYTES = 512;               // up to two groups x 128 halves
constexpr int W_SLOT = WBLOCK_BYTES + SCALE_BYTES;
constexpr int W_STAGES = 14;
constexpr int GROUP_M = 8;                     // rasterisation band (m-tiles)

// CG = 1: one CTA per tile, weights dequantised into TMEM (operand A from
// TMEM). CG = 2: a CTA pair (cluster of two) per tile of 2 x 128 weight
// columns, each CTA loading half of the TILE_M activation rows and
// dequantising its 128 weight columns into 128B-swizzled shared memory (both
// operands from shared memory), so that all of TMEM holds two accumulators.
template <int TILE_M, int CG>
struct Cfg {
  static constexpr bool SS = CG == 2;                          // weights in smem
  static constexpr int ACC = (SS || TILE_M <= 128) ? 2 : 1;    // accumulators in TMEM
  static constexpr int ACC_COL = SS ? 0 : ACC_COL0;            // first accumulator column
  static constexpr int ROWS = TILE_M / CG;                     // activation rows this CTA loads
  static constexpr int ACT_BYTES = ROWS * BK * 2;
  static constexpr int A_STAGES = SS ? 6 : (TILE_M <= 128 ? 8 : 5);
  static constexpr int W_ST = SS ? 8 : W_STAGES;               // packed weight stages
  // dequantised weight stages; single CTAs: one per activation stage, the
  // two sharing one pair of barriers (one wait and one commit per block for
  // the MMA thread)
  static constexpr int T_ST = SS ? 4 : A_STAGES;
  static constexpr int DEQ_BYTES = TILE_N * BK * 2;            // one smem weight tile (SS)
  static constexpr int ACT_OFF = 0;
  static constexpr int DEQ_OFF = ACT_OFF + A_STAGES * ACT_BYTES;
  static constexpr int W_OFF = DEQ_OFF + (SS ? T_ST * DEQ_BYTES : 0);
  static constexpr int BAR_OFF = W_OFF + W_ST * W_SLOT;
  static constexpr int NUM_BARS = 2 * A_STAGES + 2 * W_ST + 2 * T_ST + 2 * ACC + 1;
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int TOTAL = MISC_OFF + 16;
  static constexpr int DYN_BYTES = TOTAL + 1024;  // slack for 1024-byte alignment
  static_assert(ACT_BYTES % 1024 == 0, "activation stage must keep 1024B alignment");
  static_assert(DEQ_BYTES % 1024 == 0, "weight tile must keep 1024B alignment");
  static_assert(ACC_COL + ACC * TILE_M <= TMEM_COLS, "TMEM budget");
  static_assert(SS || T_ST * T_COLS <= ACC_COL, "TMEM weight stages below the accumulators");
  static_assert(DYN_BYTES <= 232448, "shared memory budget");
  static_assert(T_ST % DEQ_GROUPS == 0 && W_ST % DEQ_GROUPS == 0, "stage ownership");
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

struct Item {
  int mt, nt, kb0, kb1;
  int rem;        // index among the tail tiles, or -1 for a whole tile
  int slot;       // workspace slot of this item's partial tile
  int base_slot;  // first slot of the tile's partials (contiguous)
  int nparts;     // partial items of the tile
};

// Work of CTA `b` of a grid of `g`: its `j`-th item, false past its last.
__device__ __forceinline__ bool next_item(const Sched& s, int b, int g, int j, int kblocks,
                                          int num_m, int num_n, Item& r) {
  int tile;
  if (s.chunks == 0) {
    // whole tiles, then `split` equal K splits of each tail tile
    const int item = b + j * g;
    if (item >= s.items) return false;
    if (item < s.full_tiles) {
      tile = item;
      r.kb0 = 0;
      r.kb1 = kblocks;
      r.rem = -1;
    } else {
      const int q = item - s.full_tiles;
      r.rem = q / s.split;
      const int f = q - r.rem * s.split;
      tile = s.full_tiles + r.rem;
      r.kb0 = (f * kblocks) / s.split;
      r.kb1 = ((f + 1) * kblocks) / s.split;
      r.base_slot = r.rem * s.split;
      r.slot = r.base_slot + f;
      r.nparts = s.split;
    }
  } else {
    // whole tiles (the grid is a multiple of them), then this CTA's share
    // [c0, c1) of the tail's block run: one or two tile segments
    const int whole = s.full_tiles / g;
    if (j < whole) {
      tile = b + j * g;
      r.kb0 = 0;
      r.kb1 = kblocks;
      r.rem = -1;
    } else {
      if (b >= s.chunks) return false;
      const int run = s.tail_tiles * kblocks;
      const int c0 = (b * run) / s.chunks, c1 = ((b + 1) * run) / s.chunks;
      const int t = c0 / kblocks + (j - whole);
      if (c1 <= c0 || t > (c1 - 1) / kblocks) return false;
      r.kb0 = max(c0 - t * kblocks, 0);
      r.kb1 = min(c1 - t * kblocks, kblocks);
      // shares touching tile t: owner(v), the last share starting at or
      // before block v, of the tile's first and last blocks
      const int p0 = ((t * kblocks + 1) * s.chunks - 1) / run;
      const int p1 = (((t + 1) * kblocks) * s.chunks - 1) / run;
      tile = s.full_tiles + t;
      if (p0 == p1) {
        r.rem = -1;  // the share covers the whole tile
      } else {
        r.rem = t;
        r.slot = t + b;  // unique: shares and tiles both advance monotonically
        r.base_slot = t + p0;
        r.nparts = p1 - p0 + 1;
      }
    }
  }
  tile_coords(tile, num_m, num_n, r.mt, r.nt);
  return true;
}

// Sums SPLIT partial tiles in split order (a fixed order, so results do not
// depend on which CTA finished last) and writes quads*4 rows of column n of C,
// starting at row m0. `base` points at this thread's first quad of split 0;
// quads of one split are TILE_N float4 apart, splits CG*(TILE_M/4)*TILE_N.
// B quads are loaded for every split before any is summed, to overlap the
// L2 latency.
template <int TILE_M, int SPLIT, int B, bool FP32_OUT, bool MULTI, int CG>
__device__ __forceinline__ void reduce_partials(const float4* base, const Outputs& out, int m0,
                                                int n, int M, int N, int quads) {
  // a pair's two halves interleave their slots
  constexpr size_t kSplitStride = static_cast<size_t>(CG) * (TILE_M / 4) * TILE_N;
#pragma unroll 1
  for (int q = 0; q < quads; q += B) {
    float4 t[SPLIT][B];
#pragma unroll
    for (int f = 0; f < SPLIT; ++f)
#pragma unroll
      for (int b = 0; b < B; ++b)
        t[f][b] = __ldcg(base + f * kSplitStride + static_cast<size_t>(q + b) * TILE_N);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float4 s = t[0][b];
#pragma unroll
      for (int f = 1; f < SPLIT; ++f) {
        s.x += t[f][b].x;
        s.y += t[f][b].y;
        s.z += t[f][b].z;
        s.w += t[f][b].w;
      }
      const float vals[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * (q + b) + i;
        if (m < M) {
          if constexpr (FP32_OUT) {
            static_cast<float*>(out.dst[0])[static_cast<size_t>(m) * N + n] = vals[i];
          } else if constexpr (!MULTI) {
            static_cast<__half*>(out.dst[0])[static_cast<size_t>(m) * N + n] =
                __float2half_rn(vals[i]);
          } else {
            const size_t off = static_cast<size_t>(m) * out.ldc + out.col0 + n;
            const __half h = __float2half_rn(vals[i]);
#pragma unroll 1
            for (int d = 0; d < out.count; ++d) static_cast<__half*>(out.dst[d])[off] = h;
          }
        }
      }
    }
  }
  if constexpr (MULTI) __threadfence_system();  // peer copies are read by other GPUs
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Running sum of promotion. Its high part H is kept coarse, in FP8 (e5m2,
// saturating), four values per 32-bit register: any H leaves the remainder
// S - H exact in FP32 (S has 24 significant bits, H 3 at the same or the next
// exponent), and a coarse H costs the epilogue warps few registers.
__device__ __forceinline__ float2 e5m2x2_to_float2(uint32_t pair) {
  const __half2_raw r = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair),
                                                   __NV_E5M2);
  __half2 h;
  memcpy(&h, &r, sizeof(h));
  return __half22float2(h);
}

__device__ __forceinline__ uint32_t float2_to_e5m2x2(float lo, float hi) {
  return static_cast<uint32_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E5M2));
}

// H of accumulator columns 4q .. 4q+3 of one lane, from word q of hb.
__device__ __forceinline__ void high_parts(uint32_t w, float (&h)[4]) {
  const float2 a = e5m2x2_to_float2(w & 0xFFFFu), b = e5m2x2_to_float2(w >> 16);
  h[0] = a.x;
  h[1] = a.y;
  h[2] = b.x;
  h[3] = b.y;
}

// Promotes 16 accumulator columns at taddr (hb words 0..3), read with one
// load wait: S = H + D (one FP32 rounding per value), H <- e5m2(S),
// D <- S - H (exact), stored back.
__device__ __forceinline__ void promote_chunk16(uint32_t taddr, uint32_t* hb) {
  uint32_t v[16];
  tmem_ld_32x32b_x16(taddr, v);
  tmem_ld_wait16(v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float h[4], sum[4];
    high_parts(hb[q], h);
#pragma unroll
    for (int i = 0; i < 4; ++i) sum[i] = h[i] + __uint_as_float(v[4 * q + i]);
    hb[q] = float2_to_e5m2x2(sum[0], sum[1]) | (float2_to_e5m2x2(sum[2], sum[3]) << 16);
    high_parts(hb[q], h);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[4 * q + i] = __float_as_uint(sum[i] - h[i]);
  }
  uint32_t a[8], b[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a[i] = v[i];
    b[i] = v[8 + i];
  }
  tmem_st_32x32b_x8(taddr, a);
  tmem_st_32x32b_x8(taddr + 8, b);
}

// Final read of 16 accumulator columns (hb words 0..3): v = H + D in FP32.
__device__ __forceinline__ void load_sum16(uint32_t taddr, const uint32_t* hb, uint32_t (&v)[16]) {
  tmem_ld_32x32b_x16(taddr, v);
  tmem_ld_wait16(v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float h[4];
    high_parts(hb[q], h);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[4 * q + i] = __float_as_uint(h[i] + __uint_as_float(v[4 * q + i]));
  }
}

// Moves words 4.. of a running-sum array down by four, so that a rolled loop
// over 16-column chunks always reads words 0..3 (static register indices).
template <int NW>
__device__ __forceinline__ void shift_down4(uint32_t (&hb)[NW]) {
#pragma unroll
  for (int q = 0; q + 4 < NW; ++q) hb[q] = hb[q + 4];
}

// Whole-tile epilogue with several copies of C (this GPU's and peers'), for
// one thread's slice (TMEM lane `row`, COLS accumulator columns from col0):
// the slice is read, converted and stored into this GPU's copy (dst[0]), the
// accumulator released once the last chunk is in registers. Then a GPU-scope
// fence and the epilogue barrier (which every epilogue thread takes whatever
// `ok` is: a failed wait skips the work, never the barrier); true when every
// thread's slice is stored. The tile then goes to the peers' copies piece by
// piece while the epilogue waits for later accumulators (PeerCopier).
template <int TILE_M, int CG>
__device__ __forceinline__ bool copies_epilogue(bool ok, const Outputs& out, int M, int mt, int nt,
                                                int half, int row, int m0, uint32_t col0,
                                                const uint32_t* hb, uint32_t empty_bar) {
  constexpr int COLS = TILE_M / 4;
  constexpr int EPI_THREADS = NUM_EPI_WARPS * 32;
  const size_t ldc = static_cast<size_t>(out.ldc);
  const size_t tile_off = static_cast<size_t>(mt * TILE_M) * ldc + out.col0 + nt * TILE_N;
  __half* const tile0 = static_cast<__half*>(out.dst[0]) + tile_off;
  if (ok) {
    tc_fence_after();
    // each 16-column chunk is stored into this GPU's copy as it is read; the
    // accumulator is released once the last chunk is in registers
    __half* cp = tile0 + static_cast<size_t>(half * COLS) * ldc + row;
    const int valid = min(COLS, M - m0);
#pragma unroll
    for (int c = 0; c < COLS / 16; ++c) {
      uint32_t v[16];
      load_sum16(col0 + c * 16, &hb[c * 4], v);
      if (c == COLS / 16 - 1) {
        tc_fence_before();
        if constexpr (CG == 2) mbar_arrive_cluster_relaxed(empty_bar);  // the even CTA's
        else mbar_arrive(empty_bar);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (c * 16 + j < valid) *cp = __float2half_rn(__uint_as_float(v[j]));
        cp += ldc;
      }
    }
  }
  __threadfence();
  return epi_bar_and(EPI_THREADS, ok);
}

// One epilogue thread's share of copying finished whole tiles from this
// GPU's copy of C to the peers' copies: pieces t, t + 512, ... of each tile
// (16 bytes each, 16 per 128-column row), read back from L2 (the tile's
// local stores were fenced before the epilogue barrier that made it
// `ready`). Tiles are this CTA's items in order; `ready` counts the items
// the epilogue has finished (split items, which the reduction writes to
// every copy itself, are skipped). Each thread walks its own pieces, so no
// barrier is needed between pieces, and the copying fills the time the
// epilogue would otherwise spend waiting for the next accumulator.
template <int TILE_M, int CG>
struct PeerCopier {
  const Outputs* out;
  int M, first;        // rows of C; this thread's first piece
  int next = 0;        // item being copied
  int ready = 0;       // items finished by the epilogue
  int piece = 0;       // this thread's next piece of item `next`
  int rows = -1;       // rows of item `next` (-1: not looked up yet; 0: nothing to copy)
  size_t tile_off = 0;

  __device__ __forceinline__ bool pending() const { return next < ready; }

  // Copies up to `budget` pieces; `item(j, w)` looks up this CTA's item j.
  template <typename ItemFn>
  __device__ __forceinline__ void copy(int budget, ItemFn item, int rank) {
    const size_t ldc = static_cast<size_t>(out->ldc);
    while (budget > 0 && next < ready) {
      if (rows < 0) {
        Item w;
        item(next, w);
        const int nt = w.nt * CG + rank;
        rows = w.rem < 0 ? min(TILE_M, M - w.mt * TILE_M) : 0;
        tile_off = static_cast<size_t>(w.mt * TILE_M) * ldc + out->col0 + nt * TILE_N;
        piece = first;
      }
      if (piece >= rows * 16) {
        ++next;
        rows = -1;
        continue;
      }
      const size_t off = tile_off + static_cast<size_t>(piece >> 4) * ldc + (piece & 15) * 8;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(static_cast<__half*>(out->dst[0]) + off));
#pragma unroll 1
      for (int d = 1; d < out->count; ++d)
        *reinterpret_cast<uint4*>(static_cast<__half*>(out->dst[d]) + off) = v;
      piece += NUM_EPI_WARPS * 32;
      --budget;
    }
  }
};

// Rotates a running-sum array down by two words (the first two move to the
// end), so that a rolled loop over 8-column chunks always updates words 0, 1
// and a full pass leaves the array in its original order.
template <int NW>
__device__ __forceinline__ void rotate_down2(uint32_t (&hb)[NW]) {
  const uint32_t w0 = hb[0], w1 = hb[1];
#pragma unroll
  for (int q = 0; q + 2 < NW; ++q) hb[q] = hb[q + 2];
  hb[NW - 2] = w0;
  hb[NW - 1] = w1;
}

// OUT selects the C epilogue at compile time, so the plain kernels carry no
// code for the general one: half C or float C as one row-major [M][N] matrix
// (out.dst[0]; ldc == N, col0 == 0), or half C written to columns
// [col0, col0 + N) of out.count row-major [M][ldc] copies (this GPU's and
// peers').
enum OutKind : int { kOutHalf = 0, kOutFloat = 1, kOutHalfCopies = 2 };

template <int TILE_M, int GROUP, int OUT, int CG>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap act_map,
                   const uint8_t* __restrict__ tiles, const __half* __restrict__ scales,
                   const __grid_constant__ Outputs out, int M, int N, int K, const Sched sched,
                   uint32_t* __restrict__ tickets, float* __restrict__ partials, int* status,
                   unsigned long long wait_limit_ns) {
  using L = Cfg<TILE_M, CG>;
  constexpr int A_STAGES = L::A_STAGES;
  constexpr int ACC = L::ACC;
  constexpr int W_STAGES = L::W_ST;
  constexpr int T_STAGES = L::T_ST;
  constexpr int ACC_COL0 = L::ACC_COL;
  constexpr bool FP32_OUT = OUT == kOutFloat;
  constexpr bool MULTI = OUT == kOutHalfCopies;
  constexpr bool PAIR = CG == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const uint32_t act_base = smem_u32(smem + L::ACT_OFF);
  const uint32_t w_base = smem_u32(smem + L::W_OFF);
  const uint32_t deq_base = smem_u32(smem + L::DEQ_OFF);  // pairs: weight tiles
  const uint32_t bar_base = smem_u32(smem + L::BAR_OFF);
  // barrier order: afull, aempty, wfull, wempty, tfull, tempty, dfull, dempty, drain
  auto afull = [&](int i) { return bar_base + 8u * i; };
  auto aempty = [&](int i) { return bar_base + 8u * (A_STAGES + i); };
  auto wfull = [&](int i) { return bar_base + 8u * (2 * A_STAGES + i); };
  auto wempty = [&](int i) { return bar_base + 8u * (2 * A_STAGES + W_STAGES + i); };
  // single CTAs: a block's activation stage and TMEM weight stage share
  // afull (TMA bytes + every dequant thread) and aempty (MMA completion)
  constexpr bool UNI = !(CG == 2);
  auto tfull = [&](int i) {
    return UNI ? afull(i) : bar_base + 8u * (2 * A_STAGES + 2 * W_STAGES + i);
  };
  auto tempty = [&](int i) {
    return UNI ? aempty(i) : bar_base + 8u * (2 * A_STAGES + 2 * W_STAGES + T_STAGES + i);
  };
  auto dfull = [&](int i) {
    return bar_base + 8u * (2 * A_STAGES + 2 * W_STAGES + 2 * T_STAGES + i);
  };
  auto dempty = [&](int i) {
    return bar_base + 8u * (2 * A_STAGES + 2 * W_STAGES + 2 * T_STAGES + ACC + i);
  };
  const uint32_t drain_bar = bar_base + 8u * (L::NUM_BARS - 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  volatile uint32_t* ticket_slot = reinterpret_cast<volatile uint32_t*>(smem + L::MISC_OFF + 8);
  // a flag nobody sets: the "abort" of the bounded waits that must not be cut
  // short by another warp's abort (draining copies, the final MMA drain)
  volatile int* never = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 12);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pairs: the even CTA (rank 0) issues the pair's MMAs; both CTAs load
  // their own half of the activation rows, dequantise their own 128 weight
  // columns into their own TMEM and drain their own accumulator. Barriers
  // the MMA waits on (afull, tfull, dempty) live in the even CTA and count
  // both CTAs' arrivals; the MMA's completions (aempty, tempty, dfull, drain)
  // arrive in both CTAs at once (multicast commit).
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int unit = blockIdx.x / CG, units = gridDim.x / CG;  // work is handed out per pair
  const int num_m = (M + TILE_M - 1) / TILE_M;
  const int num_n = N / (TILE_N * CG);
  const int kblocks = K / BK;
  const int groups = K / GROUP;
  // the even CTA's copy of a barrier (for arrivals from the odd CTA): the
  // shared::cluster window of a CTA is linear, so one mapa serves them all
  const uint32_t lead_bar_base = PAIR ? mapa_shared(bar_base, 0) : bar_base;
  auto lead = [&](uint32_t bar) { return lead_bar_base + (bar - bar_base); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < A_STAGES; ++i) {
      // own producer's expected bytes; in the even CTA of a pair also the odd
      // CTA's relay (its half landed)
      // single CTAs: also every dequant thread (the TMEM stage of the block)
      mbar_init(afull(i), PAIR ? (leader ? 2 : 1) : 1 + 4 * 32);
      mbar_init(aempty(i), 1);  // MMA completion
    }
    for (int i = 0; i < W_STAGES; ++i) {
      mbar_init(wfull(i), 1);
      mbar_init(wempty(i), 4);  // the four warps of the dequant group that read it
    }
    for (int i = 0; !UNI && i < T_STAGES; ++i) {
      // pairs: one arrival per local dequant warp, and in the even CTA also
      // the odd CTA's relay
      mbar_init(tfull(i), leader ? 4 + 1 : 4);
      mbar_init(tempty(i), 1);  // MMA completion
    }
    for (int i = 0; i < ACC; ++i) {
      mbar_init(dfull(i), 1);
      mbar_init(dempty(i), CG * NUM_EPI_WARPS * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *never = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&act_map);
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // a pair's barriers are initialised before either CTA arrives on the other's
  if constexpr (PAIR) cluster_barrier();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Launched as a programmatic dependent of the previous kernel on the stream,
  // this CTA may set up (barriers, TMEM, descriptor prefetch) while that
  // kernel's last CTAs still run; A, the weights, C and the split-K workspace
  // are touched only after the dependency wait.
  grid_dependency_wait();
  if (threadIdx.x == 0) launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------- activation producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      Item w;
      for (int j = 0; ok && next_item(sched, unit, units, j, kblocks, num_m, num_n, w); ++j) {
        const int row0 = w.mt * TILE_M + static_cast<int>(rank) * L::ROWS;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % A_STAGES;
          const uint32_t ph = (it / A_STAGES) & 1u;
          const bool free = PAIR ? mbar_wait_cluster(aempty(s), ph ^ 1u, abort_flag, status,
                                                     wait_limit_ns)
                                 : mbar_wait(aempty(s), ph ^ 1u, abort_flag, status,
                                             wait_limit_ns);
          if (!free) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(afull(s), L::ACT_BYTES);
          tma_load_2d(act_base + s * L::ACT_BYTES, &act_map, afull(s), kb * BK, row0);
        }
      }
      if (!ok) {  // let every copy already issued (the last `it`, at most A_STAGES) land
        for (uint32_t i = it > A_STAGES ? it - A_STAGES : 0; i < it; ++i)
          mbar_wait(afull(i % A_STAGES), (i / A_STAGES) & 1u, never, nullptr, 100000000ull);
      }
    }
  } else if (warp == 2) {
    // ----------------------------------------------------- weight producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      Item w;
      for (int j = 0; ok && next_item(sched, unit, units, j, kblocks, num_m, num_n, w); ++j) {
        const int nt = w.nt * CG + static_cast<int>(rank);
        const uint8_t* wblk = tiles + static_cast<size_t>(nt) * kblocks * WBLOCK_BYTES;
        const __half* sblk = scales + static_cast<size_t>(nt) * groups * TILE_N;
        for (int kb = w.kb0; kb < w.kb1; ++kb, ++it) {
          const int s = it % W_STAGES;
          const uint32_t ph = (it / W_STAGES) & 1u;
          if (!mbar_wait(wempty(s), ph ^ 1u, abort_flag, status, wait_limit_ns)) {
            ok = false;
            break;
          }
          int g0, sbytes;
          if (GROUP == 32) { g0 = 2 * kb; sbytes = 512; }
          else if (GROUP == 64) { g0 = kb; sbytes = 256; }
          else { g0 = kb >> 1; sbytes = 256; }
          mbar_arrive_expect_tx(wfull(s), WBLOCK_BYTES + sbytes);
          bulk_load(w_base + s * W_SLOT, wblk + static_cast<size_t>(kb) * WBLOCK_BYTES,
                    WBLOCK_BYTES, wfull(s));
          bulk_load(w_base + s * W_SLOT + WBLOCK_BYTES, sblk + static_cast<size_t>(g0) * TILE_N,
                    sbytes, wfull(s));
        }
      }
      if (!ok) {  // let every copy already issued (the last `it`, at most W_STAGES) land
        for (uint32_t i = it > W_STAGES ? it - W_STAGES : 0; i < it; ++i)
          mbar_wait(wfull(i % W_STAGES), (i / W_STAGES) & 1u, never, nullptr, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0 && leader) {
      // pair: MMA-M 256 (128 weight columns from each CTA's TMEM)
      constexpr uint32_t IDESC = idesc_f16_f32(TILE_N * CG, TILE_M);
      uint32_t t_local = 0;
      // stage and phase of the next block in the activation ring (s, ph) and
      // the weight-stage ring (ts, tph; the same ring for single CTAs),
      // advanced by counting rather than dividing
      uint32_t s = 0, ph = 0, ts = 0, tph = 0;
      // shared-memory descriptors of stage 0; a stage or k16 step moves the
      // start-address field (16-byte units, no carry below 256 KB)
      const uint64_t b_desc0 = smem_desc_sw128(act_base);
      const uint64_t a_desc0 = smem_desc_sw128(deq_base);
      uint32_t uses0 = 0, uses1 = 0;  // segments committed on accumulator 0 / 1
      const int promo = sched.promo > 0 ? sched.promo : INT_MAX;
      bool ok = true;
      auto wait_in = [&](uint32_t bar, uint32_t parity) {
        return PAIR ? mbar_wait_cluster(bar, parity, abort_flag, status, wait_limit_ns)
                    : mbar_wait_lean(bar, parity, abort_flag, status, wait_limit_ns);
      };
      auto commit = [&](uint32_t bar) {
        if constexpr (PAIR) tc_commit_pair(bar);
        else tc_commit(bar);
      };
      Item w;
      for (int j = 0; ok && next_item(sched, unit, units, j, kblocks, num_m, num_n, w);
           ++j, ++t_local) {
        const int acc = t_local % ACC;
        uint32_t uses = acc == 0 ? uses0 : uses1;
        // the accumulator is free (its last segment drained)
        if (!wait_in(dempty(acc), (uses & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ACC_COL0 + acc * TILE_M;
        int left = promo;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (left == 0) {
            // segment boundary: hand the accumulator to the epilogue for
            // promotion; continue once the remainder is written back
            commit(dfull(acc));
            ++uses;
            if (!wait_in(dempty(acc), (uses & 1u) ^ 1u)) {
              ok = false;
              break;
            }
            tc_fence_after();
            left = promo;
          }
          --left;
          if (!wait_in(afull(s), ph) || (!UNI && !wait_in(tfull(ts), tph))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t b_desc = b_desc0 + ((s * L::ACT_BYTES) >> 4);
          // the item's first MMA starts the sum; later ones (including a
          // segment's first, onto the promoted remainder) accumulate
          const uint32_t first_acc = kb != w.kb0;
          if constexpr (PAIR) {
            const uint64_t a_desc = a_desc0 + ((ts * L::DEQ_BYTES) >> 4);
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16)  // 32 bytes of k per step
              mma_f16_ss_pair(d_tmem, a_desc + 2 * k16, b_desc + 2 * k16, IDESC,
                              k16 == 0 ? first_acc : 1u);
          } else {
            const uint32_t a_tmem = tmem_base + ts * T_COLS;
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16)  // 8 TMEM columns of k per step
              mma_f16_ts(d_tmem, a_tmem + 8 * k16, b_desc + 2 * k16, IDESC,
                         k16 == 0 ? first_acc : 1u);
          }
          commit(aempty(s));
          if constexpr (!UNI) commit(tempty(ts));
          if (++s == static_cast<uint32_t>(A_STAGES)) {
            s = 0;
            ph ^= 1u;
          }
          if constexpr (UNI) {
            ts = s;
            tph = ph;
          } else if (++ts == static_cast<uint32_t>(T_STAGES)) {
            ts = 0;
            tph ^= 1u;
          }
        }
        if (!ok) break;
        commit(dfull(acc));
        ++uses;
        if (acc == 0) uses0 = uses; else uses1 = uses;
      }
      // Every MMA this thread issued has completed before TMEM is freed (in
      // both CTAs of a pair: the commit arrives in each).
      commit(drain_bar);
    }
    if (PAIR && !leader && lane == 0) {
      // odd CTA of a pair: its activation half landed, its weight tile is
      // stored -> tell the even CTA, whose MMAs read them
      uint32_t total = 0;
      Item w;
      for (int j = 0; next_item(sched, unit, units, j, kblocks, num_m, num_n, w); ++j)
        total += static_cast<uint32_t>(w.kb1 - w.kb0);
      for (uint32_t it = 0; it < total; ++it) {
        const int s = it % A_STAGES;
        if (!mbar_wait(afull(s), (it / A_STAGES) & 1u, abort_flag, status, wait_limit_ns)) break;
        mbar_arrive_cluster_relaxed(lead(afull(s)));
        const int ts = it % T_STAGES;
        if (!mbar_wait(tfull(ts), (it / T_STAGES) & 1u, abort_flag, status, wait_limit_ns)) break;
        mbar_arrive_cluster_relaxed(lead(tfull(ts)));
      }
    }
    if (lane == 0) mbar_wait(drain_bar, 0, never, nullptr, 100000000ull);
  } else if (warp < FIRST_EPI_WARP) {
    // ---------------------------------------------------------------- dequant
    const int dgroup = (warp - FIRST_DEQ_WARP) >> 2;  // 0 (one group of four warps)
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;   // weight column inside the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t it = static_cast<uint32_t>(dgroup);
    uint32_t total = 0;  // 64-k blocks this CTA processes, over all its items
    Item w;
    for (int j = 0; next_item(sched, unit, units, j, kblocks, num_m, num_n, w); ++j) {
      total += static_cast<uint32_t>(w.kb1 - w.kb0);
    }
    for (; it < total; it += DEQ_GROUPS) {
      const int s = it % W_STAGES;
      const uint32_t ph = (it / W_STAGES) & 1u;
      const int ts = it % T_STAGES;
      const uint32_t tph = (it / T_STAGES) & 1u;
      {
        const bool landed = mbar_wait(wfull(s), ph, abort_flag, status, wait_limit_ns);
        if (!(PAIR ? __all_sync(0xffffffffu, landed) : landed)) break;
      }
      const uint32_t wsrc = w_base + s * W_SLOT + row * 16;
      uint4 c0, c1;
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(c0.x), "=r"(c0.y), "=r"(c0.z), "=r"(c0.w)
                   : "r"(wsrc));
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(c1.x), "=r"(c1.y), "=r"(c1.z), "=r"(c1.w)
                   : "r"(wsrc + 2048));
      uint16_t sb0, sb1;
      const uint32_t ssrc = w_base + s * W_SLOT + WBLOCK_BYTES + row * 2;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sb0) : "r"(ssrc));
      if (GROUP == 32)
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sb1) : "r"(ssrc + TILE_N * 2));
      else
        sb1 = sb0;
      __syncwarp();
      if (lane == 0) mbar_arrive(wempty(s));
      const uint32_t s0 = half_bits_x2(sb0), s1 = half_bits_x2(sb1);
      uint32_t r[32];
      const uint32_t wv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t sc = i < 4 ? s0 : s1;
        r[4 * i + 0] = decode_pair<0>(wv[i], sc);
        r[4 * i + 1] = decode_pair<1>(wv[i], sc);
        r[4 * i + 2] = decode_pair<2>(wv[i], sc);
        r[4 * i + 3] = decode_pair<3>(wv[i], sc);
      }
      const bool free = PAIR ? mbar_wait_cluster(tempty(ts), tph ^ 1u, abort_flag, status,
                                                 wait_limit_ns)
                             : mbar_wait(tempty(ts), tph ^ 1u, abort_flag, status, wait_limit_ns);
      if constexpr (PAIR) {
        // row `row` (128 bytes, 64 k) of this CTA's 128-row weight tile, in
        // the 128-byte swizzle the MMA's descriptor expects (16-byte chunk c
        // of row r at chunk c ^ (r % 8)); then, once every lane's stores are
        // visible to the tensor core (async proxy), one arrival per warp on
        // this CTA's barrier (the odd CTA's relay forwards it to the even
        // CTA). The wait's outcome is made warp-uniform so that no warp
        // splits across __syncwarp.
        if (!__all_sync(0xffffffffu, free)) break;
        const uint32_t tile = deq_base + ts * L::DEQ_BYTES + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                           tile + ((c ^ (row & 7)) << 4)),
                       "r"(r[4 * c]), "r"(r[4 * c + 1]), "r"(r[4 * c + 2]), "r"(r[4 * c + 3])
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(tfull(ts));
      } else {
        if (!free) break;
        tc_fence_after();
        tmem_st_32x32b_x32(tmem_base + lane_addr + ts * T_COLS, r);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(tfull(ts));
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue
    // Four warps per lane quarter; warp e covers accumulator columns
    // [part*TILE_M/4, (part+1)*TILE_M/4) of its 32 lanes. At each promotion
    // boundary of an item the warps fold the accumulator into the running sum
    // (hb: FP8 high parts, in registers) and write the remainder back. At
    // the item's end the whole slice (plus hb) is read into registers before
    // the accumulator is released, so the next tile's MMAs start while the
    // stores drain. A pair's epilogues release into the even CTA's barrier.
    constexpr int COLS = TILE_M / 4;
    const int e = warp - FIRST_EPI_WARP;
    const int quarter = warp & 3;
    const int half = e >> 2;  // which quarter of the columns
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int EPI_THREADS = NUM_EPI_WARPS * 32;
    auto release = [&](int acc) {
      if constexpr (PAIR) mbar_arrive_cluster_relaxed(lead(dempty(acc)));
      else mbar_arrive(dempty(acc));
    };
    auto item_at = [&](int jj, Item& wi) {
      next_item(sched, unit, units, jj, kblocks, num_m, num_n, wi);
    };
    PeerCopier<TILE_M, CG> copier{&out, M, (warp - FIRST_EPI_WARP) * 32 + lane};
    auto wait_full = [&](int acc, uint32_t parity) {
      if constexpr (MULTI) {
        // finished tiles go to the peers while this accumulator fills
        while (copier.pending()) {
          if (PAIR ? mbar_test_cluster(dfull(acc), parity) : mbar_test(dfull(acc), parity))
            return true;
          if (*abort_flag) return false;
          copier.copy(2, item_at, static_cast<int>(rank));
        }
      }
      return PAIR ? mbar_wait_cluster(dfull(acc), parity, abort_flag, status, wait_limit_ns)
                  : mbar_wait(dfull(acc), parity, abort_flag, status, wait_limit_ns);
    };
    uint32_t t_local = 0;
    uint32_t uses0 = 0, uses1 = 0;  // segments drained from accumulator 0 / 1
    bool failed = false;
    Item w;
    for (int j = 0; next_item(sched, unit, units, j, kblocks, num_m, num_n, w); ++j, ++t_local) {
      const int acc = t_local % ACC;
      uint32_t uses = acc == 0 ? uses0 : uses1;
      const uint32_t col0 = tmem_base + lane_addr + ACC_COL0 + acc * TILE_M + half * COLS;
      const int nblk = w.kb1 - w.kb0;
      const int nseg = sched.promo > 0 ? (nblk + sched.promo - 1) / sched.promo : 1;
      uint32_t hb[COLS / 4];  // running sum's high parts (e5m2 x4), zero at the start
#pragma unroll
      for (int q = 0; q < COLS / 4; ++q) hb[q] = 0u;
      for (int sg = 0; sg + 1 < nseg; ++sg, ++uses) {
        const bool ok = !failed && wait_full(acc, uses & 1u);
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < COLS / 16; ++c) {
            promote_chunk16(col0 + c * 16, hb);
            rotate_down2(hb);
            rotate_down2(hb);
          }
          tmem_st_wait();
        } else {
          failed = true;
        }
        tc_fence_before();
        release(acc);
      }
      const bool ok = !failed && wait_full(acc, uses & 1u);
      ++uses;
      if (acc == 0) uses0 = uses; else uses1 = uses;
      const int nt = w.nt * CG + static_cast<int>(rank);  // this CTA's 128 columns
      const int n = nt * TILE_N + row;
      const int m0 = w.mt * TILE_M + half * COLS;
      if (w.rem < 0) {
        // ------------------------------------------------ whole tile -> C
        if constexpr (MULTI) {
          const bool all = copies_epilogue<TILE_M, CG>(ok, out, M, w.mt, nt, half, row, m0, col0,
                                                       hb, lead(dempty(acc)));
          if (!ok) failed = true;
          if (all) copier.ready = j + 1;
          continue;
        }
        if (!ok) {
          failed = true;
          continue;
        }
        tc_fence_after();
        if constexpr (FP32_OUT) {
          // FP32 C: store each 16-column chunk as it is read.
          float* cp = static_cast<float*>(out.dst[0]) + static_cast<size_t>(m0) * N + n;
#pragma unroll 1
          for (int c = 0; c < COLS / 16; ++c) {
            uint32_t v[16];
            load_sum16(col0 + c * 16, hb, v);
            shift_down4(hb);
            if (c == COLS / 16 - 1) {
              tc_fence_before();
              release(acc);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (m0 + c * 16 + j < M)
                cp[static_cast<size_t>(c * 16 + j) * N] = __uint_as_float(v[j]);
          }
        } else {
          // each 16-column chunk is stored as it is read; the accumulator
          // is released once the last chunk is in registers
          __half* cp = static_cast<__half*>(out.dst[0]) + static_cast<size_t>(m0) * N + n;
          const int valid = min(COLS, M - m0);
          // the whole slice is read and rounded to FP16 pairs before the
          // accumulator is released; the stores follow
          __half2 hv[COLS / 2];
#pragma unroll
          for (int c = 0; c < COLS / 16; ++c) {
            uint32_t v[16];
            load_sum16(col0 + c * 16, &hb[c * 4], v);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              hv[c * 8 + j] = __floats2half2_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          }
          tc_fence_before();
          release(acc);
#pragma unroll
          for (int j = 0; j < COLS; ++j) {
            if (j < valid) *cp = (j & 1) ? __high2half(hv[j >> 1]) : __low2half(hv[j >> 1]);
            cp += N;
          }
        }
        continue;
      }
      // ------------------------------------------------ split item -> partial
      // Every epilogue warp takes the same barriers below whatever happened,
      // so a failed wait cannot strand the others at a barrier. A partial
      // tile is stored as float4 quads [m / 4][n][m % 4], so that each warp
      // access is 512 contiguous bytes. The two CTAs of a pair use their own
      // slots (slot * CG + rank) and tickets (tile * CG + rank).
      float4* mine = reinterpret_cast<float4*>(partials) +
                     static_cast<size_t>(w.slot * CG + static_cast<int>(rank)) * (TILE_M / 4) *
                         TILE_N;
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < COLS / 16; ++c) {
          uint32_t v[16];
          load_sum16(col0 + c * 16, &hb[c * 4], v);
          const int q0 = (half * COLS + c * 16) / 4;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            __stcg(mine + static_cast<size_t>(q0 + j) * TILE_N + row,
                   make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                               __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3])));
        }
        tc_fence_before();
        release(acc);
        __threadfence();
      }
      if (!epi_bar_and(EPI_THREADS, ok)) {
        failed = true;
        continue;
      }
      const int ticket = w.rem * CG + static_cast<int>(rank);
      if (warp == FIRST_EPI_WARP && lane == 0) *ticket_slot = atomicAdd(&tickets[ticket], 1u);
      epi_bar_sync(EPI_THREADS);
      const bool last = *ticket_slot == static_cast<uint32_t>(w.nparts - 1);
      if (last) {
        __threadfence();
        const float4* base = reinterpret_cast<const float4*>(partials) +
                             static_cast<size_t>(w.base_slot * CG + static_cast<int>(rank)) *
                                 (TILE_M / 4) * TILE_N +
                             static_cast<size_t>(half * COLS / 4) * TILE_N + row;
        const int mq = w.mt * TILE_M + half * COLS;
        switch (w.nparts) {
          case 2:
            reduce_partials<TILE_M, 2, 4, FP32_OUT, MULTI, CG>(base, out, mq, n, M, N, COLS / 4);
            break;
          case 3:
            reduce_partials<TILE_M, 3, 2, FP32_OUT, MULTI, CG>(base, out, mq, n, M, N, COLS / 4);
            break;
          default:
            reduce_partials<TILE_M, 4, 2, FP32_OUT, MULTI, CG>(base, out, mq, n, M, N, COLS / 4);
            break;
        }
      }
      epi_bar_sync(EPI_THREADS);  // the ticket slot is read by all before it changes
      if (last && warp == FIRST_EPI_WARP && lane == 0) tickets[ticket] = 0u;
      if constexpr (MULTI) copier.ready = j + 1;  // (split items are not copied)
    }
    if constexpr (MULTI) {
      // the rest of the copies, then make every peer store visible to the
      // other GPUs before the kernel ends
      if (!failed) copier.copy(INT_MAX, item_at, static_cast<int>(rank));
      __threadfence_system();
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves (or frees TMEM) while the other may still
  // arrive on its barriers or its MMAs run on its TMEM
  if constexpr (PAIR) cluster_barrier();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host

// Tail schedules are compared with a cost model fitted to B200 timings:
// one tile of `kblocks` blocks takes kblocks * kBlockUs; a tail of equal
// splits adds kSplitUs (the partial stores, tickets and reduction), a
// stream-K tail kStreamKUs (two partial items per CTA and up to four partial
// tiles per output tile).
constexpr double kBlockUs256 = 0.45, kBlockUs128 = 0.5;

int promote_blocks() {
  static const int v = [] {
    const char* e = std::getenv("I4G_PROMOTE_BLOCKS");
    const int b = e ? std::atoi(e) : 32;
    return b >= 0 ? b : 32;
  }();
  return v;
}
constexpr double kSplitUs = 12.0, kStreamKUs = 20.0;

int pair_mode() {
  static const int v = [] {
    const char* e = std::getenv("I4G_PAIR");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

// The stream-K tail is opt-in (I4G_STREAMK=1, read once): on B200 it gave an
// intermittently wrong output tile (about one launch in 12-16 at
// M = 1024, N = 3200, K = 12288, where every CTA owns two partial tiles), a
// race not yet found; whole tiles and equal splits were exact in every run.
int streamk_mode() {
  static const int v = [] {
    const char* e = std::getenv("I4G_STREAMK");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

int choose_cg(int tile_m, int N, int sm_count) {
  // CTA pairs for the 256-row tiles when the weight columns split into
  // 256-column pair tiles, with I4G_PAIR=1 (single CTAs by default: pairs run
  // no faster on B200 here).
  return (pair_mode() != 0 && tile_m == 256 && N % 256 == 0 && sm_count >= 2) ? 2 : 1;
}

int max_pairs(int sm_count) {
  // CTA pairs that can be resident at once (clusters are placed within GPCs,
  // so this can be fewer than sm_count / 2); per device, asked once.
  constexpr int kDevices = 64;
  static std::atomic<int> cached[kDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevices) return sm_count / 2;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  auto kernel = gemm_tc_kernel<256, 128, kOutHalf, 2>;
  using L = Cfg<256, 2>;
  static std::atomic<uint64_t> configured{0};
  int n = 0;
  if (ensure_dynamic_smem(kernel, L::DYN_BYTES, configured) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sm_count / 2));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = L::DYN_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();  // a failed query leaves no error behind
  v = (n > 0 && n < sm_count / 2) ? n : sm_count / 2;
  cached[dev].store(v, std::memory_order_relaxed);
  return v;
}

Plan make_plan(int tile_m, int M, int N, int K, int sm_count, size_t budget,
               bool allow_stream_k, int pairs) {
  // Work units are tiles of tile_m rows x (128 * cg) columns, one per CTA or
  // CTA pair; `units` of them run at once (pairs: `pairs` when given, else
  // sm_count / 2).
  const int cg = choose_cg(tile_m, N, sm_count);
  const int units = cg == 2 ? (pairs > 0 ? pairs : sm_count / 2) : sm_count;
  Plan p;
  p.cg = cg;
  const int tiles = ((M + tile_m - 1) / tile_m) * (N / (TILE_N * cg));
  const int kblocks = K / BK;
  const int promo = promote_blocks();
  p.sched = Sched{tiles, 1, tiles, 0, 0, promo};
  p.grid = cg * (tiles < units ? tiles : units);
  p.workspace_bytes = 0;
  if (budget == 0) return p;
  const int waves = tiles / units;
  const int rem = tiles - waves * units;
  if (rem == 0 || rem * cg * 4 > static_cast<int>(kTicketBytes)) return p;
  const size_t tile_bytes = static_cast<size_t>(cg) * tile_m * TILE_N * 4;
  const double t_tile = kblocks * (tile_m > 128 ? kBlockUs256 : kBlockUs128);
  double best = (waves + 1) * t_tile;  // whole tiles

  // equal splits of each tail tile: at most four, each at least eight blocks
  int f = units / rem;
  f = f < 4 ? f : 4;
  f = f < kblocks / 8 ? f : kblocks / 8;
  const size_t split_bytes = kTicketBytes + static_cast<size_t>(rem) * f * tile_bytes;
  if (f >= 2 && split_bytes <= budget && (waves + 1.0 / f) * t_tile + kSplitUs < best) {
    best = (waves + 1.0 / f) * t_tile + kSplitUs;
    p.sched = Sched{waves * units, f, waves * units + rem * f, 0, 0, promo};
    p.grid = cg * (p.sched.items < units ? p.sched.items : units);
    p.workspace_bytes = split_bytes;
  }
  if (allow_stream_k && cg == 1 && streamk_mode() != 0) {
    // equal shares of the tail's blocks, one per unit: at least eight blocks
    // each, at most four shares per tile, more shares than tiles (single
    // CTAs only, and only with I4G_STREAMK=1: see streamk_mode)
    const long run = static_cast<long>(rem) * kblocks;
    int chunks = units;
    chunks = chunks < 3 * rem ? chunks : 3 * rem;
    chunks = static_cast<long>(chunks) < run / 8 ? chunks : static_cast<int>(run / 8);
    int most = 0;
    for (int t = 0; t < rem && chunks > rem; ++t) {
      const long p0 = ((static_cast<long>(t) * kblocks + 1) * chunks - 1) / run;
      const long p1 = ((static_cast<long>(t + 1) * kblocks) * chunks - 1) / run;
      most = static_cast<int>(p1 - p0 + 1) > most ? static_cast<int>(p1 - p0 + 1) : most;
    }
    const size_t sk_bytes = kTicketBytes + static_cast<size_t>(rem + chunks - 1) * tile_bytes;
    const double sk_time = (waves + static_cast<double>(rem) / chunks) * t_tile + kStreamKUs;
    if (chunks > rem && most <= 4 && run * chunks < (1l << 31) && sk_bytes <= budget &&
        sk_time < best) {
      p.sched = Sched{waves * units, 1, 0, chunks, rem, promo};
      p.grid = cg * (waves > 0 ? units : chunks);
      p.workspace_bytes = sk_bytes;
    }
  }
  return p;
}

template <int TILE_M, int GROUP, int OUT, int CG>
cudaError_t launch_impl(const CUtensorMap& act_map, const uint8_t* tiles, const __half* scales,
                        const Outputs& out, int M, int N, int K, const Plan& plan, void* workspace,
                        int* status, unsigned long long wait_limit_ns, cudaStream_t stream) {
  using L = Cfg<TILE_M, CG>;
  auto kernel = gemm_tc_kernel<TILE_M, GROUP, OUT, CG>;
  static std::atomic<uint64_t> configured{0};  // devices set, per instantiation
  cudaError_t e = ensure_dynamic_smem(kernel, L::DYN_BYTES, configured);
  if (e != cudaSuccess) return e;
  uint32_t* tickets = static_cast<uint32_t*>(workspace);
  float* partials = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                                         kTicketBytes)
                              : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = L::DYN_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (CG > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = CG;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, act_map, tiles, scales, out, M, N, K, plan.sched,
                            tickets, partials, status, wait_limit_ns);
}

template <int TILE_M, int OUT, int CG>
cudaError_t launch_group(const CUtensorMap& act_map, const uint8_t* tiles,
                         const __half* scales, const Outputs& out, int M, int N, int K,
                         int group, const Plan& plan, void* workspace, int* status,
                         unsigned long long wait_limit_ns, cudaStream_t stream) {
  switch (group) {
    case 32:
      return launch_impl<TILE_M, 32, OUT, CG>(act_map, tiles, scales, out, M, N, K, plan,
                                              workspace, status, wait_limit_ns, stream);
    case 64:
      return launch_impl<TILE_M, 64, OUT, CG>(act_map, tiles, scales, out, M, N, K, plan,
                                              workspace, status, wait_limit_ns, stream);
    default:
      return launch_impl<TILE_M, 128, OUT, CG>(act_map, tiles, scales, out, M, N, K, plan,
                                               workspace, status, wait_limit_ns, stream);
  }
}

template <int TILE_M, int GROUP>
KernelConfig config_of() {
  using L = Cfg<TILE_M, 1>;
  return KernelConfig{TILE_M, TILE_N, BK, TILE_N, TILE_M, L::A_STAGES, THREADS, L::DYN_BYTES};
}

template <int TILE_M, int GROUP>
cudaError_t resources_of(KernelResources* out) {
  auto kernel = gemm_tc_kernel<TILE_M, GROUP, kOutHalf, 1>;
  static std::atomic<uint64_t> configured{0};
  cudaError_t e = ensure_dynamic_smem(kernel, Cfg<TILE_M, 1>::DYN_BYTES, configured);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes a{};
  if ((e = cudaFuncGetAttributes(&a, kernel)) != cudaSuccess) return e;
  int active = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, kernel, THREADS,
                                                    Cfg<TILE_M, 1>::DYN_BYTES);
  if (e != cudaSuccess) return e;
  *out = KernelResources{a.numRegs, static_cast<int>(a.sharedSizeBytes), a.maxThreadsPerBlock,
                         active};
  return cudaSuccess;
}

bool config(int tile_m, int group, KernelConfig* out) {
#define I4G_TC_CFG(TM, G) \
  if (tile_m == TM && group == G) { *out = config_of<TM, G>(); return true; }
  I4G_TC_CFG(128, 32) I4G_TC_CFG(128, 64) I4G_TC_CFG(128, 128)
  I4G_TC_CFG(256, 32) I4G_TC_CFG(256, 64) I4G_TC_CFG(256, 128)
#undef I4G_TC_CFG
  return false;
}

cudaError_t resources(int tile_m, int group, KernelResources* out) {
#define I4G_TC_RES(TM, G) \
  if (tile_m == TM && group == G) return resources_of<TM, G>(out);
  I4G_TC_RES(128, 32) I4G_TC_RES(128, 64) I4G_TC_RES(128, 128)
  I4G_TC_RES(256, 32) I4G_TC_RES(256, 64) I4G_TC_RES(256, 128)
#undef I4G_TC_RES
  return cudaErrorInvalidValue;
}

int choose_tile_m(int M, int N, int sm_count) {
  // A 128 x N x 16 MMA costs about the same for any N <= 256, so N = 256
  // wins unless the activation rows (M) do not fill it.
  (void)N;
  (void)sm_count;
  return M <= 128 ? 128 : 256;
}

cudaError_t launch(const CUtensorMap& act_map, int tile_m, const uint8_t* tiles,
                   const __half* scales, const Outputs& out, bool fp32_out, int M, int N, int K,
                   int group, const Plan& plan, void* workspace, int* status,
                   unsigned long long wait_limit_ns, cudaStream_t stream) {
  const bool plain = out.count == 1 && out.ldc == N && out.col0 == 0;
  if (fp32_out && !plain) return cudaErrorInvalidValue;  // float C is one plain matrix
  const int kind = fp32_out ? kOutFloat : (plain ? kOutHalf : kOutHalfCopies);
#define I4G_TC_CASE(TM, KIND, CG)                                                          \
  if (tile_m == TM && kind == KIND && plan.cg == CG)                                       \
    return launch_group<TM, KIND, CG>(act_map, tiles, scales, out, M, N, K, group, plan,   \
                                      workspace, status, wait_limit_ns, stream);
  I4G_TC_CASE(128, kOutHalf, 1)
  I4G_TC_CASE(128, kOutFloat, 1)
  I4G_TC_CASE(128, kOutHalfCopies, 1)
  I4G_TC_CASE(256, kOutHalf, 1)
  I4G_TC_CASE(256, kOutFloat, 1)
  I4G_TC_CASE(256, kOutHalfCopies, 1)
  I4G_TC_CASE(256, kOutHalf, 2)
  I4G_TC_CASE(256, kOutFloat, 2)
  I4G_TC_CASE(256, kOutHalfCopies, 2)
#undef I4G_TC_CASE
  return cudaErrorInvalidValue;
}

}  // namespace tc
}  // namespace i4g
