// Preprocessing kernels: INT4 quantisation, dequantisation and the weight /
// scale layouts. All byte and index work; bit-exact against the reference's
// CPU path (quantize_cpu / dequantize_cpu, src/reference.cu:6-37) and its
// layouts (include/layout.cuh:8-48).
//
// Compiled without fast-math: the quantiser's two divisions (vmax / 7 and
// x / s) must be IEEE round-to-nearest to reproduce quantize_cpu's codes at
// rounding ties. (The reference's own GPU quantiser, src/quantize.cu:22,36,
// is built with --use_fast_math and so may differ from quantize_cpu there.)
#include "gemm_tc.h"
#include "ptx.cuh"

#include <climits>
#include <cuda_runtime.h>

namespace i4g {
namespace prep {
namespace {

constexpr int THREADS = 256;

__device__ __forceinline__ float max_like_std(float a, float b) { return (a < b) ? b : a; }

// int(x) of an integral float as x86-64 cvttss2si evaluates it in the
// reference's host build: NaN and out-of-range values give INT_MIN.
__device__ __forceinline__ int x86_float_to_int(float r) {
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT_MIN;
  return static_cast<int>(r);
}

__device__ __forceinline__ int quantize_one(float x, float s) {
  int q = x86_float_to_int(rintf(__fdiv_rn(x, s)));
  q = q < 7 ? q : 7;
  return q > -8 ? q : -8;
}

__device__ __forceinline__ int nibble_at(const uint8_t* __restrict__ p, size_t logical) {
  const uint8_t byte = p[logical >> 1];
  return (logical & 1) ? (byte >> 4) : (byte & 15);
}

// One thread per (column pair, group): the group abs-max of two adjacent
// columns (one 4-byte load per row, coalesced across the warp), the FP16
// scales, then the codes of those columns, written as whole bytes.
__global__ void quantize_kernel(const __half2* __restrict__ b, uint8_t* __restrict__ packed,
                                __half* __restrict__ scales, int K, int N, int group) {
  const int half_n = N >> 1;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  const int g = blockIdx.y;
  if (p >= half_n) return;
  const int k0 = g * group;
  const int k1 = min(K, k0 + group);
  float vmax0 = 0.0f, vmax1 = 0.0f;
  for (int k = k0; k < k1; ++k) {
    const float2 x = __half22float2(b[static_cast<size_t>(k) * half_n + p]);
    vmax0 = max_like_std(vmax0, fabsf(x.x));
    vmax1 = max_like_std(vmax1, fabsf(x.y));
  }
  const __half s0 = __float2half_rn(max_like_std(__fdiv_rn(vmax0, 7.0f), 1.0e-8f));
  const __half s1 = __float2half_rn(max_like_std(__fdiv_rn(vmax1, 7.0f), 1.0e-8f));
  scales[static_cast<size_t>(g) * N + 2 * p] = s0;
  scales[static_cast<size_t>(g) * N + 2 * p + 1] = s1;
  const float f0 = __half2float(s0), f1 = __half2float(s1);
  for (int k = k0; k < k1; ++k) {
    const float2 x = __half22float2(b[static_cast<size_t>(k) * half_n + p]);
    const int q0 = quantize_one(x.x, f0);
    const int q1 = quantize_one(x.y, f1);
    packed[static_cast<size_t>(k) * half_n + p] = static_cast<uint8_t>((q0 & 15) | ((q1 & 15) << 4));
  }
}

__device__ __forceinline__ int sext4(int nib) { return ((nib & 15) ^ 8) - 8; }

__device__ __forceinline__ __half dequant_one(int nib, __half s) {
  return __float2half_rn(static_cast<float>(sext4(nib)) * __half2float(s));
}

// Eight elements (four bytes) per thread, one 16-byte store. N % 8 == 0.
__global__ void dequant8_kernel(const uint32_t* __restrict__ packed,
                                const __half* __restrict__ scales, uint4* __restrict__ b,
                                size_t chunks, int N, int group) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const size_t e0 = i * 8;
  const int k = static_cast<int>(e0 / N);
  const int n = static_cast<int>(e0 - static_cast<size_t>(k) * N);
  const uint32_t w = packed[i];
  const __half* srow = scales + static_cast<size_t>(k / group) * N + n;
  __align__(16) __half out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) out[j] = dequant_one(static_cast<int>(w >> (4 * j)), srow[j]);
  b[i] = *reinterpret_cast<const uint4*>(out);
}

// Generic fallback: two elements (one byte) per thread. N even.
__global__ void dequant2_kernel(const uint8_t* __restrict__ packed,
                                const __half* __restrict__ scales, __half* __restrict__ b,
                                size_t bytes, int N, int group) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= bytes) return;
  const size_t e0 = i * 2;
  const int k = static_cast<int>(e0 / N);
  const int n = static_cast<int>(e0 - static_cast<size_t>(k) * N);
  const uint8_t w = packed[i];
  const __half* srow = scales + static_cast<size_t>(k / group) * N + n;
  b[e0] = dequant_one(w & 15, srow[0]);
  b[e0 + 1] = dequant_one(w >> 4, srow[1]);
}

// include/layout.cuh:12-20 with BN = 128, BK = 32.
__device__ __forceinline__ size_t tile128x32_element(int k, int n, int K) {
  const int nt = n >> 7, kt = k >> 5, ni = n & 127, ki = k & 31;
  return (static_cast<size_t>(nt) * (K >> 5) + kt) * 4096 + ki * 128 + ni;
}

// One output byte (two adjacent columns of one k row) per thread.
__global__ void repack_128x32_kernel(const uint8_t* __restrict__ packed,
                                     uint8_t* __restrict__ out, size_t bytes, int K, int N) {
  const size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (o >= bytes) return;
  const size_t e0 = o * 2;
  const size_t tile = e0 >> 12;
  const int within = static_cast<int>(e0 & 4095);
  const int ktiles = K >> 5;
  const int nt = static_cast<int>(tile / ktiles);
  const int kt = static_cast<int>(tile - static_cast<size_t>(nt) * ktiles);
  const int k = kt * 32 + (within >> 7);
  const int n = nt * 128 + (within & 127);
  const size_t logical = static_cast<size_t>(k) * N + n;
  out[o] = static_cast<uint8_t>(nibble_at(packed, logical) | (nibble_at(packed, logical + 1) << 4));
}

__global__ void inverse_repack_128x32_kernel(const uint8_t* __restrict__ rep,
                                             uint8_t* __restrict__ out, size_t bytes, int K,
                                             int N) {
  const size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (o >= bytes) return;
  const size_t e0 = o * 2;
  const int k = static_cast<int>(e0 / N);
  const int n = static_cast<int>(e0 - static_cast<size_t>(k) * N);
  out[o] = static_cast<uint8_t>(nibble_at(rep, tile128x32_element(k, n, K)) |
                                (nibble_at(rep, tile128x32_element(k, n + 1, K)) << 4));
}

// [K/g][N] -> [N/128][K/g][128] (include/layout.cuh:27-32).
__global__ void repack_scales_128_kernel(const __half* __restrict__ src, __half* __restrict__ dst,
                                         size_t count, int N, int groups) {
  const size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (o >= count) return;
  const int ni = static_cast<int>(o & 127);
  const size_t x = o >> 7;
  const int g = static_cast<int>(x % groups);
  const int nt = static_cast<int>(x / groups);
  dst[o] = src[static_cast<size_t>(g) * N + nt * 128 + ni];
}

// Four nibbles {k0, k0+1, k0+8, k0+9} of column n: one lane's mma.m16n8k16
// B-fragment word (include/layout.cuh:34-40).
__device__ __forceinline__ uint32_t mma_word(const uint8_t* __restrict__ p, int k0, int n,
                                             int N) {
  const size_t base = static_cast<size_t>(k0) * N + n;
  return static_cast<uint32_t>(nibble_at(p, base) | (nibble_at(p, base + N) << 4) |
                               (nibble_at(p, base + 8 * static_cast<size_t>(N)) << 8) |
                               (nibble_at(p, base + 9 * static_cast<size_t>(N)) << 12));
}

// Word order [k16][warp_n][n8][lane] inside each 32x128 tile.
__global__ void repack_mma_kernel(const uint8_t* __restrict__ packed, uint16_t* __restrict__ out,
                                  size_t words, int K, int N) {
  const size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (o >= words) return;
  const size_t tile = o >> 10;
  const int within = static_cast<int>(o & 1023);
  const int lane = within & 31, n8 = (within >> 5) & 7, wn = (within >> 8) & 1, k16 = within >> 9;
  const int ktiles = K >> 5;
  const int nt = static_cast<int>(tile / ktiles);
  const int kt = static_cast<int>(tile - static_cast<size_t>(nt) * ktiles);
  const int n = nt * 128 + wn * 64 + n8 * 8 + (lane >> 2);
  const int k0 = kt * 32 + k16 * 16 + (lane & 3) * 2;
  out[o] = static_cast<uint16_t>(mma_word(packed, k0, n, N));
}

// Word order [warp_n][n8][lane], k16 = 0 in the low half, 1 in the high half.
__global__ void repack_mma_pair_kernel(const uint8_t* __restrict__ packed,
                                       uint32_t* __restrict__ out, size_t pairs, int K, int N) {
  const size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (o >= pairs) return;
  const size_t tile = o >> 9;
  const int within = static_cast<int>(o & 511);
  const int lane = within & 31, n8 = (within >> 5) & 7, wn = within >> 8;
  const int ktiles = K >> 5;
  const int nt = static_cast<int>(tile / ktiles);
  const int kt = static_cast<int>(tile - static_cast<size_t>(nt) * ktiles);
  const int n = nt * 128 + wn * 64 + n8 * 8 + (lane >> 2);
  const int k0 = kt * 32 + (lane & 3) * 2;
  out[o] = mma_word(packed, k0, n, N) | (mma_word(packed, k0 + 16, n, N) << 16);
}

// Tile layout for the sm_100a kernels, one 128-column x 64-k block per CTA.
// The block's 64 rows x 64 bytes of row-major nibbles are staged in shared
// memory with 16-byte coalesced loads; each output word then gathers the
// eight k of one column: element k%8 = 2p + hi at bit 4p + 16hi.
__global__ void repack_umma_kernel(const uint8_t* __restrict__ packed, uint32_t* __restrict__ out,
                                   int K, int N) {
  __shared__ uint4 stage[64 * 4];  // [k][64 bytes]
  const int kblocks = K >> 6;
  const int blk = blockIdx.x;
  const int nt = blk / kblocks, kb = blk - nt * kblocks;
  const size_t row_bytes = static_cast<size_t>(N) >> 1;
  for (int i = threadIdx.x; i < 64 * 4; i += blockDim.x) {
    const int k = i >> 2, c = i & 3;
    stage[i] = *reinterpret_cast<const uint4*>(packed + static_cast<size_t>(kb * 64 + k) * row_bytes +
                                               nt * 64 + c * 16);
  }
  __syncthreads();
  const uint8_t* sb = reinterpret_cast<const uint8_t*>(stage);
  uint32_t* dst = out + static_cast<size_t>(blk) * 1024;
  for (int wi = threadIdx.x; wi < 1024; wi += blockDim.x) {
    const int h = wi >> 9, ni = (wi >> 2) & 127, w = wi & 3;
    const int kk0 = h * 32 + w * 8;
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint8_t byte = sb[(kk0 + e) * 64 + (ni >> 1)];
      const uint32_t nib = (ni & 1) ? (byte >> 4) : (byte & 15);
      word |= nib << (4 * (e >> 1) + 16 * (e & 1));
    }
    dst[wi] = word;
  }
}

__global__ void inverse_repack_umma_kernel(const uint32_t* __restrict__ tiles,
                                           uint8_t* __restrict__ packed, int K, int N) {
  __shared__ uint32_t stage[1024];
  const int kblocks = K >> 6;
  const int blk = blockIdx.x;
  const int nt = blk / kblocks, kb = blk - nt * kblocks;
  for (int i = threadIdx.x; i < 1024; i += blockDim.x)
    stage[i] = tiles[static_cast<size_t>(blk) * 1024 + i];
  __syncthreads();
  const size_t row_bytes = static_cast<size_t>(N) >> 1;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int kk = i >> 6, byte = i & 63;
    const int h = kk >> 5, w = (kk & 31) >> 3, e = kk & 7;
    const int shift = 4 * (e >> 1) + 16 * (e & 1);
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int ni = byte * 2 + j;
      v |= ((stage[h * 512 + ni * 4 + w] >> shift) & 15u) << (4 * j);
    }
    packed[static_cast<size_t>(kb * 64 + kk) * row_bytes + nt * 64 + byte] = static_cast<uint8_t>(v);
  }
}

inline unsigned blocks_for(size_t n) { return static_cast<unsigned>((n + THREADS - 1) / THREADS); }


// quantize_one(x, s) for eight rows of two columns of a group, without a
// division per element, for a scale s that is a finite normal FP16 number
// (the caller takes quantize_one for the rest). Such an s is vmax / 7
// rounded to FP16 (relative error <= 2^-11), so |x / s| <= 7.004 for every
// x of the group and no code needs clamping. With r = 1/s rounded,
// y = x * r is within 2^-20 of the quotient x / s and the rounded quotient
// fl(x / s) within 2^-22 of it. n = y rounded to an integer by adding
// 1.5 * 2^23 (ties to even; the low four bits of the sum are then n's code)
// and d = y - n (exact); when |d| < 1/2 - 2^-18 the quotient and its
// rounding lie strictly inside (n - 1/2, n + 1/2), so rint(fl(x / s)) = n.
// Otherwise (within 2^-18 of a rounding tie, or x NaN) the element needs
// quantize_one and codes8 returns false. Float pairs carry two columns.
__device__ __forceinline__ bool codes8(const __half2 (&x)[8], float2 r, uint32_t& lo,
                                       uint32_t& hi) {
  const float2 magic = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
  const float2 minus_one = make_float2(-1.0f, -1.0f);
  constexpr float kLim = 0.5f - 0x1p-18f;
  uint32_t tl[8], th[8];
  bool ok = true;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float2 y = __fmul2_rn(__half22float2(x[e]), r);
    const float2 t = __fadd2_rn(y, magic);
    const float2 d = __ffma2_rn(__fadd2_rn(t, neg_magic), minus_one, y);  // y - n
    ok &= (fabsf(d.x) < kLim) & (fabsf(d.y) < kLim);
    tl[e] = __float_as_uint(t.x);
    th[e] = __float_as_uint(t.y);
  }
  // element e of a column sits at bit 4 (e / 2) + 16 (e % 2): bytes 0..3 of
  // the word hold codes (e0, e2), (e4, e6), (e1, e3), (e5, e7) as low, high
  // nibble; gather each code's low byte, then merge the two nibbles
  auto pack = [](const uint32_t (&t)[8]) {
    const uint32_t a = __byte_perm(__byte_perm(t[0], t[4], 0x0040), __byte_perm(t[1], t[5], 0x0040),
                                   0x5410);
    const uint32_t b = __byte_perm(__byte_perm(t[2], t[6], 0x0040), __byte_perm(t[3], t[7], 0x0040),
                                   0x5410);
    return (a & 0x0F0F0F0Fu) | ((b << 4) & 0xF0F0F0F0u);
  };
  lo = pack(tl);
  hi = pack(th);
  return ok;
}

// One pass from FP16 weights to the GEMM's inputs: a CTA reads a 128-column
// x KC-row slab of B once (KC = max(64, group), whole groups and whole tile
// blocks), computes the slab's scales exactly as quantize_kernel does, and
// writes the codes straight into the tile layout of repack_umma_kernel and
// the scales into the 128-column layout of repack_scales_128_kernel. Output
// bytes are identical to quantize -> repack_umma + repack_scales_128.
//
// The slab sits in shared memory as rows of sixteen 16-byte chunks, chunk c
// of row k stored at c ^ (2 ((k / 8) % 4)): the code pass reads rows k, k+8,
// k+16, k+24 at once, which this spreads over all 32 banks.
//
// ROWMAJOR = true writes the reference's formats instead (quantize_cpu's
// packed bytes, row-major scales [K / g][N]); its code pass maps a warp to 32
// consecutive column pairs of the same 8 rows, so each row's 32 code bytes
// are one store.
template <int GROUP, bool ROWMAJOR>
__global__ void __launch_bounds__(THREADS)
    quantize_repack_kernel(const __half* __restrict__ b, void* __restrict__ codes,
                           __half* __restrict__ scales_out, int K, int N) {
  constexpr int KC = GROUP > 64 ? GROUP : 64;
  constexpr int GPC = KC / GROUP;           // groups per slab
  constexpr int P = THREADS / (64 * GPC);   // threads per (group, column pair)
  constexpr int RPP = GROUP / P;            // rows each of them scans
  static_assert(P >= 1 && (P & (P - 1)) == 0 && RPP % 8 == 0, "scale pass split");
  __shared__ __align__(16) __half slab[KC * 128];
  __shared__ float sf[GPC][128];  // scales
  __shared__ float sr[GPC][128];  // their rounded reciprocals; NaN: not a normal scale
  const int nt = blockIdx.x;
  const int kc = blockIdx.y;
  const int k0 = kc * KC;
  auto chunk_at = [](int row, int ch) { return row * 128 + ((ch ^ (2 * ((row >> 3) & 3))) << 3); };
  // B rows k0..k0+KC, columns 128 nt..: 16 chunks of 16 bytes per row
#pragma unroll
  for (int j = 0; j < KC * 16 / THREADS; ++j) {
    const int i = j * THREADS + threadIdx.x;
    const int r = i >> 4, ch = i & 15;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(
        b + static_cast<size_t>(k0 + r) * N + static_cast<size_t>(nt) * 128 + ch * 8));
    *reinterpret_cast<uint4*>(&slab[chunk_at(r, ch)]) = v;
  }
  __syncthreads();
  const int groups = K / GROUP;
  {
    // group abs-max of a column pair over RPP rows per thread, combined over
    // the P adjacent lanes of the pair (the maximum ignores NaN, as the
    // reference's std::max-style update does). Lane `part` takes the group's
    // 8-row runs part, part + P, ...: the eight rows of a run share one chunk
    // swizzle (one base address, then a 128-half row stride), and the P lanes
    // of a pair read runs with different swizzles, i.e. different banks.
    const int part = threadIdx.x % P;
    const int np = (threadIdx.x / P) % 64;
    const int gl = threadIdx.x / (P * 64);
    __half2 m = __float2half2_rn(0.0f);
#pragma unroll
    for (int q = 0; q < RPP / 8; ++q) {
      const int r8 = gl * GROUP + (q * P + part) * 8;
      const __half2* xp =
          reinterpret_cast<const __half2*>(&slab[chunk_at(r8, np >> 2) + 2 * (np & 3)]);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = __hmax2(m, __habs2(xp[e * 64]));
    }
#pragma unroll
    for (int o = 1; o < P; o <<= 1) m = __hmax2(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float2 vmax = __half22float2(m);
    const __half s0 = __float2half_rn(max_like_std(__fdiv_rn(vmax.x, 7.0f), 1.0e-8f));
    const __half s1 = __float2half_rn(max_like_std(__fdiv_rn(vmax.y, 7.0f), 1.0e-8f));
    if (part == 0) {
      // two 2-byte stores: the scale buffer need only be 2-byte aligned
      __half* sdst =
          ROWMAJOR ? scales_out + static_cast<size_t>(kc * GPC + gl) * N + nt * 128 + 2 * np
                   : scales_out + (static_cast<size_t>(nt) * groups + kc * GPC + gl) * 128 + 2 * np;
      sdst[0] = s0;
      sdst[1] = s1;
      const float f0 = __half2float(s0), f1 = __half2float(s1);
      const float kNaN = __int_as_float(0x7fffffff);
      sf[gl][2 * np] = f0;
      sf[gl][2 * np + 1] = f1;
      sr[gl][2 * np] = (f0 >= 0x1p-14f && f0 <= 65504.0f) ? __frcp_rn(f0) : kNaN;
      sr[gl][2 * np + 1] = (f1 >= 0x1p-14f && f1 <= 65504.0f) ? __frcp_rn(f1) : kNaN;
    }
  }
  __syncthreads();
  // tile-layout words of the slab's KC / 64 blocks: block [h][n][w]; each
  // thread makes the words of columns 2np and 2np + 1 (4 words apart)
  const int kblocks = K >> 6;
#pragma unroll 1
  for (int i = threadIdx.x; i < (KC / 64) * 512; i += THREADS) {
    const int jb = i >> 9, rr = i & 511;
    const int h = rr >> 8;
    const int np = ROWMAJOR ? (rr & 63) : ((rr >> 2) & 63);
    const int w = ROWMAJOR ? ((rr >> 6) & 3) : (rr & 3);
    const int kk0 = jb * 64 + h * 32 + w * 8;  // row inside the slab
    const int gl = kk0 / GROUP;
    // the 8 rows kk0 .. kk0 + 7 share one chunk swizzle: one base address,
    // then a row stride of 128 halves
    const __half2* xp =
        reinterpret_cast<const __half2*>(&slab[chunk_at(kk0, np >> 2) + 2 * (np & 3)]);
    __half2 x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = xp[e * 64];
    uint32_t lo, hi;
    // a NaN reciprocal (scale not a finite normal number) makes every d NaN
    if (!codes8(x, make_float2(sr[gl][2 * np], sr[gl][2 * np + 1]), lo, hi)) {
      const float f0 = sf[gl][2 * np], f1 = sf[gl][2 * np + 1];
      lo = hi = 0u;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int sh = 4 * (e >> 1) + 16 * (e & 1);
        const float2 v = __half22float2(x[e]);
        lo |= static_cast<uint32_t>(quantize_one(v.x, f0) & 15) << sh;
        hi |= static_cast<uint32_t>(quantize_one(v.y, f1) & 15) << sh;
      }
    }
    if constexpr (ROWMAJOR) {
      // row k0 + kk0 + e: byte (column pair nt * 64 + np) = lo code | hi code << 4
      uint8_t* dst = static_cast<uint8_t*>(codes) + static_cast<size_t>(k0 + kk0) * (N / 2) +
                     nt * 64 + np;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int sh = 4 * (e >> 1) + 16 * (e & 1);
        dst[static_cast<size_t>(e) * (N / 2)] =
            static_cast<uint8_t>(((lo >> sh) & 15u) | (((hi >> sh) & 15u) << 4));
      }
    } else {
      uint32_t* dst = static_cast<uint32_t*>(codes) +
                      (static_cast<size_t>(nt) * kblocks + kc * (KC / 64) + jb) * 1024 + h * 512 +
                      (2 * np) * 4 + w;
      dst[0] = lo;
      dst[4] = hi;
    }
  }
}

template <int GROUP, bool ROWMAJOR>
void launch_slab(dim3 grid, const __half* b, void* codes, __half* scales, int K, int N,
                 cudaStream_t stream) {
  quantize_repack_kernel<GROUP, ROWMAJOR><<<grid, THREADS, 0, stream>>>(b, codes, scales, K, N);
}

}  // namespace

cudaError_t quantize_repack(const __half* b, uint8_t* tiles, __half* rscales, int K, int N,
                            int group, cudaStream_t stream) {
  const int kc = group > 64 ? group : 64;
  const dim3 grid(N / 128, K / kc);
  switch (group) {
    case 32: launch_slab<32, false>(grid, b, tiles, rscales, K, N, stream); break;
    case 64: launch_slab<64, false>(grid, b, tiles, rscales, K, N, stream); break;
    case 128: launch_slab<128, false>(grid, b, tiles, rscales, K, N, stream); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t quantize(const __half* b, uint8_t* packed, __half* scales, int K, int N, int group,
                     cudaStream_t stream) {
  // whole slabs (and a 16-byte aligned B): one pass, B read once
  const int kc = group > 64 ? group : 64;
  if ((group == 32 || group == 64 || group == 128) && N % 128 == 0 && K >= kc && K % kc == 0 &&
      reinterpret_cast<uintptr_t>(b) % 16 == 0) {
    const dim3 grid(N / 128, K / kc);
    switch (group) {
      case 32: launch_slab<32, true>(grid, b, packed, scales, K, N, stream); break;
      case 64: launch_slab<64, true>(grid, b, packed, scales, K, N, stream); break;
      default: launch_slab<128, true>(grid, b, packed, scales, K, N, stream); break;
    }
    return cudaGetLastError();
  }
  // any other shape (partial groups, odd widths): one thread per column pair and group
  const int groups = (K + group - 1) / group;
  const int pairs = N / 2;
  const dim3 grid((pairs + 127) / 128, groups);
  quantize_kernel<<<grid, 128, 0, stream>>>(reinterpret_cast<const __half2*>(b), packed, scales, K,
                                            N, group);
  return cudaGetLastError();
}

cudaError_t dequantize(const uint8_t* packed, const __half* scales, __half* b, int K, int N,
                       int group, cudaStream_t stream) {
  const size_t elements = static_cast<size_t>(K) * N;
  if (N % 8 == 0) {
    const size_t chunks = elements / 8;
    dequant8_kernel<<<blocks_for(chunks), THREADS, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(packed), scales, reinterpret_cast<uint4*>(b), chunks, N,
        group);
  } else {
    const size_t bytes = elements / 2;
    dequant2_kernel<<<blocks_for(bytes), THREADS, 0, stream>>>(packed, scales, b, bytes, N, group);
  }
  return cudaGetLastError();
}

cudaError_t repack_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                          cudaStream_t stream) {
  const size_t bytes = static_cast<size_t>(K) * N / 2;
  repack_128x32_kernel<<<blocks_for(bytes), THREADS, 0, stream>>>(packed, repacked, bytes, K, N);
  return cudaGetLastError();
}

cudaError_t inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed, int K, int N,
                                  cudaStream_t stream) {
  const size_t bytes = static_cast<size_t>(K) * N / 2;
  inverse_repack_128x32_kernel<<<blocks_for(bytes), THREADS, 0, stream>>>(repacked, packed, bytes,
                                                                          K, N);
  return cudaGetLastError();
}

cudaError_t repack_scales_128(const __half* scales, __half* repacked, int K, int N, int group,
                              cudaStream_t stream) {
  const int groups = K / group;
  const size_t count = static_cast<size_t>(groups) * N;
  repack_scales_128_kernel<<<blocks_for(count), THREADS, 0, stream>>>(scales, repacked, count, N,
                                                                      groups);
  return cudaGetLastError();
}

cudaError_t repack_mma_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                              cudaStream_t stream) {
  const size_t words = static_cast<size_t>(K) * N / 4;
  repack_mma_kernel<<<blocks_for(words), THREADS, 0, stream>>>(
      packed, reinterpret_cast<uint16_t*>(repacked), words, K, N);
  return cudaGetLastError();
}

cudaError_t repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N,
                                   cudaStream_t stream) {
  const size_t pairs = static_cast<size_t>(K) * N / 8;
  repack_mma_pair_kernel<<<blocks_for(pairs), THREADS, 0, stream>>>(
      packed, reinterpret_cast<uint32_t*>(repacked), pairs, K, N);
  return cudaGetLastError();
}

cudaError_t repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N, cudaStream_t stream) {
  const int blocks = (N / 128) * (K / 64);
  repack_umma_kernel<<<blocks, THREADS, 0, stream>>>(packed, reinterpret_cast<uint32_t*>(tiles), K,
                                                     N);
  return cudaGetLastError();
}

cudaError_t inverse_repack_umma(const uint8_t* tiles, uint8_t* packed, int K, int N,
                                cudaStream_t stream) {
  const int blocks = (N / 128) * (K / 64);
  inverse_repack_umma_kernel<<<blocks, THREADS, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(tiles), packed, K, N);
  return cudaGetLastError();
}

}  // namespace prep
}  // namespace i4g
