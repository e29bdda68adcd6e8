/*
 * CPU oracle (test infrastructure only; see oracle.h for what it restates).
 * Build: oracle/Makefile, with -ffp-contract=off so that every multiply and
 * add rounds separately, as the reference's x86-64 host build does.
 */
#include "oracle.h"

#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

float i4o_h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      /* subnormal half: man * 2^-24, exact in binary32 */
      float v = (float)man * 0x1p-24f;
      return sign ? -v : v;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

uint16_t i4o_f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof(x));
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf stays inf, NaN becomes a quiet NaN */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  const int e = (int)(ax >> 23) - 127;
  const uint32_t mant = (ax & 0x7fffffu) | (ax >= 0x00800000u ? 0x800000u : 0u);
  if (e >= -14) {
    /* normal binary16 candidate: keep 10 of the 23 fraction bits */
    uint32_t h = ((uint32_t)(e + 15) << 10) | ((ax & 0x7fffffu) >> 13);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    if (h >= 0x7c00u) h = 0x7c00u; /* overflow rounds to infinity */
    return (uint16_t)(sign | h);
  }
  /* subnormal binary16: m = round(|f| * 2^24) */
  const int shift = -e - 1; /* >= 14 */
  if (shift > 24) return sign;
  uint32_t m = mant >> shift;
  const uint32_t rem = mant & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (m & 1u))) ++m;
  return (uint16_t)(sign | m);
}

void i4o_h2f_array(const uint16_t* h, float* f, size_t count) {
  for (size_t i = 0; i < count; ++i) f[i] = i4o_h2f(h[i]);
}

void i4o_f2h_array(const float* f, uint16_t* h, size_t count) {
  for (size_t i = 0; i < count; ++i) h[i] = i4o_f2h(f[i]);
}

int i4o_sign_extend(uint8_t nibble) {
  nibble &= 0x0f;
  return (int)(int8_t)(uint8_t)((nibble ^ 0x08u) - 0x08u);
}

/* std::max(a, b) == (a < b) ? b : a */
static float max_like_std(float a, float b) { return (a < b) ? b : a; }

/* int(x) for a float that is already integral, as x86-64 cvttss2si does it:
 * NaN and values outside int range give INT_MIN. */
static int x86_float_to_int(float r) {
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return INT_MIN;
  return (int)r;
}

void i4o_quantize(const uint16_t* b, uint8_t* packed, uint16_t* scales,
                  int K, int N, int group) {
  const int groups = (K + group - 1) / group;
  for (int g = 0; g < groups; ++g) {
    const int kend = (K < (g + 1) * group) ? K : (g + 1) * group;
    for (int n = 0; n < N; ++n) {
      float vmax = 0.0f;
      for (int k = g * group; k < kend; ++k)
        vmax = max_like_std(vmax, fabsf(i4o_h2f(b[(size_t)k * N + n])));
      scales[(size_t)g * N + n] = i4o_f2h(max_like_std(vmax / 7.0f, 1.0e-8f));
    }
  }
  const size_t total = (size_t)K * N;
  memset(packed, 0, total / 2);
  for (size_t e = 0; e < total; ++e) {
    const int k = (int)(e / (size_t)N);
    const int n = (int)(e % (size_t)N);
    const float s = i4o_h2f(scales[(size_t)(k / group) * N + n]);
    int q = x86_float_to_int(nearbyintf(i4o_h2f(b[e]) / s));
    q = q < 7 ? q : 7;
    q = q > -8 ? q : -8;
    if (e & 1) packed[e >> 1] |= (uint8_t)((q & 15) << 4);
    else packed[e >> 1] = (uint8_t)(q & 15);
  }
}

void i4o_dequantize(const uint8_t* packed, const uint16_t* scales, uint16_t* b,
                    int K, int N, int group) {
  const size_t total = (size_t)K * N;
  for (size_t e = 0; e < total; ++e) {
    const int k = (int)(e / (size_t)N);
    const int n = (int)(e % (size_t)N);
    const uint8_t x = packed[e >> 1];
    const int q = (e & 1) ? i4o_sign_extend((uint8_t)(x >> 4)) : i4o_sign_extend(x);
    b[e] = i4o_f2h((float)q * i4o_h2f(scales[(size_t)(k / group) * N + n]));
  }
}

void i4o_gemm_rows_fb(const uint16_t* a, const float* bf, float* c,
                      int M, int N, int K, int row0, int rows) {
  (void)M;
  for (int r = 0; r < rows; ++r) {
    float* crow = c + (size_t)r * N;
    for (int n = 0; n < N; ++n) crow[n] = 0.0f;
    const uint16_t* arow = a + (size_t)(row0 + r) * K;
    for (int k = 0; k < K; ++k) {
      const float av = i4o_h2f(arow[k]);
      const float* brow = bf + (size_t)k * N;
      for (int n = 0; n < N; ++n) crow[n] += av * brow[n];
    }
  }
}

void i4o_gemm_rows_fb_noise(const uint16_t* a, const float* bf, float* c, double* p2,
                            int M, int N, int K, int row0, int rows) {
  (void)M;
  for (int r = 0; r < rows; ++r) {
    float* crow = c + (size_t)r * N;
    double* prow = p2 + (size_t)r * N;
    for (int n = 0; n < N; ++n) {
      crow[n] = 0.0f;
      prow[n] = 0.0;
    }
    const uint16_t* arow = a + (size_t)(row0 + r) * K;
    for (int k = 0; k < K; ++k) {
      const float av = i4o_h2f(arow[k]);
      const float* brow = bf + (size_t)k * N;
      for (int n = 0; n < N; ++n) {
        crow[n] += av * brow[n];
        prow[n] += (double)crow[n] * (double)crow[n];
      }
    }
  }
}

void i4o_gemm_rows_f64(const uint16_t* a, const float* bf, double* c,
                       int M, int N, int K, int row0, int rows) {
  (void)M;
  for (int r = 0; r < rows; ++r) {
    double* crow = c + (size_t)r * N;
    for (int n = 0; n < N; ++n) crow[n] = 0.0;
    const uint16_t* arow = a + (size_t)(row0 + r) * K;
    for (int k = 0; k < K; ++k) {
      const double av = (double)i4o_h2f(arow[k]);
      const float* brow = bf + (size_t)k * N;
      for (int n = 0; n < N; ++n) crow[n] += av * (double)brow[n];
    }
  }
}

void i4o_gemm_rows(const uint16_t* a, const uint16_t* b, float* c,
                   int M, int N, int K, int row0, int rows) {
  /* B is widened to binary32 once (exact); the arithmetic is the reference
   * loop's: one FP32 product and one FP32 add per (m, k, n), k ascending. */
  const size_t bcount = (size_t)K * N;
  float* bf = (float*)malloc(bcount * sizeof(float));
  if (bf == NULL) {
    for (int r = 0; r < rows; ++r) {
      float* crow = c + (size_t)r * N;
      for (int n = 0; n < N; ++n) crow[n] = 0.0f;
      const uint16_t* arow = a + (size_t)(row0 + r) * K;
      for (int k = 0; k < K; ++k) {
        const float av = i4o_h2f(arow[k]);
        const uint16_t* brow = b + (size_t)k * N;
        for (int n = 0; n < N; ++n) crow[n] += av * i4o_h2f(brow[n]);
      }
    }
    return;
  }
  i4o_h2f_array(b, bf, bcount);
  i4o_gemm_rows_fb(a, bf, c, M, N, K, row0, rows);
  free(bf);
}

void i4o_abs_gemm_rows(const uint16_t* a, const uint16_t* b, float* c,
                       int M, int N, int K, int row0, int rows) {
  (void)M;
  for (int r = 0; r < rows; ++r) {
    float* crow = c + (size_t)r * N;
    for (int n = 0; n < N; ++n) crow[n] = 0.0f;
    const uint16_t* arow = a + (size_t)(row0 + r) * K;
    for (int k = 0; k < K; ++k) {
      const float av = fabsf(i4o_h2f(arow[k]));
      const uint16_t* brow = b + (size_t)k * N;
      for (int n = 0; n < N; ++n) crow[n] += av * fabsf(i4o_h2f(brow[n]));
    }
  }
}

i4o_error_metrics i4o_compare_half(const uint16_t* got, const uint16_t* ref,
                                   size_t count) {
  long double abs_sum = 0, sq_sum = 0, ref_sq = 0;
  i4o_error_metrics m = {0.0, 0.0, 0.0, 0.0};
  for (size_t i = 0; i < count; ++i) {
    const double g = i4o_h2f(got[i]), r = i4o_h2f(ref[i]);
    const double d = fabs(g - r);
    m.max_abs = m.max_abs < d ? d : m.max_abs;
    abs_sum += d;
    sq_sum += d * d;
    ref_sq += r * r;
  }
  m.mean_abs = (double)(abs_sum / count);
  m.rmse = sqrt((double)(sq_sum / count));
  m.relative_l2 = sqrt((double)(sq_sum / (ref_sq > 1.0e-30L ? ref_sq : 1.0e-30L)));
  return m;
}

static int ordered_half(uint16_t h) {
  /* map the sign-magnitude bit pattern onto a monotone integer line */
  return (h & 0x8000u) ? -(int)(h & 0x7fffu) : (int)h;
}

int i4o_ulp_distance(uint16_t a, uint16_t b) {
  const int d = ordered_half(a) - ordered_half(b);
  return d < 0 ? -d : d;
}

/* ------------------------------------------------------------------------ */
/* reference layouts                                                          */

static int q4(const uint8_t* packed, int k, int n, int N) {
  const size_t logical = (size_t)k * N + n;
  return (logical & 1) ? (packed[logical >> 1] >> 4) : (packed[logical >> 1] & 15);
}

static void put_nibble(uint8_t* dst, size_t idx, int q) {
  if (idx & 1) dst[idx >> 1] = (uint8_t)((dst[idx >> 1] & 0x0f) | ((q & 15) << 4));
  else dst[idx >> 1] = (uint8_t)((dst[idx >> 1] & 0xf0) | (q & 15));
}

/* layout.cuh:12-20, BN=128 BK=32 */
static size_t repacked_element_128x32(int k, int n, int K) {
  const int nt = n / 128, kt = k / 32, ni = n % 128, ki = k % 32;
  return ((size_t)nt * (K / 32) + kt) * (32 * 128) + (size_t)ki * 128 + ni;
}

void i4o_repack_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N) {
  memset(repacked, 0, (size_t)K * N / 2);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n)
      put_nibble(repacked, repacked_element_128x32(k, n, K), q4(packed, k, n, N));
}

void i4o_inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed,
                               int K, int N) {
  memset(packed, 0, (size_t)K * N / 2);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) {
      const size_t r = repacked_element_128x32(k, n, K);
      const int q = (r & 1) ? (repacked[r >> 1] >> 4) : (repacked[r >> 1] & 15);
      put_nibble(packed, (size_t)k * N + n, q);
    }
}

void i4o_repack_scales_128(const uint16_t* scales, uint16_t* repacked,
                           int K, int N, int group) {
  const int groups = K / group;
  for (int g = 0; g < groups; ++g)
    for (int n = 0; n < N; ++n)
      repacked[((size_t)(n / 128) * groups + g) * 128 + n % 128] =
          scales[(size_t)g * N + n];
}

static uint16_t mma_fragment(const uint8_t* packed, int k0, int n, int N) {
  return (uint16_t)(q4(packed, k0, n, N) | (q4(packed, k0 + 1, n, N) << 4) |
                    (q4(packed, k0 + 8, n, N) << 8) |
                    (q4(packed, k0 + 9, n, N) << 12));
}

void i4o_repack_mma_128x32(const uint8_t* packed, uint8_t* repacked,
                           int K, int N) {
  const int ktiles = K / 32, ntiles = N / 128;
  for (int nt = 0; nt < ntiles; ++nt)
    for (int kt = 0; kt < ktiles; ++kt)
      for (int k16 = 0; k16 < 2; ++k16)
        for (int wn = 0; wn < 2; ++wn)
          for (int j = 0; j < 8; ++j)
            for (int lane = 0; lane < 32; ++lane) {
              const int n = nt * 128 + wn * 64 + j * 8 + (lane >> 2);
              const int k0 = kt * 32 + k16 * 16 + (lane & 3) * 2;
              const uint16_t w = mma_fragment(packed, k0, n, N);
              const size_t wi = ((size_t)nt * ktiles + kt) * 1024 +
                                (size_t)(((k16 * 2 + wn) * 8 + j) * 32 + lane);
              repacked[wi * 2] = (uint8_t)w;
              repacked[wi * 2 + 1] = (uint8_t)(w >> 8);
            }
}

void i4o_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked,
                                int K, int N) {
  const int ktiles = K / 32, ntiles = N / 128;
  for (int nt = 0; nt < ntiles; ++nt)
    for (int kt = 0; kt < ktiles; ++kt)
      for (int wn = 0; wn < 2; ++wn)
        for (int j = 0; j < 8; ++j)
          for (int lane = 0; lane < 32; ++lane) {
            const int n = nt * 128 + wn * 64 + j * 8 + (lane >> 2);
            uint32_t w = 0;
            for (int k16 = 0; k16 < 2; ++k16)
              w |= (uint32_t)mma_fragment(packed, kt * 32 + k16 * 16 + (lane & 3) * 2,
                                          n, N) << (16 * k16);
            const size_t wi = ((size_t)nt * ktiles + kt) * 512 +
                              (size_t)((wn * 8 + j) * 32 + lane);
            for (int byte = 0; byte < 4; ++byte)
              repacked[wi * 4 + byte] = (uint8_t)(w >> (8 * byte));
          }
}

/* ------------------------------------------------------------------------ */
/* B200 tile layout                                                           */

size_t i4o_umma_nibble_index(int k, int n, int K) {
  const int nt = n / 128, ni = n % 128;
  const int kb = k / 64, kk = k % 64;
  const int h = kk / 32, w = (kk % 32) / 8, e = kk % 8;
  const int p = e / 2, hi = e % 2;
  const size_t word_byte = ((size_t)nt * (K / 64) + kb) * 4096 + (size_t)h * 2048 +
                           (size_t)ni * 16 + (size_t)w * 4;
  return word_byte * 2 + (size_t)(p + 4 * hi);
}

void i4o_repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N) {
  memset(tiles, 0, (size_t)K * N / 2);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n)
      put_nibble(tiles, i4o_umma_nibble_index(k, n, K), q4(packed, k, n, N));
}

void i4o_inverse_repack_umma(const uint8_t* tiles, uint8_t* packed,
                             int K, int N) {
  memset(packed, 0, (size_t)K * N / 2);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) {
      const size_t r = i4o_umma_nibble_index(k, n, K);
      const int q = (r & 1) ? (tiles[r >> 1] >> 4) : (tiles[r >> 1] & 15);
      put_nibble(packed, (size_t)k * N + n, q);
    }
}
