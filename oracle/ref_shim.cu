// C entry points over the reference's own CPU path.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the unmodified src/reference.cu of zichaowen8-prog/SM_120__GEMM, where it
// lies in the reference checkout, into oracle/_ref/libi4g_ref.so. Tests use
// it to pin the C restatement in oracle/oracle.c and to generate the golden
// fixtures in tests/golden/; bench.py's reference arm times it as the
// reference's CPU implementation. Nothing in the product links it.
//
// The functions below only adapt pointers to the std::vector signatures of
// include/quant.cuh:24-29 (quantize_cpu, dequantize_cpu, compare_half,
// cpu_gemm_fp32) and fan row slices of cpu_gemm_fp32 out over threads.
#include "layout.cuh"
#include "quant.cuh"

#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

std::vector<half> to_half_vec(const uint16_t* p, size_t n) {
  std::vector<half> v(n);
  std::memcpy(v.data(), p, n * sizeof(uint16_t));
  return v;
}

void gemm_slice(const std::vector<half>& b, const uint16_t* a, float* c,
                int N, int K, int row0, int rows) {
  std::vector<half> a_rows = to_half_vec(a + static_cast<size_t>(row0) * K,
                                         static_cast<size_t>(rows) * K);
  std::vector<float> out;
  int4gemm::cpu_gemm_fp32(a_rows, b, out, rows, N, K);
  std::memcpy(c, out.data(), out.size() * sizeof(float));
}

}  // namespace

extern "C" {

void i4r_quantize(const uint16_t* b, uint8_t* packed, uint16_t* scales,
                  int K, int N, int group) {
  std::vector<half> hb = to_half_vec(b, static_cast<size_t>(K) * N);
  std::vector<uint8_t> p;
  std::vector<half> s;
  int4gemm::quantize_cpu(hb, p, s, K, N, group);
  std::memcpy(packed, p.data(), p.size());
  std::memcpy(scales, s.data(), s.size() * sizeof(uint16_t));
}

void i4r_dequantize(const uint8_t* packed, const uint16_t* scales, uint16_t* b,
                    int K, int N, int group) {
  const int groups = (K + group - 1) / group;
  std::vector<uint8_t> p(packed, packed + static_cast<size_t>(K) * N / 2);
  std::vector<half> s = to_half_vec(scales, static_cast<size_t>(groups) * N);
  std::vector<half> out;
  int4gemm::dequantize_cpu(p, s, out, K, N, group);
  std::memcpy(b, out.data(), out.size() * sizeof(uint16_t));
}

// Rows [row0, row0 + rows) of cpu_gemm_fp32(A, B16) into c (rows x N floats),
// split over `threads` std::threads, each running the unmodified
// cpu_gemm_fp32 on a disjoint row slice (rows are independent).
void i4r_gemm_rows(const uint16_t* a, const uint16_t* b16, float* c,
                   int M, int N, int K, int row0, int rows, int threads) {
  (void)M;
  const std::vector<half> b = to_half_vec(b16, static_cast<size_t>(K) * N);
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows;
  std::vector<std::thread> pool;
  const int base = rows / threads, extra = rows % threads;
  int r = 0;
  for (int t = 0; t < threads; ++t) {
    const int count = base + (t < extra ? 1 : 0);
    float* dst = c + static_cast<size_t>(r) * N;
    pool.emplace_back(gemm_slice, std::cref(b), a, dst, N, K, row0 + r, count);
    r += count;
  }
  for (auto& th : pool) th.join();
}

void i4r_compare_half(const uint16_t* got, const uint16_t* ref, size_t count,
                      double* out4) {
  const int4gemm::ErrorMetrics m =
      int4gemm::compare_half(to_half_vec(got, count), to_half_vec(ref, count));
  out4[0] = m.max_abs;
  out4[1] = m.mean_abs;
  out4[2] = m.rmse;
  out4[3] = m.relative_l2;
}

// The CUDA host conversions the reference relies on.
uint16_t i4r_f2h(float f) {
  const half h = __float2half(f);
  uint16_t bits;
  std::memcpy(&bits, &h, sizeof(bits));
  return bits;
}

float i4r_h2f(uint16_t bits) {
  half h;
  std::memcpy(&h, &bits, sizeof(bits));
  return __half2float(h);
}

// The input distribution of the reference's harness (src/main.cu:75-81):
// mt19937_64 seeded with `seed`, uniform float in [-0.5, 0.5), rounded to half.
void i4r_random_half(uint16_t* out, size_t count, uint64_t seed) {
  std::mt19937_64 gen(seed);
  std::uniform_real_distribution<float> dist(-0.5f, 0.5f);
  for (size_t i = 0; i < count; ++i) out[i] = i4r_f2h(dist(gen));
}

// Reference weight layouts built from the reference's own index functions
// (include/layout.cuh:8-48); the loops restate the CPU mapping checks of
// src/main.cu:147-207.
static int ref_q4(const uint8_t* src, int k, int n, int N) {
  const size_t logical = static_cast<size_t>(k) * N + n;
  return int((logical & 1) ? (src[logical >> 1] >> 4) : (src[logical >> 1] & 15));
}

void i4r_repack_128x32(const uint8_t* packed, uint8_t* out, int K, int N) {
  std::memset(out, 0, static_cast<size_t>(K) * N / 2);
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) {
      const int q = ref_q4(packed, k, n, N);
      const size_t dst = int4gemm::repacked_element<128, 32>(k, n, N, K);
      if (dst & 1) out[dst >> 1] |= uint8_t((q & 15) << 4);
      else out[dst >> 1] |= uint8_t(q & 15);
    }
}

void i4r_repack_scales_128(const uint16_t* scales, uint16_t* out, int K, int N,
                           int group) {
  const int groups = K / group;
  for (int g = 0; g < groups; ++g)
    for (int n = 0; n < N; ++n)
      out[int4gemm::repacked_scale_index<128>(g, n, N, groups)] =
          scales[static_cast<size_t>(g) * N + n];
}

void i4r_repack_mma_128x32(const uint8_t* packed, uint8_t* out, int K, int N) {
  const int ktiles = K / 32, ntiles = N / 128;
  for (int nt = 0; nt < ntiles; ++nt) for (int kt = 0; kt < ktiles; ++kt)
    for (int k16 = 0; k16 < 2; ++k16) for (int wn = 0; wn < 2; ++wn)
      for (int j = 0; j < 8; ++j) for (int lane = 0; lane < 32; ++lane) {
        const int n = nt * 128 + wn * 64 + j * 8 + (lane >> 2);
        const int k0 = kt * 32 + k16 * 16 + (lane & 3) * 2;
        const uint16_t word = uint16_t(ref_q4(packed, k0, n, N) |
            (ref_q4(packed, k0 + 1, n, N) << 4) | (ref_q4(packed, k0 + 8, n, N) << 8) |
            (ref_q4(packed, k0 + 9, n, N) << 12));
        const size_t wi = (static_cast<size_t>(nt) * ktiles + kt) * 1024 +
                          int4gemm::mma_fragment_word(k16, wn, j, lane);
        out[wi * 2] = uint8_t(word);
        out[wi * 2 + 1] = uint8_t(word >> 8);
      }
}

void i4r_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* out, int K, int N) {
  const int ktiles = K / 32, ntiles = N / 128;
  for (int nt = 0; nt < ntiles; ++nt) for (int kt = 0; kt < ktiles; ++kt)
    for (int wn = 0; wn < 2; ++wn) for (int j = 0; j < 8; ++j)
      for (int lane = 0; lane < 32; ++lane) {
        const int n = nt * 128 + wn * 64 + j * 8 + (lane >> 2);
        uint32_t pair = 0;
        for (int k16 = 0; k16 < 2; ++k16) {
          const int k0 = kt * 32 + k16 * 16 + (lane & 3) * 2;
          const uint16_t f = uint16_t(ref_q4(packed, k0, n, N) |
              (ref_q4(packed, k0 + 1, n, N) << 4) | (ref_q4(packed, k0 + 8, n, N) << 8) |
              (ref_q4(packed, k0 + 9, n, N) << 12));
          pair |= uint32_t(f) << (k16 * 16);
        }
        const size_t wi = (static_cast<size_t>(nt) * ktiles + kt) * 512 +
                          int4gemm::mma_fragment_pair_word(wn, j, lane);
        for (int b = 0; b < 4; ++b) out[wi * 4 + b] = uint8_t(pair >> (8 * b));
      }
}

}  // extern "C"
