/*
 * CPU oracle for the fused W4A16 INT4 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: it is linked or
 * loaded by tests/, by __graft_entry__.smoke() and by the cpu_baseline leg of
 * bench.py, never by the product library (sm_120__gemm_b200/libi4g.so).
 *
 * It restates, in plain C, the CPU path of zichaowen8-prog/SM_120__GEMM:
 *   - i4o_quantize      follows src/reference.cu:6-26   (quantize_cpu)
 *   - i4o_dequantize    follows src/reference.cu:28-37  (dequantize_cpu)
 *   - i4o_compare_half  follows src/reference.cu:39-53  (compare_half)
 *   - i4o_gemm_rows     follows src/reference.cu:55-64  (cpu_gemm_fp32)
 *   - i4o_sign_extend   follows include/common.cuh:60-63 (sign_extend_int4)
 *   - the reference weight layouts follow include/layout.cuh:8-48 and the
 *     CPU mapping loops of src/main.cu:140-208.
 * Parity of this restatement is pinned against the reference's own compiled
 * sources (oracle/_ref, built by oracle/Makefile) through golden fixtures in
 * tests/golden/.
 *
 * Half values travel as uint16_t bit patterns (IEEE binary16).
 */
#ifndef I4G_ORACLE_H
#define I4G_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  double max_abs;
  double mean_abs;
  double rmse;
  double relative_l2;
} i4o_error_metrics;

/* IEEE binary16 <-> binary32, round-to-nearest-even (the semantics of the
 * CUDA host conversions __half2float / __float2half used by reference.cu). */
float i4o_h2f(uint16_t h);
uint16_t i4o_f2h(float f);
void i4o_h2f_array(const uint16_t* h, float* f, size_t count);
void i4o_f2h_array(const float* f, uint16_t* h, size_t count);

/* include/common.cuh:60-63 */
int i4o_sign_extend(uint8_t nibble);

/* src/reference.cu:6-26. packed: K*N/2 bytes, row-major, even element in the
 * low nibble. scales: ceil(K/group) x N halves, row-major. */
void i4o_quantize(const uint16_t* b, uint8_t* packed, uint16_t* scales,
                  int K, int N, int group);

/* src/reference.cu:28-37 */
void i4o_dequantize(const uint8_t* packed, const uint16_t* scales, uint16_t* b,
                    int K, int N, int group);

/* src/reference.cu:55-64 restricted to rows [row0, row0+rows) of A: the
 * single-accumulator m-k-n loop, FP32 multiply then FP32 add, sequential in k.
 * c holds rows*N floats (row row0 of A lands in row 0 of c). */
void i4o_gemm_rows(const uint16_t* a, const uint16_t* b, float* c,
                   int M, int N, int K, int row0, int rows);

/* i4o_gemm_rows with B already widened to binary32 (K*N floats). */
void i4o_gemm_rows_fb(const uint16_t* a, const float* bf, float* c,
                      int M, int N, int K, int row0, int rows);

/* Same loop with |a|*|b| in place of a*b: the per-output sum of absolute
 * products, used to bound the FP32 summation-order error of a different
 * (tensor-core) accumulation order. */
void i4o_abs_gemm_rows(const uint16_t* a, const uint16_t* b, float* c,
                       int M, int N, int K, int row0, int rows);

/* i4o_gemm_rows_fb that also returns, per output, the sum of the squares of
 * the loop's own running FP32 partial sums p_k (k = 1..K), in binary64.
 * 2^-24 * sqrt(sum p_k^2) is the scale of the rounding noise of FP32
 * summation for that output: each add contributes an error of at most
 * 2^-24 |p_k|, of either sign. */
void i4o_gemm_rows_fb_noise(const uint16_t* a, const float* bf, float* c, double* p2,
                            int M, int N, int K, int row0, int rows);

/* The exact product of the same operands: each FP16 x FP16 product is exact
 * in binary64 and the K products are summed in binary64 (k ascending), so
 * for K <= 2^20 the result is within far less than an FP16 ulp of the exact
 * sum. Rounded once to FP16 it is the best FP16 answer for each output: the
 * anchor of the GEMM parity gate. bf is B widened to binary32 (exact). */
void i4o_gemm_rows_f64(const uint16_t* a, const float* bf, double* c,
                       int M, int N, int K, int row0, int rows);

/* src/reference.cu:39-53 */
i4o_error_metrics i4o_compare_half(const uint16_t* got, const uint16_t* ref,
                                   size_t count);

/* Distance in units in the last place between two finite halves (ordered
 * integer distance of their bit patterns). */
int i4o_ulp_distance(uint16_t a, uint16_t b);

/* ---- reference weight layouts (include/layout.cuh, src/main.cu:140-208) --- */

/* Tile-contiguous nibbles [N/128][K/32][32][128] (layout.cuh:12-25). */
void i4o_repack_128x32(const uint8_t* packed, uint8_t* repacked, int K, int N);
/* Inverse of i4o_repack_128x32. */
void i4o_inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed,
                               int K, int N);
/* Scales [K/g][N] -> [N/128][K/g][128] (layout.cuh:27-32). */
void i4o_repack_scales_128(const uint16_t* scales, uint16_t* repacked,
                           int K, int N, int group);
/* Lane-native mma.m16n8k16 B-fragment words (layout.cuh:34-40,
 * main.cu:157-179). */
void i4o_repack_mma_128x32(const uint8_t* packed, uint8_t* repacked,
                           int K, int N);
/* Fragment pairs, two k16 fragments per uint32 (layout.cuh:42-48,
 * main.cu:181-207). */
void i4o_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked,
                                int K, int N);

/* ---- the B200 tile layout of this project (independent CPU mapping) ------
 * Blocks of 128 columns x 64 k, ordered [N/128][K/64]; 4096 bytes each.
 * Inside a block: [h = (k%64)/32][n%128][word = (k%32)/8] of uint32, and in
 * a word the element k%8 = 2p+hi sits at bit 4p + 16hi. */
size_t i4o_umma_nibble_index(int k, int n, int K);
void i4o_repack_umma(const uint8_t* packed, uint8_t* tiles, int K, int N);
void i4o_inverse_repack_umma(const uint8_t* tiles, uint8_t* packed,
                             int K, int N);

#ifdef __cplusplus
}
#endif

#endif
