/*
 * i4g: B200-native (sm_100a) fused W4A16 INT4 weight-only GEMM, C ABI.
 *
 *   C[M,N] = A_fp16[M,K] x dequant(B_int4[K,N], fp16 group scale),
 *   FP32 accumulation, FP16 (or FP32) output, group size 32 / 64 / 128.
 *
 * This is the drop-in boundary for the hot path of zichaowen8-prog/SM_120__GEMM.
 * Each entry point replaces one host function of the reference's C++ API
 * (cited beside it); the C++ wrappers with the reference's exact signatures
 * are in int4gemm.hpp.
 *
 * Conventions
 *   - Pointers are caller-owned device memory; no entry point allocates
 *     device memory. `half` data is passed as void* (IEEE binary16).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is
 *     stream-ordered; no entry point synchronises the host.
 *   - Return 0 (I4G_OK) or a negative i4g_status. Shapes, group and
 *     alignment are checked before anything is launched.
 *   - Layouts: A is row-major [M][K]; C row-major [M][N]; `packed` is the
 *     reference's row-major nibble stream (element k*N+n, even element in the
 *     low nibble, src/quantize.cu:25-39); `scales` is [ceil(K/g)][N].
 *     The GEMM consumes the "tile" weight layout written by i4g_repack_umma
 *     (blocks of 128 columns x 64 k) and the scale layout written by
 *     i4g_repack_scales_128 ([N/128][K/g][128], include/layout.cuh:27-32).
 */
#ifndef I4G_H
#define I4G_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  I4G_OK = 0,
  I4G_ERR_NULL_POINTER = -1,   /* a required pointer is NULL */
  I4G_ERR_SHAPE = -2,          /* M/N/K out of range or not a tile multiple */
  I4G_ERR_GROUP = -3,          /* group size not 32, 64 or 128, or K % group */
  I4G_ERR_ALIGNMENT = -4,      /* pointer not aligned as the layout needs */
  I4G_ERR_CUDA = -5,           /* a CUDA runtime call failed */
  I4G_ERR_DRIVER = -6,         /* tensor-map encoding failed */
  I4G_ERR_DEVICE = -7,         /* current device is not sm_100 */
  I4G_ERR_TIMEOUT = -8,        /* a device-side wait hit its limit */
  I4G_ERR_VARIANT = -9         /* unknown kernel variant */
} i4g_status;

/* Kernel selection for i4g_gemm_variant. */
typedef enum {
  I4G_VARIANT_AUTO = 0,        /* the dispatch i4g_gemm uses */
  I4G_VARIANT_TC = 1,          /* tcgen05 + TMEM warp-specialised kernel */
  I4G_VARIANT_DECODE = 2       /* tensor-core GEMV-style kernel, M <= 16 */
} i4g_variant;

/* Human-readable text for a status code (static storage). */
const char* i4g_status_string(int status);
/* Text of the last CUDA / driver error seen on this host thread. */
const char* i4g_last_error(void);
/* Version of the tile layout written by i4g_repack_umma. */
int i4g_layout_version(void);

/* ---- preprocessing (include/quant.cuh:6-21) ------------------------------ */

/* launch_quantize (include/quant.cuh:6-7, src/quantize.cu:54-62).
 * Codes and scales are bit-identical to quantize_cpu (src/reference.cu:6-26).
 * K % group may be non-zero (the last group is partial), as in the reference.
 * N must be even. */
int i4g_quantize(const void* b, uint8_t* packed, void* scales,
                 int K, int N, int group, void* stream);

/* launch_dequantize (include/quant.cuh:8-9, src/quantize.cu:64-69):
 * b[k][n] = half(q * scale), bit-identical to dequantize_cpu. */
int i4g_dequantize(const uint8_t* packed, const void* scales, void* b,
                   int K, int N, int group, void* stream);

/* launch_repack_128x32 (include/quant.cuh:10-12, src/repack.cu:124-135):
 * tile-contiguous nibbles [N/128][K/32][32][128] plus the 128-column scale
 * layout. K % 32 == 0, N % 128 == 0, K % group == 0. */
int i4g_repack_128x32(const uint8_t* packed, const void* scales,
                      uint8_t* repacked, void* repacked_scales,
                      int K, int N, int group, void* stream);

/* launch_inverse_repack_128x32 (include/quant.cuh:13-14, src/repack.cu:137-142). */
int i4g_inverse_repack_128x32(const uint8_t* repacked, uint8_t* packed,
                              int K, int N, void* stream);

/* launch_repack_mma_128x32 (include/quant.cuh:15-16, src/repack.cu:144-152):
 * the reference's mma.sync lane-native B-fragment words. */
int i4g_repack_mma_128x32(const uint8_t* packed, uint8_t* repacked,
                          int K, int N, void* stream);

/* launch_repack_mma_pair_128x32 (include/quant.cuh:17-18, src/repack.cu:154-162). */
int i4g_repack_mma_pair_128x32(const uint8_t* packed, uint8_t* repacked,
                               int K, int N, void* stream);

/* launch_repack_scales_128 (include/quant.cuh:19-21, src/repack.cu:164-174):
 * [K/g][N] -> [N/128][K/g][128]. This is also the GEMM's scale layout. */
int i4g_repack_scales_128(const void* scales, void* repacked_scales,
                          int K, int N, int group, void* stream);

/* New layout for the sm_100a kernels (replaces the lane-native repacks that
 * launch_final consumes, src/main.cu:322-329). Blocks of 128 columns x 64 k,
 * ordered [N/128][K/64], 4096 bytes each; inside a block
 * [h = (k%64)/32][n%128][w = (k%32)/8] uint32 words, and in a word element
 * k%8 = 2p + hi at bit 4p + 16hi. An N-slice at a multiple of 128 columns is
 * one contiguous byte range. K % 64 == 0, N % 128 == 0. */
int i4g_repack_umma(const uint8_t* packed, uint8_t* tiles,
                    int K, int N, void* stream);
/* Inverse of i4g_repack_umma (test and serialisation aid). */
int i4g_inverse_repack_umma(const uint8_t* tiles, uint8_t* packed,
                            int K, int N, void* stream);

/* One-pass quantize + repack (the one-shot path of src/main.cu:320-331,
 * launch_quantize followed by the repacks, fused): B fp16 [K][N] ->
 * tiles (i4g_repack_umma layout) + scales in the i4g_repack_scales_128 layout,
 * reading B once. Bytes identical to i4g_quantize -> i4g_repack_umma +
 * i4g_repack_scales_128. K % max(64, group) == 0, N % 128 == 0. */
int i4g_quantize_repack(const void* b, uint8_t* tiles, void* scales_repacked,
                        int K, int N, int group, void* stream);

/* ---- fused GEMM (include/kernels.cuh:24-25, 81-83) ------------------------ */

/* launch_final (kernels/gemm_final.cu:5-13): C fp16 [M][N] = A x dequant(B).
 * tiles: i4g_repack_umma output; scales: i4g_repack_scales_128 output.
 * Any M >= 1; N % 128 == 0; K % 64 == 0; K % group == 0; group in {32,64,128}
 * (other groups are rejected, where the reference silently ran g128).
 * Dispatch: M <= 16 uses the decode kernel, larger M the tcgen05 kernel. */
int i4g_gemm(const void* A, const uint8_t* tiles, const void* scales, void* C,
             int M, int N, int K, int group, void* stream);

/* launch_final_fp32 (include/kernels.cuh:81, kernels/gemm_v09_async.cu:61):
 * the same product with an FP32 C (tcgen05 kernel, FP32 epilogue). */
int i4g_gemm_fp32(const void* A, const uint8_t* tiles, const void* scales,
                  float* C, int M, int N, int K, int group, void* stream);

/* i4g_gemm with an explicit kernel choice (tests and benchmarks). */
int i4g_gemm_variant(const void* A, const uint8_t* tiles, const void* scales,
                     void* C, int M, int N, int K, int group, int variant,
                     void* stream);

/* ---- split-K workspace (no counterpart in the reference) ------------------ */

/* The tcgen05 kernel runs ceil(M/TILE_M) x N/128 output tiles on one CTA per
 * SM. When the tile count is not a multiple of the SM count, the *_ws entry
 * points share the tiles of the last, partial wave out along K over all SMs
 * (each leftover tile split 2 to 4 ways; with the I4G_STREAMK=1 environment
 * variable, read at the first launch, stream-K where it is cheaper: equal
 * shares of the leftover tiles' 64-k blocks, one per CTA; opt-in because it
 * gave an intermittently wrong tile on B200, a race not yet found) and
 * reduce the FP32 partial tiles through a caller-owned workspace, in a fixed
 * order, so results are bitwise reproducible and within the usual FP32
 * accumulation tolerance of the unsplit kernel. The decode kernel (M <= 16,
 * FP16 C) uses the workspace the same way for its own stream-K schedule:
 * two CTAs per SM take equal runs of (128-column tile, 64-k block) units, so
 * every SM does the same work whatever N is, and a tile split between CTAs
 * is reduced by the last of them to finish, in run order. Without a
 * workspace it spreads each tile's K over a thread-block cluster instead.
 *
 * i4g_gemm_workspace_size: bytes needed for this shape on the current device
 * (0 when nothing would be split, e.g. a whole number of waves).
 *
 * i4g_gemm_ws / i4g_gemm_fp32_ws: i4g_gemm / i4g_gemm_fp32 with a workspace.
 * workspace: 256-byte aligned device memory, ZEROED ONCE before its first use
 * (its first 4096 bytes are arrival counters that every launch returns to
 * zero). A workspace smaller than i4g_gemm_workspace_size reports gets the
 * best schedule that fits (equal splits, or whole tiles; NULL: whole tiles;
 * the decode kernel: its cluster schedule). Launches sharing one workspace
 * must be ordered (one stream); concurrent launches on the same workspace
 * race. A launch that gave up on a device-side wait (i4g_device_status
 * reports I4G_ERR_TIMEOUT) may leave counters non-zero: zero the workspace
 * again before reusing it (i4g_gemm_static_scratch does this itself). */
int i4g_gemm_workspace_size(int M, int N, int K, size_t* bytes);
int i4g_gemm_ws(const void* A, const uint8_t* tiles, const void* scales, void* C,
                int M, int N, int K, int group, void* workspace,
                size_t workspace_bytes, void* stream);
int i4g_gemm_fp32_ws(const void* A, const uint8_t* tiles, const void* scales,
                     float* C, int M, int N, int K, int group, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ---- GEMM without any allocation (no counterpart in the reference) -------- */

/* i4g_gemm_ws for callers that cannot allocate device memory or own a
 * workspace (e.g. a host framework whose memory is fully pooled, or a plugin
 * given only A, B and C): the split-K workspace is a fixed 40 MiB array in
 * static device memory, one per device that loads the library, held until
 * the process exits; nothing is allocated per call.
 * Limit: a tcgen05 plan needs at most (2 * SMs - 2) x 128 KiB + 4 KiB, which
 * fits for up to 160 SMs (B200 has 148); a larger need is rejected with
 * I4G_ERR_SHAPE. A decode shape (M <= 16) whose stream-K workspace would not
 * fit runs the decode kernel's cluster schedule, which needs none.
 * Set-up: the first call on a device loads the scratch and looks up its
 * address with that device current; make that call before any stream
 * capture. The address is kept for the life of the process, so the entry
 * point is not for use across a cudaDeviceReset. Each call clears the
 * scratch's 4 KiB of arrival counters on `stream` before its launch (they
 * must start at zero).
 * Calls on one device share the scratch: calls that overlap in time (e.g. on
 * two streams without ordering between them) race and give wrong results. */
int i4g_gemm_static_scratch(const void* A, const uint8_t* tiles,
                            const void* scales, void* C, int M, int N, int K,
                            int group, void* stream);

/* ---- GEMM with the all-gather fused in (no counterpart in the reference) -- */

/* Column-parallel GEMM that writes its column block straight into every
 * rank's full C: dsts[0..ndst) are the base pointers of ndst row-major
 * [M][ldc] FP16 matrices (this GPU's and, through pointers from
 * i4g_ipc_open, its peers'); the launch computes C[:, col0 : col0 + N] =
 * A x dequant(B) for its slice (tiles, scales: as for i4g_gemm, e.g. a
 * rank's i4g_shard_range slice) and stores it into all of them over NVLink,
 * so no separate all-gather runs. 1 <= ndst <= 8. The caller orders the
 * readers of C after every rank's launch (a cross-rank barrier on the
 * stream). workspace: as for i4g_gemm_ws (may be NULL). */
int i4g_gemm_to_peers(const void* A, const uint8_t* tiles, const void* scales,
                      void* const* dsts, int ndst, int ldc, int col0, int M, int N,
                      int K, int group, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Peer mapping of device memory between processes (CUDA IPC; plain
 * peer-to-peer mappings, no multicast). i4g_ipc_handle: a 64-byte handle of
 * the allocation holding `ptr` and ptr's byte offset in it. i4g_ipc_open: map
 * a peer's handle into this process (*base; add the peer's offset).
 * i4g_ipc_close: unmap. */
int i4g_ipc_handle(const void* ptr, void* handle, size_t* offset);
int i4g_ipc_open(const void* handle, void** base);
int i4g_ipc_close(void* base);

/* ---- column-parallel sharding --------------------------------------------- */

/* Byte offsets of rank `rank`'s slice of a G-way column-parallel split of the
 * tile layout and the scale layout, and its columns [*n0, *n1). N / G must
 * be a multiple of 128. The slices are contiguous, so a rank's weights are
 * (tiles + *tile_offset, scales + *scale_offset) with N_local = *n1 - *n0. */
int i4g_shard_range(int K, int N, int group, int world, int rank,
                    size_t* tile_offset, size_t* scale_offset,
                    int* n0, int* n1);

/* ---- launch plan query (no counterpart in the reference) ------------------ */

/* The kernel and schedule a GEMM of this shape would run on a device with
 * sm_count SMs when given workspace_bytes of workspace (0: none), computed on
 * the host without touching a device, by the same planners the launches use
 * (and under the current i4g_set_decode_schedule choice).
 *   *kernel:   I4G_PLAN_KERNEL_TC256 / _TC128 (tcgen05, 256- or 128-row
 *              activation tiles) or I4G_PLAN_KERNEL_DECODE
 *   *schedule: tcgen05: WHOLE (*param = grid), SPLIT (*param = ways each
 *              tail tile is split), STREAMK (*param = tail shares);
 *              decode: SLICES (*param = grid), CLUSTER (*param = cluster
 *              size), STREAMK (*param = grid)
 *   *bytes:    workspace bytes that schedule uses
 * fp32_out: as i4g_gemm_fp32 (never the decode kernel). */
enum {
  I4G_PLAN_KERNEL_TC256 = 0,
  I4G_PLAN_KERNEL_TC128 = 1,
  I4G_PLAN_KERNEL_DECODE = 2
};
enum {
  I4G_PLAN_WHOLE = 0,
  I4G_PLAN_SPLIT = 1,
  I4G_PLAN_STREAMK = 2,
  I4G_PLAN_CLUSTER = 3,
  I4G_PLAN_SLICES = 4
};
int i4g_plan(int M, int N, int K, int group, int fp32_out, int sm_count,
             size_t workspace_bytes, int* kernel, int* schedule, int* param,
             size_t* bytes);

/* With the I4G_PAIR=1 environment variable (read at the first launch) the
 * tcgen05 kernel runs 256-row tiles on CTA pairs (thread-block clusters of
 * two, one 2-SM tensor-core instruction per pair, both operands from
 * shared memory) when N % 256 == 0, with whole-tile or equal-split tails (no
 * stream-K); by default it runs single CTAs, which measured slightly faster
 * on B200. i4g_plan assumes sm_count / 2 pairs resident at
 * once; launches on a device use the number of pairs that fit on it
 * (clusters are placed within GPCs), which i4g_max_pairs reports for the
 * current device. WHOLE schedules report the grid in CTAs. */
int i4g_max_pairs(int* pairs);

/* ---- kernel registry queries (include/kernels.cuh:6-22, 85-105) ---------- */

/* What the reference's KernelMetadata (kernels.cuh:6-14) and KernelResources
 * (kernels.cuh:16-22) describe, for one instance of this library's kernels:
 * variant I4G_VARIANT_TC with rows = 128 or 256 (activation rows per tile),
 * or I4G_VARIANT_DECODE with rows = 8 (M <= 8) or 16 (M <= 16); group 32, 64
 * or 128. int4gemm.hpp builds kernel_registry() / query_resources() on these.
 * i4g_kernel_config is static (no device); i4g_kernel_resources asks the
 * current device (cudaFuncGetAttributes and the occupancy calculator), as
 * the reference's query_*_resources do. */
typedef struct {
  int rows;               /* activation rows per tile (the reference's BM) */
  int cols;               /* weight columns per tile (BN) */
  int bk;                 /* k per pipeline stage (BK) */
  int mma_m, mma_n;       /* tensor-core instruction: weight columns x rows */
  int stages;             /* activation pipeline stages */
  int threads;            /* threads per CTA */
  int dynamic_smem_bytes; /* dynamic shared memory per CTA */
} i4g_kernel_config_t;

typedef struct {
  int registers_per_thread;
  int static_smem_bytes;
  int max_threads_per_block;
  int active_blocks_per_sm;
} i4g_kernel_resources_t;

int i4g_kernel_config(int variant, int rows, int group, i4g_kernel_config_t* out);
int i4g_kernel_resources(int variant, int rows, int group, i4g_kernel_resources_t* out);

/* ---- decode schedule (no counterpart in the reference) --------------------- */

/* The decode kernel (M <= 16, FP16 C) has three schedules: the slice schedule
 * (each CTA owns a run of 16-column slices over all of K; needs no
 * workspace; possible when N / 16 <= 8 x the SM count), the cluster schedule
 * (each 128-column tile's K split over a thread-block cluster, reduced
 * through distributed shared memory; needs no workspace) and the stream-K
 * schedule of the *_ws entry points (see the workspace section). AUTO (the
 * default, or the I4G_DECODE_SCHEDULE environment variable's "slices" /
 * "cluster" / "streamk" at the first call) takes stream-K when it takes
 * enough work off the busiest SM to pay for its reduction through global
 * memory, else the cluster schedule (the slice schedule measured slower on
 * every shape); the others force one (slices where possible, stream-K only
 * where a large enough workspace is given, the cluster schedule otherwise).
 * Process-wide; affects launches issued after the call. */
enum {
  I4G_DECODE_AUTO = 0,
  I4G_DECODE_CLUSTER = 1,
  I4G_DECODE_STREAMK = 2,
  I4G_DECODE_SLICES = 3
};
int i4g_set_decode_schedule(int schedule);

/* ---- cross-GPU barrier (no counterpart in the reference) ------------------- */

/* Stream-ordered barrier among `world` (<= 8) ranks, one per GPU, after
 * i4g_gemm_to_peers: rank r owns an array of `world` 64-bit flags in device
 * memory (zeroed once, before any rank's first barrier), mapped into every
 * rank (CUDA IPC, i4g_ipc_*). peer_flags[q] is rank q's array as mapped here
 * (peer_flags[rank] is not read). The call stores `epoch` into every peer's
 * flag for this rank (release, system scope) and then waits until every
 * peer has stored at least `epoch` into this rank's array (acquire), so the
 * peer stores of the launches before it on every rank are visible to the
 * launches after it. `epoch` must grow by one per barrier on every rank.
 * The wait gives up after limit_ns (0: the GEMM kernels' 2 s limit) and then
 * records I4G_ERR_TIMEOUT in the device status word (i4g_device_status),
 * e.g. when a peer never arrives; it never faults or hangs the GPU. */
int i4g_peer_barrier(unsigned long long* local_flags,
                     unsigned long long* const* peer_flags, int world, int rank,
                     unsigned long long epoch, unsigned long long limit_ns,
                     void* stream);

/* ---- device status --------------------------------------------------------- */

/* Reads and clears this device's kernel status word (set when a device-side
 * wait hits its limit). Synchronises `stream`. *out = 0 when clean. */
int i4g_device_status(int* out, void* stream);

/* Diagnostic: launches a one-warp kernel whose mbarrier wait can never
 * complete, through the same bounded wait the GEMM kernels use. It gives up
 * after limit_ns (at most 1 s) and records I4G_ERR_TIMEOUT in the device
 * status word, without faulting the GPU. */
int i4g_selftest_wait_timeout(unsigned long long limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* I4G_H */
