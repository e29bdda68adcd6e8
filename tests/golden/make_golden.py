"""Generate the golden fixtures in this directory from the reference itself.

Run from the repository root, where the reference checkout exists:

    make -C oracle all ref REF=/path/to/SM_120__GEMM
    python tests/golden/make_golden.py

Every output array here is produced by ``oracle/_ref/libi4g_ref.so``, i.e. by
the reference's unmodified ``src/reference.cu`` (``quantize_cpu``,
``dequantize_cpu``, ``cpu_gemm_fp32``) and by the reference's own layout
index functions (``include/layout.cuh``). Inputs are seeded; the ``refdist``
cases use the reference harness's own input generator (mt19937_64, uniform
[-0.5, 0.5), ``src/main.cu:75-81``). The files are committed, so the GPU box
(where the reference checkout does not exist) only reads them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def f2h_ref(x):
    R = oracle.ref_lib()
    flat = np.asarray(x, np.float32).reshape(-1)
    return np.array([R.i4r_f2h(float(v)) for v in flat], np.uint16).reshape(np.shape(x))


def normal_weights(K, N, seed, sigma=0.02):
    rng = np.random.default_rng(seed)
    return f2h_ref(rng.standard_normal((K, N)).astype(np.float32) * np.float32(sigma))


def uniform_act(M, K, seed, lo=-1.0, hi=1.0):
    rng = np.random.default_rng(seed)
    return f2h_ref(rng.uniform(lo, hi, (M, K)).astype(np.float32))


def edge_weights(K=128, N=128):
    """Hand-made columns that exercise the quantizer's corner cases."""
    rng = np.random.default_rng(99)
    w = rng.standard_normal((K, N)).astype(np.float32) * 0.02
    w[:, 0] = 0.0                                    # all-zero groups: scale 0
    w[:, 1] = -0.0                                   # negative zeros
    w[:, 2] = 1.0e-7 * np.sign(rng.standard_normal(K))  # scale underflows to 0
    w[:, 3] = 4.0e-7 * np.sign(rng.standard_normal(K))  # subnormal scale
    w[:, 4] = 65504.0 * np.sign(rng.standard_normal(K))  # max-magnitude values
    # exact halfway cases: vmax = 7 gives scale 1, x/s = n + 0.5
    w[:, 5] = np.tile(np.array([7.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5,
                                -3.5, 4.5, -4.5, 5.5, 6.5, -6.5, -7.0, 0.25],
                               np.float32), K // 16)
    w[:, 6] = rng.standard_normal(K).astype(np.float32) * 1.0e-5  # subnormal inputs
    w[::7, 7] = 3.0                                   # sparse column
    w[:, 8] = np.float32(1.0e-3)                      # constant column
    w[:, 9] = -np.float32(2.0)                        # constant negative column
    return f2h_ref(w)


def quant_case(out, name, b, K, N, group):
    packed, scales = oracle.ref_quantize(b, K, N, group)
    deq = oracle.ref_dequantize(packed, scales, K, N, group)
    out[name] = dict(b=b.reshape(K, N), packed=packed, scales=scales, dequant=deq,
                     K=K, N=N, group=group)


def gemm_case(out, name, M, N, K, group, seed_a=1234, seed_b=5678, refdist=False):
    if refdist:
        a = oracle.ref_random_half(M * K, seed_a).reshape(M, K)
        b = oracle.ref_random_half(K * N, seed_b).reshape(K, N)
    else:
        a = uniform_act(M, K, seed_a)
        b = normal_weights(K, N, seed_b)
    packed, scales = oracle.ref_quantize(b, K, N, group)
    deq = oracle.ref_dequantize(packed, scales, K, N, group)
    c32 = oracle.ref_gemm_rows(a, deq, M, N, K)
    c16 = f2h_ref(c32)
    out[name] = dict(a=a, b=b, packed=packed, scales=scales, c32=c32, c16=c16,
                     M=M, N=N, K=K, group=group)


def layout_case(out, name, K, N, group, seed):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, K * N // 2, dtype=np.uint8)
    scales = rng.integers(0, 0x7C00, (K // group, N), dtype=np.uint16)
    out[name] = dict(
        packed=packed, scales=scales,
        tile=oracle.ref_repack_128x32(packed, K, N),
        mma=oracle.ref_repack_mma_128x32(packed, K, N),
        pair=oracle.ref_repack_mma_pair_128x32(packed, K, N),
        scales128=oracle.ref_repack_scales_128(scales, K, N, group),
        K=K, N=N, group=group)


def main():
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/libi4g_ref.so is missing: make -C oracle ref")
    cases = {}
    for g in (32, 64, 128):
        K, N = 128, 256
        quant_case(cases, f"quant_refdist_g{g}",
                   oracle.ref_random_half(K * N, 5678).reshape(K, N), K, N, g)
        quant_case(cases, f"quant_normal_g{g}", normal_weights(256, 128, 5678), 256, 128, g)
    quant_case(cases, "quant_edge_g32", edge_weights(), 128, 128, 32)
    quant_case(cases, "quant_edge_g128", edge_weights(), 128, 128, 128)
    quant_case(cases, "quant_partial_g64", normal_weights(96, 128, 7), 96, 128, 64)
    for g in (32, 64, 128):
        gemm_case(cases, f"gemm_m64_n128_k128_g{g}", 64, 128, 128, g)
        gemm_case(cases, f"gemm_refdist_m64_n256_k256_g{g}", 64, 256, 256, g, refdist=True)
    gemm_case(cases, "gemm_m5_n256_k256_g64", 5, 256, 256, 64)
    gemm_case(cases, "gemm_m1_n128_k512_g128", 1, 128, 512, 128)
    gemm_case(cases, "gemm_m16_n256_k448_g32", 16, 256, 448, 32)
    gemm_case(cases, "gemm_m200_n384_k192_g64", 200, 384, 192, 64)
    layout_case(cases, "layout_k128_n256_g32", 128, 256, 32, 11)
    layout_case(cases, "layout_k64_n384_g64", 64, 384, 64, 12)
    for name, arrays in cases.items():
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {len(cases)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
