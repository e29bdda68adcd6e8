"""Shared helpers for the GPU parity tests (CPU-side checking only).

Tolerance of the GEMM parity: each FP16 output is
within 1 FP16 ulp of the reference's CPU path (dequantize_cpu + the
sequential-k FP32 cpu_gemm_fp32, rounded to FP16), except where the two FP32
summation orders themselves may differ by more than that: there the bound is
1 ulp + gamma * sum_k |a_k * b_k| with gamma = 2 * K * 2^-24 (the standard
worst-case bound for two different FP32 summation orders of K terms).
"""
from __future__ import annotations

import numpy as np
import torch

import oracle


def make_inputs(M, N, K, seed_a=1234, seed_b=5678, a_dist="uniform", w_sigma=0.02):
    """Seeded synthetic inputs with the configs' distributions (torch CPU RNG):
    A fp16 uniform[-1, 1] (or N(0, 1) for decode), W fp32 N(0, sigma) -> fp16."""
    ga = torch.Generator().manual_seed(seed_a)
    gb = torch.Generator().manual_seed(seed_b)
    if a_dist == "normal":
        a = torch.randn(M, K, generator=ga)
    else:
        a = torch.rand(M, K, generator=ga) * 2 - 1
    w = torch.randn(K, N, generator=gb) * w_sigma
    return a.half(), w.half()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def fp16_spacing(x: np.ndarray) -> np.ndarray:
    ax = np.abs(x.astype(np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0**-24)))
    return np.where(ax < 2.0**-14, 2.0**-24, 2.0 ** (e - 10))


def gemm_report(got16: np.ndarray, ref32: np.ndarray, abs32: np.ndarray, K: int) -> dict:
    """Check FP16 GEMM output against the FP32 oracle; returns stats and 'ok'."""
    ref16 = oracle.f2h(ref32)
    ulp = oracle.ulp_distance(got16, ref16)
    got = oracle.h2f(got16).astype(np.float64)
    ref = oracle.h2f(ref16).astype(np.float64)
    gamma = 2.0 * K * 2.0**-24
    bound = fp16_spacing(ref32) + gamma * abs32.astype(np.float64)
    ok = (ulp <= 1) | (np.abs(got - ref) <= bound)
    hist = {"0": int((ulp == 0).sum()), "1": int((ulp == 1).sum()),
            "2": int((ulp == 2).sum()), ">2": int((ulp > 2).sum())}
    m = oracle.compare_half(got16, ref16)
    return {"ok": bool(ok.all()), "bad": int((~ok).sum()), "ulp_hist": hist,
            "max_ulp": int(ulp.max()), "max_abs": m.max_abs, "rel_l2": m.relative_l2}


def fp32_report(got32: np.ndarray, ref32: np.ndarray, abs32: np.ndarray, K: int) -> dict:
    gamma = 2.0 * K * 2.0**-24
    diff = np.abs(got32.astype(np.float64) - ref32.astype(np.float64))
    bound = gamma * abs32.astype(np.float64) + 1e-30
    return {"ok": bool((diff <= bound).all()), "max_abs": float(diff.max()),
            "max_rel_to_bound": float((diff / bound).max())}


def fp64_attribution(a16_rows: np.ndarray, deq16: np.ndarray, got16: np.ndarray,
                     ref32: np.ndarray) -> dict:
    """Attribute the residual against an FP64 oracle: the dequantized FP16
    products (exact in FP64) summed in FP64 and rounded once to FP16 give the
    best FP16 answer for each output; this output and the reference's FP32
    path (rounded to FP16) are both measured from it in ulps. Where the two
    differ by more than an ulp, this says which one the summation order put
    further from the exact product."""
    a = oracle.h2f(a16_rows).astype(np.float64)
    w = oracle.h2f(deq16).astype(np.float64)
    truth16 = (a @ w).astype(np.float16).view(np.uint16)
    ours = oracle.ulp_distance(got16, truth16)
    ref = oracle.ulp_distance(oracle.f2h(ref32), truth16)
    return {"fp64_max_ulp_ours": int(ours.max()), "fp64_max_ulp_ref": int(ref.max()),
            "fp64_outputs_closer_ours": int((ours < ref).sum()),
            "fp64_outputs_closer_ref": int((ref < ours).sum())}
