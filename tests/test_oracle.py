"""The CPU oracle (oracle/oracle.c) against the reference's own outputs.

The golden fixtures were produced by the reference's unmodified
src/reference.cu (quantize_cpu, dequantize_cpu, cpu_gemm_fp32) and by its
layout index functions (include/layout.cuh); see tests/golden/make_golden.py.
Everything here is bit-exact.
"""
import numpy as np
import pytest

from conftest import golden_names, load_golden


@pytest.mark.parametrize("name", golden_names("quant_"))
def test_quantize_matches_reference(oracle_mod, name):
    g = load_golden(name)
    packed, scales = oracle_mod.quantize(g["b"], g["K"], g["N"], g["group"])
    np.testing.assert_array_equal(scales, g["scales"])
    np.testing.assert_array_equal(packed, g["packed"])


@pytest.mark.parametrize("name", golden_names("quant_"))
def test_dequantize_matches_reference(oracle_mod, name):
    g = load_golden(name)
    deq = oracle_mod.dequantize(g["packed"], g["scales"], g["K"], g["N"], g["group"])
    np.testing.assert_array_equal(deq, g["dequant"])


@pytest.mark.parametrize("name", golden_names("gemm_"))
def test_gemm_matches_reference_bitwise(oracle_mod, name):
    g = load_golden(name)
    M, N, K, grp = g["M"], g["N"], g["K"], g["group"]
    packed, scales = oracle_mod.quantize(g["b"], K, N, grp)
    np.testing.assert_array_equal(packed, g["packed"])
    deq = oracle_mod.dequantize(packed, scales, K, N, grp)
    c32 = oracle_mod.gemm_rows(g["a"], deq, M, N, K)
    np.testing.assert_array_equal(c32.view(np.uint32), g["c32"].view(np.uint32))
    np.testing.assert_array_equal(oracle_mod.f2h(c32), g["c16"])


@pytest.mark.parametrize("name", golden_names("layout_"))
def test_reference_layouts(oracle_mod, name):
    g = load_golden(name)
    K, N, grp = g["K"], g["N"], g["group"]
    np.testing.assert_array_equal(oracle_mod.repack_128x32(g["packed"], K, N), g["tile"])
    np.testing.assert_array_equal(oracle_mod.repack_mma_128x32(g["packed"], K, N), g["mma"])
    np.testing.assert_array_equal(oracle_mod.repack_mma_pair_128x32(g["packed"], K, N), g["pair"])
    np.testing.assert_array_equal(
        oracle_mod.repack_scales_128(g["scales"], K, N, grp), g["scales128"])
    np.testing.assert_array_equal(
        oracle_mod.inverse_repack_128x32(g["tile"], K, N), g["packed"])


def test_umma_layout_is_a_permutation(oracle_mod):
    K, N = 192, 384
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, K * N // 2, dtype=np.uint8)
    tiles = oracle_mod.repack_umma(packed, K, N)
    np.testing.assert_array_equal(oracle_mod.inverse_repack_umma(tiles, K, N), packed)
    idx = {oracle_mod.lib().i4o_umma_nibble_index(k, n, K)
           for k in range(0, K, 5) for n in range(0, N, 3)}
    assert len(idx) == len(range(0, K, 5)) * len(range(0, N, 3))


def test_sign_extend(oracle_mod):
    L = oracle_mod.lib()
    assert [L.i4o_sign_extend(x) for x in range(16)] == list(range(8)) + list(range(-8, 0))


def test_half_conversions_match_cuda_host(oracle_mod):
    if not oracle_mod.ref_available():
        pytest.skip("reference checker not built here")
    R = oracle_mod.ref_lib()
    L = oracle_mod.lib()
    for h in range(0, 65536, 7):
        a, b = L.i4o_h2f(h), R.i4r_h2f(h)
        assert a == b or (a != a and b != b)
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32)
    xs = bits.view(np.float32)
    xs = xs[~np.isnan(xs)]
    mine = oracle_mod.f2h(xs)
    ref = np.array([R.i4r_f2h(float(x)) for x in xs], np.uint16)
    np.testing.assert_array_equal(mine, ref)


def test_quantize_live_against_reference(oracle_mod):
    """Fresh seeded inputs (beyond the fixtures) where the reference exists."""
    if not oracle_mod.ref_available():
        pytest.skip("reference checker not built here")
    rng = np.random.default_rng(2024)
    for K, N, g in ((256, 256, 32), (192, 128, 64), (512, 128, 128)):
        b = oracle_mod.f2h(rng.standard_normal((K, N)).astype(np.float32) * 0.02)
        p0, s0 = oracle_mod.quantize(b, K, N, g)
        p1, s1 = oracle_mod.ref_quantize(b, K, N, g)
        np.testing.assert_array_equal(s0, s1)
        np.testing.assert_array_equal(p0, p1)


def test_compare_half_matches_reference_formula(oracle_mod):
    g = load_golden("gemm_m64_n128_k128_g64")
    ref = g["c16"]
    got = ref.copy()
    got[0, :5] ^= 1
    m = oracle_mod.compare_half(got, ref)
    assert m.max_abs > 0 and m.relative_l2 < 1e-2
    assert oracle_mod.compare_half(ref, ref).max_abs == 0


@pytest.mark.parametrize("name", golden_names("gemm_"))
def test_parity_gate_on_the_reference_path(oracle_mod, name):
    """The GEMM parity gate, applied to the reference's own output (the
    fixture's c16, made by the reference's cpu_gemm_fp32): it passes with
    every output at 0 ulps, and the exact-sum anchor puts the reference's
    path within a few ulps of the exact answer on these cases. A planted
    3-ulp error in the largest output fails the gate."""
    from parity import gemm_report, reference_rows
    g = load_golden(name)
    M, N, K, grp = g["M"], g["N"], g["K"], g["group"]
    deq = oracle_mod.dequantize(g["packed"], g["scales"], K, N, grp)
    exp = reference_rows(g["a"], deq, M, N, K, np.arange(M), threads=2)
    np.testing.assert_array_equal(exp.ref32.view(np.uint32), g["c32"].view(np.uint32))
    rep = gemm_report(g["c16"], exp)
    assert rep["ok"] and rep["max_ulp"] == 0, rep
    assert rep["max_ulp_vs_exact_ref"] <= 8, rep
    planted = g["c16"].copy()
    idx = np.unravel_index(np.argmax(np.abs(oracle_mod.h2f(planted))), planted.shape)
    planted[idx] = planted[idx] + 3  # 3 ulps away (same sign, far from zero)
    bad = gemm_report(planted, exp)
    assert not bad["ok"] and bad["bad"] == 1, bad
