"""Parity of the CUDA path (through the C ABI) with the reference's CPU path.

Byte and index work (quantize codes and scales, dequantize, every weight
layout) is compared bit-exactly with the golden fixtures made by the
reference itself and with the oracle. The GEMM is compared with the oracle
under the gate stated in tests/parity.py: within 1 FP16 ulp of the
reference's FP32 path, or no further from the exact (binary64) sum than that
path is plus one ulp, or, where FP32 summation noise exceeds the FP16
resolution of the result, within a few noise scales of the exact sum.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden_names, load_golden
from parity import (assert_gemm_parity, fp32_report, gemm_report, make_inputs, oracle_case,
                    reference_rows, u16)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def i4g():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as m
    m.load()
    return m


def dev_u16(arr):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda().view(torch.float16)


def dev_u8(arr):
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.uint8)).cuda()


def gpu_quantize(i4g, b16_u16, K, N, group):
    b = dev_u16(b16_u16.reshape(K, N))
    packed = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty((K + group - 1) // group, N, dtype=torch.float16, device="cuda")
    i4g.launch_quantize(b, packed, scales, K, N, group)
    torch.cuda.synchronize()
    return packed, scales


# ------------------------------------------------------------ byte exactness

@pytest.mark.parametrize("name", golden_names("quant_"))
def test_quantize_bit_exact(i4g, name):
    g = load_golden(name)
    packed, scales = gpu_quantize(i4g, g["b"], g["K"], g["N"], g["group"])
    np.testing.assert_array_equal(u16(scales), g["scales"])
    np.testing.assert_array_equal(packed.cpu().numpy(), g["packed"])


@pytest.mark.parametrize("name", golden_names("quant_"))
def test_dequantize_bit_exact(i4g, name):
    g = load_golden(name)
    K, N = g["K"], g["N"]
    out = torch.empty(K, N, dtype=torch.float16, device="cuda")
    i4g.launch_dequantize(dev_u8(g["packed"]), dev_u16(g["scales"]), out, K, N, g["group"])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(u16(out), g["dequant"])


@pytest.mark.parametrize("name", golden_names("layout_"))
def test_reference_layouts_bit_exact(i4g, name):
    g = load_golden(name)
    K, N, grp = g["K"], g["N"], g["group"]
    packed = dev_u8(g["packed"])
    nbytes = K * N // 2
    tile = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    rsc = torch.empty((K // grp) * N, dtype=torch.float16, device="cuda")
    i4g.launch_repack_128x32(packed, dev_u16(g["scales"]), tile, rsc, K, N, grp)
    mma = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    i4g.launch_repack_mma_128x32(packed, mma, K, N)
    pair = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    i4g.launch_repack_mma_pair_128x32(packed, pair, K, N)
    rsc2 = torch.empty_like(rsc)
    i4g.launch_repack_scales_128(dev_u16(g["scales"]), rsc2, K, N, grp)
    inv = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    i4g.launch_inverse_repack_128x32(tile, inv, K, N)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tile.cpu().numpy(), g["tile"])
    np.testing.assert_array_equal(mma.cpu().numpy(), g["mma"])
    np.testing.assert_array_equal(pair.cpu().numpy(), g["pair"])
    np.testing.assert_array_equal(u16(rsc), g["scales128"])
    np.testing.assert_array_equal(u16(rsc2), g["scales128"])
    np.testing.assert_array_equal(inv.cpu().numpy(), g["packed"])


@pytest.mark.parametrize("K,N", [(64, 128), (192, 384), (4096, 512)])
def test_tile_layout_matches_oracle(i4g, K, N):
    rng = np.random.default_rng(K + N)
    packed_np = rng.integers(0, 256, K * N // 2, dtype=np.uint8)
    tiles = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
    i4g.launch_repack_umma(dev_u8(packed_np), tiles, K, N)
    back = torch.empty_like(tiles)
    i4g.launch_inverse_repack_umma(tiles, back, K, N)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tiles.cpu().numpy(), oracle.repack_umma(packed_np, K, N))
    np.testing.assert_array_equal(back.cpu().numpy(), packed_np)


def test_quantize_large_matches_oracle(i4g):
    K, N = 4096, 4096
    _, w = make_inputs(1, N, K)
    w16 = u16(w)
    for grp in (32, 64, 128):
        packed, scales = gpu_quantize(i4g, w16, K, N, grp)
        p_ref, s_ref = oracle.quantize(w16, K, N, grp)
        np.testing.assert_array_equal(u16(scales), s_ref)
        np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)


# ------------------------------------------------------------------- GEMM

def prepared(i4g, g):
    """GPU quantize + repack of a golden case; returns device buffers."""
    K, N, grp = g["K"], g["N"], g["group"]
    packed, scales = gpu_quantize(i4g, g["b"], K, N, grp)
    np.testing.assert_array_equal(packed.cpu().numpy(), g["packed"])
    lin = i4g.QuantizedLinear.from_packed(packed, scales, K, N, grp)
    return lin


def golden_truth(g):
    """(Expected, deq16) of a golden GEMM case; the oracle's FP32 path is
    checked against the fixture's c32, which the reference's own
    cpu_gemm_fp32 produced."""
    deq = oracle.dequantize(g["packed"], g["scales"], g["K"], g["N"], g["group"])
    exp = reference_rows(g["a"], deq, g["M"], g["N"], g["K"], np.arange(g["M"]))
    np.testing.assert_array_equal(exp.ref32.view(np.uint32), g["c32"].view(np.uint32))
    return exp, deq


@pytest.mark.parametrize("name", golden_names("gemm_"))
def test_gemm_golden(i4g, name):
    g = load_golden(name)
    M, N, K = g["M"], g["N"], g["K"]
    lin = prepared(i4g, g)
    a = dev_u16(g["a"])
    exp, _ = golden_truth(g)
    variants = [i4g.VARIANT_TC] + ([i4g.VARIANT_DECODE] if M <= 16 else [])
    for variant in variants:
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_gemm_variant(a, lin.tiles, lin.scales, c, M, N, K, g["group"], variant)
        torch.cuda.synchronize()
        assert i4g.device_status() == 0
        rep = gemm_report(u16(c), exp)
        print(name, "variant", variant, rep)
        assert_gemm_parity(rep)


@pytest.mark.parametrize("name", ["gemm_m64_n128_k128_g32", "gemm_m200_n384_k192_g64",
                                  "gemm_m5_n256_k256_g64"])
def test_gemm_fp32_output(i4g, name):
    g = load_golden(name)
    M, N, K = g["M"], g["N"], g["K"]
    lin = prepared(i4g, g)
    c = lin(dev_u16(g["a"]), fp32_out=True)
    torch.cuda.synchronize()
    exp, _ = golden_truth(g)
    rep = fp32_report(c.cpu().numpy(), exp)
    print(name, rep)
    assert rep["ok"], rep


def run_case(i4g, M, N, K, grp, rows=None, a_dist="uniform", variant=0, seed=0, device_w=False,
             production=False):
    """One GEMM through the C ABI on seeded inputs, checked on `rows` against
    the oracle. device_w: draw A and W on the GPU (seeded) for shapes whose
    weight is too large to draw quickly on the host; the oracle gets the same
    FP16 values. production: call through QuantizedLinear (launch_final_ws
    with its split-K workspace) instead of i4g_gemm_variant."""
    if device_w:
        ga = torch.Generator(device="cuda").manual_seed(1234 + seed)
        gb = torch.Generator(device="cuda").manual_seed(5678 + seed)
        ad = (torch.rand(M, K, generator=ga, device="cuda") * 2 - 1).half()
        wd = (torch.randn(K, N, generator=gb, device="cuda") * 0.02).half()
        a16, w16 = u16(ad), u16(wd)
    else:
        a, w = make_inputs(M, N, K, seed_a=1234 + seed, seed_b=5678 + seed, a_dist=a_dist)
        ad, wd = a.cuda(), w.cuda()
        a16, w16 = u16(a), u16(w)
    lin = i4g.QuantizedLinear.from_weight(wd, grp)
    del wd
    c = torch.empty(M, N, dtype=torch.float16, device="cuda")
    if production:
        lin(ad, out=c)
    else:
        i4g.launch_gemm_variant(ad, lin.tiles, lin.scales, c, M, N, K, grp, variant)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    exp, _ = oracle_case(a16, w16, M, N, K, grp, rows)
    rep = gemm_report(u16(c)[exp.rows], exp)
    return rep, c


def config_rows(M, seed):
    """Rows to check at a large M: the first and last row blocks, a block
    edge in the middle, and a seeded random sample."""
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([
        np.arange(0, min(M, 4)), np.arange(max(0, M // 2 - 2), min(M, M // 2 + 2)),
        np.arange(max(0, M - 4), M), rng.choice(M, min(M, 12), replace=False)]))


@pytest.mark.parametrize("M,N,K,grp", [
    (8192, 3584, 8192, 128),    # configs[3]: one rank's column slice at G = 8
    (8192, 28672, 8192, 128),   # configs[3]: all of N on one GPU (G = 1)
    (128, 7168, 8192, 64),      # configs[4]: one rank's slice at G = 8, M = 128
    (4096, 7168, 8192, 64),     # configs[4], M = 4096
    (16384, 7168, 8192, 64),    # configs[4], M = 16384
])
def test_gemm_config_shapes(i4g, M, N, K, grp):
    """The prefill and M-sweep configurations, through the production call
    (QuantizedLinear: launch_final_ws with the split-K workspace)."""
    rep, _ = run_case(i4g, M, N, K, grp, rows=config_rows(M, M + N), device_w=True,
                      production=True)
    print("config", M, N, K, grp, rep)
    assert_gemm_parity(rep)


@pytest.mark.parametrize("grp", [32, 64, 128])
def test_gemm_4096_sampled_rows(i4g, grp):
    M = N = K = 4096
    rows = np.unique(np.concatenate([
        np.arange(0, 8), np.arange(185, 200), np.arange(250, 262), np.arange(4088, 4096),
        np.random.default_rng(grp).choice(4096, 96, replace=False)]))
    rep, _ = run_case(i4g, M, N, K, grp, rows=rows)
    print("4096^3 g", grp, rep)
    assert_gemm_parity(rep)


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("K,N", [(4096, 14336), (14336, 4096)])
def test_gemm_decode_shapes(i4g, M, K, N):
    rep, _ = run_case(i4g, M, N, K, 128, a_dist="normal")
    print("decode", M, K, N, rep)
    assert_gemm_parity(rep)


@pytest.mark.parametrize("M,N,K,grp", [(17, 256, 256, 32), (100, 384, 512, 64),
                                       (333, 640, 320, 64), (1000, 256, 1024, 128),
                                       (64, 128, 64, 32), (3, 128, 64, 64)])
def test_gemm_ragged_shapes(i4g, M, N, K, grp):
    rep, _ = run_case(i4g, M, N, K, grp)
    print("ragged", M, N, K, grp, rep)
    assert_gemm_parity(rep)


def test_gemm_deterministic(i4g):
    M = N = K = 1024
    _, c0 = run_case(i4g, M, N, K, 64, rows=np.arange(4))
    outs = []
    a, w = make_inputs(M, N, K)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), 64)
    ad = a.cuda()
    for _ in range(5):
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final(ad, lin.tiles, lin.scales, c, M, N, K, 64)
        outs.append(c)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    assert torch.equal(outs[0].view(torch.int16), c0.view(torch.int16))


def test_wait_timeout_is_reported_not_faulted(i4g):
    assert i4g.device_status() == 0
    i4g.selftest_wait_timeout(2_000_000)  # 2 ms limit on a barrier nobody completes
    assert i4g.device_status() == -8
    assert i4g.device_status() == 0  # reading clears it
    # the context is still usable
    rep, _ = run_case(i4g, 64, 128, 128, 32)
    assert_gemm_parity(rep)


# ------------------------------------------------- one-pass quantize + repack

def special_weights(K, N, seed):
    """N(0, 0.02) weights with the quantiser's edge cases planted: an all-zero
    group, subnormal and tie values, +-65504, a lone large outlier and
    columns of exact rounding ties."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(K, N, generator=g) * 0.02
    w[0:32, 0] = 0.0
    w[0:32, 1] = 2.0 ** -20
    w[:, 2] = torch.tensor([(-1) ** i * (i % 16) * 0.5 for i in range(K)])
    w[5, 3] = 65504.0
    w[6, 3] = -65504.0
    w[7, 4] = 1.0e4
    # exact rounding ties: scale 0.75 with x = +-(k + 0.5) * 0.75, scale 1
    # with x = k / 2
    pattern = [5.25] + [(-1) ** k * (k + 0.5) * 0.75 for k in range(7)]
    w[:, 7] = torch.tensor([pattern[i % len(pattern)] for i in range(K)])
    w[:, 8] = torch.tensor([((i % 29) - 14) * 0.5 for i in range(K)])
    return w.half()


@pytest.mark.parametrize("K,N,grp", [(64, 128, 32), (128, 256, 64), (256, 384, 128),
                                     (4096, 1024, 32), (4096, 1024, 128), (1024, 4096, 64)])
def test_quantize_repack_one_pass_matches_three_step(i4g, K, N, grp):
    w = special_weights(K, N, K + N + grp).cuda()
    tiles = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
    rsc = torch.empty((K // grp) * N, dtype=torch.float16, device="cuda")
    i4g.launch_quantize_repack(w, tiles, rsc, K, N, grp)
    packed, scales = gpu_quantize(i4g, u16(w.cpu()), K, N, grp)
    lin = i4g.QuantizedLinear.from_packed(packed, scales, K, N, grp)
    torch.cuda.synchronize()
    assert torch.equal(tiles, lin.tiles)
    assert torch.equal(rsc.view(torch.int16), lin.scales.view(torch.int16))
    # and against the oracle's codes (through the inverse tile repack)
    pk_np, sc_np = oracle.quantize(u16(w.cpu()), K, N, grp)
    back = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
    i4g.launch_inverse_repack_umma(tiles, back, K, N)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(back.cpu().numpy(), pk_np)


@pytest.mark.parametrize("grp", [32, 64, 128])
def test_reference_gpu_quantizer_departures_from_quantize_cpu(i4g, grp):
    """The reference's own GPU quantizer is built with --use_fast_math, so its
    codes and scales may differ from quantize_cpu (the bit-exact target this
    library meets). Count the differences on the configs' weight distribution
    (4096 x 4096, N(0, 0.02)) and on the edge-case weights; report them."""
    R = oracle.ref_gpu_quantizer()
    if R is None:
        pytest.skip("oracle/_ref/libi4g_refquant.so not built")
    for name, w in (("N(0,0.02)", (torch.randn(4096, 4096, generator=torch.Generator()
                                               .manual_seed(grp)) * 0.02).half()),
                    ("edge cases", special_weights(1024, 1024, grp))):
        K, N = w.shape
        wd = w.cuda()
        packed = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
        scales = torch.empty(K // grp, N, dtype=torch.float16, device="cuda")
        assert R.i4r_gpu_quantize(wd.data_ptr(), packed.data_ptr(), scales.data_ptr(), K, N, grp,
                                  torch.cuda.current_stream().cuda_stream) == 0
        mine_p, mine_s = gpu_quantize(i4g, u16(w), K, N, grp)
        torch.cuda.synchronize()
        ref_p, ref_s = oracle.quantize(u16(w), K, N, grp)
        np.testing.assert_array_equal(mine_p.cpu().numpy(), ref_p)  # this library: exact
        np.testing.assert_array_equal(u16(mine_s), ref_s)
        rp = packed.cpu().numpy()
        codes_lo = (rp & 15) != (ref_p & 15)
        codes_hi = (rp >> 4) != (ref_p >> 4)
        code_diff = int(codes_lo.sum() + codes_hi.sum())
        scale_diff = int((u16(scales).reshape(-1) != ref_s.reshape(-1)).sum())
        print(f"reference GPU quantizer vs quantize_cpu, g{grp}, {name}: {code_diff} of "
              f"{K * N} codes and {scale_diff} of {(K // grp) * N} scales differ")
        assert code_diff <= K * N // 100 and scale_diff <= (K // grp) * N // 100
