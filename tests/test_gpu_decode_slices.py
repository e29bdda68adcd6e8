"""Slice schedule of the decode kernel (M <= 16, FP16 C, no workspace).

Each CTA owns a contiguous run of 16-column slices over all of K, fetched
with 5-D TMA boxes out of the tile layout (a run may straddle two 128-column
tiles), and sums the four 64-k block parts of each slice in order in shared
memory. Checked against the oracle under the gate of tests/parity.py, over
runs of one to eight slices, runs that straddle tiles, a K that ends inside a
ring stage, every group size and both row-block heights; bitwise
reproducible; the multi-copy output descriptor; and close to the cluster
schedule's result.
"""
import pytest
import torch

import oracle
from parity import assert_gemm_parity, gemm_report, make_inputs, oracle_case, u16
from plans import decode_slice_grid, expected_decode_schedule

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def i4g():
    """The library with the decode schedule forced to slices for this module
    (back to the automatic choice afterwards)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as m
    m.load()
    m.set_decode_schedule("slices")
    yield m
    m.set_decode_schedule("auto")


def slice_case(i4g, M, N, K, grp, seed=0):
    a, w = make_inputs(M, N, K, seed_a=701 + seed, seed_b=709 + seed, a_dist="normal")
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    i4g.launch_final(a.cuda(), lin.tiles, lin.scales, c, M, N, K, grp)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    exp, _ = oracle_case(u16(a), u16(w), M, N, K, grp)
    return gemm_report(u16(c), exp), c, (a, lin, exp)


@pytest.mark.parametrize("M,N,K,grp", [
    (1, 14336, 4096, 128), (16, 14336, 4096, 128),   # gate/up MLP: 6-7 slices, straddling tiles
    (4, 4096, 14336, 128), (8, 4096, 14336, 64),     # down MLP: 1-2 slices
    (16, 7168, 8192, 64), (1, 7168, 8192, 32),       # 3-4 slices
    (9, 18944, 1024, 32), (2, 18944, 2048, 64),      # eight slices on every CTA
    (13, 128, 4096, 64), (3, 256, 1024, 128),        # fewer slices than SMs
    (5, 2048, 320, 32), (7, 1664, 384, 128),         # K ends inside a ring stage
    (16, 3072, 64, 64), (1, 640, 192, 64),           # one or three 64-k blocks
])
def test_decode_slices_parity(i4g, M, N, K, grp):
    sched = expected_decode_schedule(M, N, K, 0, schedule="slices")
    assert sched[0] == "slices", sched
    assert i4g.plan(M, N, K, grp, torch.cuda.get_device_properties(0).multi_processor_count,
                    0)["schedule"] == "slices"
    rep, _, _ = slice_case(i4g, M, N, K, grp)
    print("decode slices", M, N, K, grp, "grid", sched[1], rep)
    assert_gemm_parity(rep)


def test_decode_slices_deterministic_and_close_to_cluster(i4g):
    M, N, K, grp = 16, 14336, 4096, 128
    rep0, c0, (a, lin, exp) = slice_case(i4g, M, N, K, grp, seed=3)
    assert_gemm_parity(rep0)
    ad = a.cuda()
    outs = []
    for _ in range(4):
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final(ad, lin.tiles, lin.scales, c, M, N, K, grp)
        outs.append(c)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o.view(torch.int16), c0.view(torch.int16))
    try:
        i4g.set_decode_schedule("cluster")
        cl = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final(ad, lin.tiles, lin.scales, cl, M, N, K, grp)
        torch.cuda.synchronize()
    finally:
        i4g.set_decode_schedule("slices")
    rep1 = gemm_report(u16(cl), exp)
    ulp = oracle.ulp_distance(u16(cl), u16(c0))
    print("slices vs cluster: max ulp", int(ulp.max()), "identical", float((ulp == 0).mean()))
    assert_gemm_parity(rep1)
    assert float((ulp <= 1).mean()) > 0.99


@pytest.mark.parametrize("M,N,K,grp", [(4, 4096, 4096, 128), (12, 1024, 1024, 64),
                                       (16, 14336, 1024, 32)])
def test_slices_output_copies_with_stride_and_offset(i4g, M, N, K, grp):
    """i4g_gemm_to_peers with two local destinations under the slice
    schedule: each gets the plain GEMM's C bit for bit in columns
    [col0, col0 + N) of rows of ldc, the other columns untouched."""
    assert decode_slice_grid(N, torch.cuda.get_device_properties(0).multi_processor_count)
    a, w = make_inputs(M, N, K, seed_a=51, seed_b=53)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ad = a.cuda()
    ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
    i4g.launch_final(ad, lin.tiles, lin.scales, ref, M, N, K, grp)
    ldc, col0 = 3 * N, N
    dsts = [torch.full((M, ldc), -7.0, dtype=torch.float16, device="cuda") for _ in range(2)]
    i4g.launch_final_to_peers(ad, lin.tiles, lin.scales, [d.data_ptr() for d in dsts], ldc, col0,
                              M, N, K, grp, None)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    for d in dsts:
        assert torch.equal(d[:, col0:col0 + N].view(torch.int16), ref.view(torch.int16))
        assert bool((d[:, :col0] == -7.0).all()) and bool((d[:, col0 + N:] == -7.0).all())


def test_weight_buffers_alternate(i4g):
    """The per-thread cache of weight tensor maps: alternating between more
    weight buffers than it holds gives the same results as fresh calls."""
    M, K, grp = 4, 1024, 64
    cases = []
    for i, N in enumerate((1024, 2048, 1536, 4096, 640, 3072)):
        a, w = make_inputs(M, N, K, seed_a=900 + i, seed_b=950 + i)
        lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final(a.cuda(), lin.tiles, lin.scales, c, M, N, K, grp)
        cases.append((a.cuda(), lin, N, c))
    torch.cuda.synchronize()
    for _ in range(2):
        for ad, lin, N, c in reversed(cases):
            again = torch.empty(M, N, dtype=torch.float16, device="cuda")
            i4g.launch_final(ad, lin.tiles, lin.scales, again, M, N, K, grp)
            torch.cuda.synchronize()
            assert torch.equal(again.view(torch.int16), c.view(torch.int16))
