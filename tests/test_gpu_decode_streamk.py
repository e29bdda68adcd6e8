"""Stream-K schedule of the decode kernel (M <= 16, FP16 C, with a workspace).

A persistent grid of two CTAs per SM splits the (column tile, 64-k block)
units into equal runs; split tiles are reduced through the workspace by the
last CTA to arrive, in run order. Checked against the oracle under the
tolerance of tests/parity.py, bitwise reproducible, workspace counters left
at zero, and the multi-copy output descriptor (several destinations, a row
stride and a column offset) on one GPU for both kernels.
"""
import numpy as np
import pytest
import torch

import oracle
from parity import assert_gemm_parity, gemm_report, make_inputs, oracle_case, u16
from plans import TICKET_BYTES, expected_decode_plan

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def i4g():
    """The library with the decode schedule forced to stream-K for this
    module (back to the automatic choice afterwards)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as m
    m.load()
    m.set_decode_schedule("streamk")
    yield m
    m.set_decode_schedule("auto")


def sk_case(i4g, M, N, K, grp, seed=0, a_dist="normal"):
    a, w = make_inputs(M, N, K, seed_a=311 + seed, seed_b=313 + seed, a_dist=a_dist)
    a16, w16 = u16(a), u16(w)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    need = i4g.gemm_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    i4g.launch_final_ws(a.cuda(), lin.tiles, lin.scales, c, M, N, K, grp, ws)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    assert int(ws[:TICKET_BYTES].count_nonzero()) == 0, "arrival counters not reset"
    exp, _ = oracle_case(a16, w16, M, N, K, grp)
    return gemm_report(u16(c), exp), c, (a, lin, ws, need, exp)


@pytest.mark.parametrize("M,N,K,grp", [
    (1, 14336, 4096, 128), (16, 14336, 4096, 128),    # decode MLP shapes, 4 parts per tile
    (4, 4096, 14336, 128), (8, 4096, 14336, 64),      # 10 parts per tile
    (9, 4096, 4096, 32), (13, 1024, 4096, 64),        # ragged M, a row block of 16
    (3, 256, 1024, 128), (1, 28672, 8192, 128),       # tiny N; 224 tiles, 1-3 parts
    (5, 640, 2048, 32),                               # odd tile count
])
def test_decode_streamk_parity(i4g, M, N, K, grp):
    pref, grid, need = expected_decode_plan(M, N, K, schedule="streamk")
    assert pref
    assert i4g.gemm_workspace_size(M, N, K) >= need
    rep, _, _ = sk_case(i4g, M, N, K, grp)
    print("decode stream-k", M, N, K, grp, "grid", grid, rep)
    assert_gemm_parity(rep)


def test_decode_streamk_deterministic_and_close_to_cluster(i4g):
    M, N, K, grp = 4, 14336, 4096, 128
    rep0, c0, (a, lin, ws, _, exp) = sk_case(i4g, M, N, K, grp)
    assert_gemm_parity(rep0)
    ad = a.cuda()
    outs = []
    for _ in range(4):
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final_ws(ad, lin.tiles, lin.scales, c, M, N, K, grp, ws)
        outs.append(c)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o.view(torch.int16), c0.view(torch.int16))
    # the cluster schedule (no workspace) sums the same products in another
    # order; both meet the parity gate (the FP32 order changes an FP16
    # output by more than an ulp only near zero)
    cl = torch.empty(M, N, dtype=torch.float16, device="cuda")
    i4g.launch_final(ad, lin.tiles, lin.scales, cl, M, N, K, grp)
    torch.cuda.synchronize()
    rep1 = gemm_report(u16(cl), exp)
    ulp = oracle.ulp_distance(u16(cl), u16(c0))
    print("stream-k vs cluster: max ulp", int(ulp.max()), "identical",
          float((ulp == 0).mean()), rep1)
    assert_gemm_parity(rep1)
    assert float((ulp <= 1).mean()) > 0.99


@pytest.mark.parametrize("M,N,K,grp", [(4, 4096, 4096, 128),      # decode, stream-K
                                       (12, 1024, 1024, 64),      # decode, row block of 16
                                       (300, 640, 2048, 32),      # tcgen05, split tail
                                       (1000, 1024, 1024, 128)])  # tcgen05, 32 tiles split
def test_output_copies_with_stride_and_offset(i4g, M, N, K, grp):
    """i4g_gemm_to_peers with two local destinations: each gets the plain
    GEMM's C bit for bit in columns [col0, col0 + N) of rows of ldc, and the
    other columns stay untouched."""
    a, w = make_inputs(M, N, K, seed_a=41, seed_b=43)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ad = a.cuda()
    ws = torch.zeros(max(i4g.gemm_workspace_size(M, N, K), 256), dtype=torch.uint8, device="cuda")
    ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
    i4g.launch_final_ws(ad, lin.tiles, lin.scales, ref, M, N, K, grp, ws)
    ldc, col0 = 3 * N, N
    dsts = [torch.full((M, ldc), -7.0, dtype=torch.float16, device="cuda") for _ in range(2)]
    i4g.launch_final_to_peers(ad, lin.tiles, lin.scales, [d.data_ptr() for d in dsts], ldc, col0,
                              M, N, K, grp, ws)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    assert int(ws[:TICKET_BYTES].count_nonzero()) == 0
    for d in dsts:
        assert torch.equal(d[:, col0:col0 + N].view(torch.int16), ref.view(torch.int16))
        assert bool((d[:, :col0] == -7.0).all()) and bool((d[:, col0 + N:] == -7.0).all())


@pytest.mark.parametrize("M,N,K", [(1, 14336, 4096), (16, 4096, 14336), (1, 28672, 8192),
                                   (4, 57344, 8192), (8, 7168, 8192)])
def test_automatic_schedule_choice(i4g, M, N, K):
    """Under "auto" the workspace query asks for the stream-K bytes exactly
    when the slice schedule is not possible and the model prefers stream-K
    (large N: many column tiles left on one CTA per SM by the cluster
    schedule); "slices" and "cluster" never ask for them."""
    from plans import expected_decode_schedule, expected_plan, expected_workspace
    try:
        for schedule in ("auto", "slices", "cluster", "streamk"):
            i4g.set_decode_schedule(schedule)
            sched, _, need = expected_decode_schedule(M, N, K, 1 << 62, schedule=schedule)
            got = i4g.gemm_workspace_size(M, N, K)
            print(schedule, M, N, K, sched, got)
            assert got == expected_workspace(M, N, K, schedule=schedule)
            assert got == (max(need, expected_plan(M, N, K)[1]) if sched == "stream-k"
                           else expected_plan(M, N, K)[1])
    finally:
        i4g.set_decode_schedule("streamk")
