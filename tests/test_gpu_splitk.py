"""Split-K schedules of the tcgen05 kernel (the *_ws entry points).

The tiles of the last, partial wave are shared out along K (equal splits;
stream-K shares over all SMs with I4G_STREAMK=1) and reduced
through a caller-owned FP32 workspace in a fixed order. Results are checked
against the oracle under the same tolerance as the unsplit kernel
(tests/parity.py), are bitwise reproducible, and leave the workspace counters
at zero.
"""
import numpy as np
import pytest
import torch

import oracle
from parity import assert_gemm_parity, fp32_report, gemm_report, make_inputs, oracle_case, u16
from plans import TICKET_BYTES, expected_plan, expected_workspace, streamk_on

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def i4g():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as m
    m.load()
    return m


def fresh_workspace(i4g, M, N, K):
    n = i4g.gemm_workspace_size(M, N, K)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device="cuda"), n


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (512, 1024, 4096), (300, 640, 2048),
                                   (16, 4096, 4096), (4096, 4096, 448), (2048, 9472, 1024),
                                   (1024, 7168, 8192), (2048, 640, 8192)])
def test_workspace_size(i4g, M, N, K):
    kind, _, _ = expected_plan(M, N, K)
    assert i4g.gemm_workspace_size(M, N, K) == expected_workspace(M, N, K), kind


def split_case(i4g, M, N, K, grp, rows=None, fp32_out=False, seed=0):
    a, w = make_inputs(M, N, K, seed_a=99 + seed, seed_b=77 + seed)
    a16, w16 = u16(a), u16(w)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ws, need = fresh_workspace(i4g, M, N, K)
    dt = torch.float32 if fp32_out else torch.float16
    c = torch.empty(M, N, dtype=dt, device="cuda")
    fn = i4g.launch_final_fp32_ws if fp32_out else i4g.launch_final_ws
    fn(a.cuda(), lin.tiles, lin.scales, c, M, N, K, grp, ws)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    assert int(ws[:TICKET_BYTES].count_nonzero()) == 0, "arrival counters not reset"
    exp, _ = oracle_case(a16, w16, M, N, K, grp, rows)
    if fp32_out:
        rep = fp32_report(c.cpu().numpy()[exp.rows], exp)
    else:
        rep = gemm_report(u16(c)[exp.rows], exp)
    return rep, c, (a.cuda(), lin, ws)


def sample_rows(M, seed):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([np.arange(0, 4), np.arange(M // 2 - 2, M // 2 + 2),
                                     np.arange(M - 4, M), rng.choice(M, 8, replace=False)]))


@pytest.mark.parametrize("M,N,K,grp,kind", [(512, 1024, 4096, 128, "split4"),
                                            (128, 7168, 8192, 64, "split2"),
                                            (2048, 640, 8192, 32, "split3"),
                                            (4096, 4864, 4096, 64, "split4")])
def test_split_parity(i4g, M, N, K, grp, kind):
    assert expected_plan(M, N, K)[0] == kind, "shape chosen to exercise this schedule"
    rep, _, _ = split_case(i4g, M, N, K, grp, rows=sample_rows(M, M + N))
    print(kind, M, N, K, grp, rep)
    assert_gemm_parity(rep)


@pytest.mark.parametrize("grp", [32, 128])
def test_split_4096_sampled_rows(i4g, grp):
    M = N = K = 4096
    # rows in the first whole-tile waves and in the split last wave (the
    # last tiles in schedule order are the highest row blocks of the last
    # column groups)
    rows = np.concatenate([np.arange(0, 8), np.arange(250, 262), np.arange(3830, 3842),
                           np.arange(4088, 4096)])
    rep, _, _ = split_case(i4g, M, N, K, grp, rows=rows)
    print("split 4096^3 g", grp, rep)
    assert_gemm_parity(rep)


@pytest.mark.parametrize("M,N,K,grp", [(512, 1024, 4096, 64), (2048, 640, 8192, 128)])
def test_split_fp32_output(i4g, M, N, K, grp):
    assert expected_plan(M, N, K)[0] != "whole"
    rep, _, _ = split_case(i4g, M, N, K, grp, fp32_out=True, rows=sample_rows(M, 7))
    print("split fp32", M, N, K, grp, rep)
    assert rep["ok"], rep


def test_split_reuse_is_bitwise_reproducible(i4g):
    """One workspace across launches of different shapes: every launch
    returns the counters to zero, so repeated results are bitwise equal."""
    _, c_a, (a_a, lin_a, _) = split_case(i4g, 512, 1024, 4096, 128, rows=np.arange(2))
    _, c_b, (a_b, lin_b, _) = split_case(i4g, 1024, 7168, 8192, 64, rows=np.arange(2), seed=1)
    need = max(i4g.gemm_workspace_size(512, 1024, 4096), i4g.gemm_workspace_size(1024, 7168, 8192))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        for (a, lin, ref, M) in ((a_a, lin_a, c_a, 512), (a_b, lin_b, c_b, 1024)):
            c = torch.empty_like(ref)
            i4g.launch_final_ws(a, lin.tiles, lin.scales, c, M, lin.N, lin.K, lin.group, ws)
            torch.cuda.synchronize()
            assert torch.equal(c.view(torch.int16), ref.view(torch.int16))
    assert i4g.device_status() == 0
    assert int(ws[:TICKET_BYTES].count_nonzero()) == 0


def test_small_workspace_runs_unsplit(i4g):
    """A workspace smaller than needed (or none) selects the unsplit schedule,
    bitwise equal to i4g_gemm."""
    M, N, K, grp = 512, 1024, 4096, 128
    a, w = make_inputs(M, N, K)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ad = a.cuda()
    c0 = torch.empty(M, N, dtype=torch.float16, device="cuda")
    i4g.launch_final(ad, lin.tiles, lin.scales, c0, M, N, K, grp)
    small = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    for ws in (None, small):
        c = torch.empty_like(c0)
        i4g.launch_final_ws(ad, lin.tiles, lin.scales, c, M, N, K, grp, ws)
        torch.cuda.synchronize()
        assert torch.equal(c.view(torch.int16), c0.view(torch.int16))


def test_misaligned_workspace_rejected(i4g):
    M, N, K = 512, 1024, 4096
    ws = torch.zeros(i4g.gemm_workspace_size(M, N, K) + 512, dtype=torch.uint8, device="cuda")
    a = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    tiles = torch.zeros(K * N // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(K // 128 * N, dtype=torch.float16, device="cuda")
    c = torch.empty(M, N, dtype=torch.float16, device="cuda")
    with pytest.raises(i4g.I4GError) as e:
        i4g.launch_final_ws(a, tiles, scales, c, M, N, K, 128, ws[16:])
    assert e.value.status == -4


@pytest.mark.parametrize("M,N,K,grp", [(1024, 7168, 8192, 64), (2048, 3968, 12288, 32),
                                       (1024, 3200, 12288, 128)])
def test_stream_k_tail_parity(i4g, M, N, K, grp):
    """The shapes the stream-K tail serves when it is enabled (I4G_STREAMK=1:
    shares over all SMs after whole waves, or as the only wave, up to three
    or four partial tiles per output tile); by default they run equal splits
    or whole tiles. Either way: parity on sampled rows covering the tail
    tiles' row blocks, and a second launch on the same workspace equal bit
    for bit."""
    kind = expected_plan(M, N, K)[0]
    assert (kind == "stream-k") == streamk_on(), kind
    rep, c, (a, lin, ws) = split_case(i4g, M, N, K, grp, rows=sample_rows(M, K))
    print(kind, M, N, K, grp, rep)
    assert_gemm_parity(rep)
    c2 = torch.empty_like(c)
    i4g.launch_final_ws(a, lin.tiles, lin.scales, c2, M, N, K, grp, ws)
    torch.cuda.synchronize()
    assert torch.equal(c.view(torch.int16), c2.view(torch.int16))


def test_smaller_workspace_falls_back_to_equal_splits(i4g):
    """4096^3 with a 20 MiB workspace: the equal two-way split; it must match
    the oracle."""
    M = N = K = 4096
    kind, need, _ = expected_plan(M, N, K, budget=20 << 20)
    assert kind == "split2"
    a, w = make_inputs(M, N, K, seed_a=5, seed_b=6)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), 128)
    ws = torch.zeros(20 << 20, dtype=torch.uint8, device="cuda")
    c = torch.empty(M, N, dtype=torch.float16, device="cuda")
    i4g.launch_final_ws(a.cuda(), lin.tiles, lin.scales, c, M, N, K, 128, ws)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    assert int(ws[:TICKET_BYTES].count_nonzero()) == 0
    exp, _ = oracle_case(u16(a), u16(w), M, N, K, 128, np.array([0, 1, 2047, 3000, 4095]))
    assert_gemm_parity(gemm_report(u16(c)[exp.rows], exp))
