"""The host planners, through i4g_plan (no device needed), against their
Python mirrors in tests/plans.py: which kernel, which schedule, its
parameter and its workspace, over a sweep of shapes, two SM counts and three
workspace sizes. The GPU tests rely on the same mirrors to know which
schedule a shape runs."""
import pytest

from plans import (TICKET_BYTES, TILE_N, decode_slice_grid, expected_decode_plan,
                   expected_decode_schedule, expected_plan, plan_cg)

MS = (1, 5, 8, 9, 16, 17, 100, 128, 129, 300, 512, 1000, 1024, 4096, 8192)
NS = (128, 640, 1024, 4096, 7168, 14336, 18944, 19072, 28672)
KS = (64, 448, 1024, 4096, 8192, 14336)
BUDGETS = (0, 20 << 20, 1 << 40)


@pytest.fixture(scope="module")
def i4g():
    import sm_120__gemm_b200 as m
    m.load()
    m.set_decode_schedule("auto")
    return m


@pytest.mark.parametrize("sms", [148, 132])
def test_plan_query_matches_the_mirrors(i4g, sms):
    checked = 0
    for M in MS:
        for N in NS:
            for K in KS:
                for budget in BUDGETS:
                    got = i4g.plan(M, N, K, 64, sms, budget)
                    if M <= 16:
                        want = ("decode",) + expected_decode_schedule(M, N, K, budget, sms=sms)
                    else:
                        kind, need, tile_m = expected_plan(M, N, K, budget=budget, sms=sms)
                        kern = f"tcgen05/{tile_m}"
                        cg = plan_cg(tile_m, N)
                        units = sms // cg
                        tiles = -(-M // tile_m) * (N // (TILE_N * cg))
                        if kind == "whole":
                            want = (kern, "whole", cg * min(tiles, units), 0)
                        elif kind.startswith("split"):
                            want = (kern, "split", int(kind[5:]), need)
                        else:
                            rem = tiles % units
                            chunks = (need - TICKET_BYTES) // (cg * tile_m * TILE_N * 4) - rem + 1
                            want = (kern, "stream-k", chunks, need)
                    have = (got["kernel"], got["schedule"], got["param"], got["workspace_bytes"])
                    assert have == want, (M, N, K, budget, sms, have, want)
                    checked += 1
    assert checked == len(MS) * len(NS) * len(KS) * len(BUDGETS)


def test_forced_decode_schedules(i4g):
    try:
        i4g.set_decode_schedule("streamk")
        _, grid, need = expected_decode_plan(4, 14336, 4096, sms=148, schedule="streamk")
        assert i4g.plan(4, 14336, 4096, 128, 148, need) == {
            "kernel": "decode", "schedule": "stream-k", "param": grid, "workspace_bytes": need}
        # too small a workspace: the cluster schedule
        assert i4g.plan(4, 14336, 4096, 128, 148, need - 1)["schedule"] == "cluster"
        i4g.set_decode_schedule("cluster")
        assert i4g.plan(1, 28672, 8192, 128, 148, 1 << 40)["schedule"] == "cluster"
        assert i4g.plan(1, 4096, 8192, 128, 148, 1 << 40)["schedule"] == "cluster"
        # slices where N / 16 <= 8 x SMs; beyond that the cluster schedule
        # (stream-K is never taken while slices are forced)
        i4g.set_decode_schedule("slices")
        assert i4g.plan(16, 18944, 8192, 64, 148, 0) == {
            "kernel": "decode", "schedule": "slices", "param": 148, "workspace_bytes": 0}
        assert i4g.plan(16, 19072, 8192, 64, 148, 1 << 40)["schedule"] == "cluster"
    finally:
        i4g.set_decode_schedule("auto")


def test_slice_grid():
    assert decode_slice_grid(128, 148) == 8            # one slice per CTA
    assert decode_slice_grid(4096, 148) == 148         # one or two slices each
    assert decode_slice_grid(148 * 8 * 16, 148) == 148  # eight each
    assert decode_slice_grid(148 * 8 * 16 + 128, 148) == 0
    assert decode_slice_grid(14336, 132) == 132


def test_auto_never_takes_slices(i4g):
    for N in (14336, 4096, 7168, 28672):
        assert i4g.plan(4, N, 4096, 128, 148, 1 << 40)["schedule"] in ("stream-k", "cluster")


def test_fp32_output_never_uses_the_decode_kernel(i4g):
    assert i4g.plan(1, 4096, 4096, 128, 148, 0, fp32_out=True)["kernel"] == "tcgen05/128"
