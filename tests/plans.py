"""Host schedules mirrored in Python, so tests can say which schedule a
shape runs and how much workspace it asks for.

expected_plan mirrors the tcgen05 kernel's make_plan and cost model
(csrc/gemm_tc.cu); expected_decode_plan mirrors the decode kernel's
choose_cluster and sk_plan, and expected_decode_schedule its pick_schedule
and slice_grid (csrc/gemm_decode.cu); expected_workspace is what
i4g_gemm_workspace_size reports.
"""
import os

import torch

TICKET_BYTES = 4096  # arrival counters at the start of every workspace
TILE_N = 128
DEC_KPS, DEC_BK, DEC_NCOL, DEC_CTAS_PER_SM, DEC_THREADS_C = 4, 64, 128, 2, 256
DEC_SLICE_COLS, DEC_SLICE_MAX = 16, 8


def sm_count():
    return torch.cuda.get_device_properties(0).multi_processor_count


def device_pairs():
    import sm_120__gemm_b200 as m
    return m.max_pairs()


def plan_cg(tile_m, N):
    """CTAs per tile: 2 (a CTA pair) for 256-row tiles of N % 256 == 0 when
    I4G_PAIR=1 is set, else 1."""
    pairs_on = os.environ.get("I4G_PAIR", "0") not in ("", "0")
    return 2 if pairs_on and tile_m == 256 and N % 256 == 0 else 1


def streamk_on():
    """The tcgen05 stream-K tail runs only with I4G_STREAMK=1 (opt-in)."""
    return os.environ.get("I4G_STREAMK", "0") not in ("", "0")


def expected_plan(M, N, K, budget=1 << 62, sms=None, pairs=None):
    """The tcgen05 schedule for this shape: (kind, workspace bytes, tile_m)
    with kind "stream-k", "split<F>" or "whole". Work units are tiles of
    tile_m rows x 128 * cg columns; `pairs` resident CTA pairs (default: the
    current device's when sms is not given, else sms // 2)."""
    if sms is None:
        sms = sm_count()
        pairs = pairs or device_pairs()
    tile_m = 128 if M <= 128 else 256
    cg = plan_cg(tile_m, N)
    units = (pairs or sms // 2) if cg == 2 else sms
    tiles = -(-M // tile_m) * (N // (TILE_N * cg))
    kb = K // 64
    waves, rem = divmod(tiles, units)
    tile_bytes = cg * tile_m * TILE_N * 4
    if rem == 0 or rem * cg * 4 > TICKET_BYTES:
        return "whole", 0, tile_m
    t_tile = kb * (0.45 if tile_m > 128 else 0.5)
    best, plan = (waves + 1) * t_tile, ("whole", 0, tile_m)
    f = min(4, units // rem, kb // 8)
    need = TICKET_BYTES + rem * f * tile_bytes
    if f >= 2 and need <= budget and (waves + 1.0 / f) * t_tile + 12.0 < best:
        best, plan = (waves + 1.0 / f) * t_tile + 12.0, (f"split{f}", need, tile_m)
    run = rem * kb
    chunks = min(units, 3 * rem, run // 8)
    if chunks > rem and cg == 1 and streamk_on():
        most = max((((t + 1) * kb) * chunks - 1) // run - ((t * kb + 1) * chunks - 1) // run + 1
                   for t in range(rem))
        need = TICKET_BYTES + (rem + chunks - 1) * tile_bytes
        t_sk = (waves + rem / chunks) * t_tile + 20.0
        if most <= 4 and run * chunks < 2**31 and need <= budget and t_sk < best:
            plan = ("stream-k", need, tile_m)
    return plan


def decode_cluster(N, K, sms):
    kb, tiles = K // DEC_BK, N // DEC_NCOL
    best, best_score = 1, -1.0
    for cl in range(1, 9):
        if cl > 1 and kb // cl < 2 * DEC_KPS:
            break
        ctas = tiles * cl
        most = -(-ctas // sms)
        if most > DEC_CTAS_PER_SM:
            break
        score = (ctas / sms) / most
        if score >= best_score - 1e-9:
            best_score, best = score, cl
    return best


def expected_decode_plan(M, N, K, sms=None, schedule="auto"):
    """The decode kernel's stream-K plan under i4g_set_decode_schedule
    `schedule`: (preferred, grid, workspace bytes)."""
    sms = sms or sm_count()
    tiles, kb = N // DEC_NCOL, K // DEC_BK
    units = tiles * kb
    grid = min(units, DEC_CTAS_PER_SM * sms)
    slot_bytes = DEC_THREADS_C * (1 if M <= 8 else 2) * 16
    need = TICKET_BYTES + (grid + tiles - 1) * slot_bytes
    cl = decode_cluster(N, K, sms)
    cluster_work = -(-(tiles * cl) // sms) * (-(-kb // cl))
    sk_work = -(-grid // sms) * (-(-units // grid))
    if schedule != "auto":
        return schedule == "streamk", grid, need
    return (cluster_work - sk_work) * 13 > 350, grid, need


def decode_slice_grid(N, sms):
    """CTAs of the slice schedule (one per SM, each owning at most eight
    16-column slices over all of K); 0 where N is too wide for it."""
    slices = N // DEC_SLICE_COLS
    grid = min(slices, sms)
    if grid < 1 or -(-slices // grid) > DEC_SLICE_MAX:
        return 0
    return grid


def expected_decode_schedule(M, N, K, budget, sms=None, schedule="auto"):
    """(schedule, param, workspace bytes) of a decode launch given `budget`
    bytes of workspace, as i4g_plan reports it: the slice schedule where
    forced and possible, else stream-K when preferred and the workspace holds
    it, else the cluster schedule."""
    sms = sms or sm_count()
    grid = decode_slice_grid(N, sms)
    if schedule == "slices" and grid:
        return "slices", grid, 0
    pref, sk_grid, need = expected_decode_plan(M, N, K, sms=sms, schedule=schedule)
    if budget > 0 and pref and budget >= need:
        return "stream-k", sk_grid, need
    return "cluster", decode_cluster(N, K, sms), 0


def expected_workspace(M, N, K, schedule="auto"):
    need = expected_plan(M, N, K)[1]
    if 1 <= M <= 16:
        sched, _, dec_need = expected_decode_schedule(M, N, K, 1 << 62, schedule=schedule)
        if sched == "stream-k":
            need = max(need, dec_need)
    return need
