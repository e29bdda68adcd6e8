"""The reference's own final GPU GEMM (kernels/gemm_final.cu:5-13 over
kernels/gemm_v17_instruction.cu, built unmodified for sm_100a by
oracle/Makefile) on B200, as a same-box context for this library's kernels:
fed the reference's layouts (made by this library's byte-exact repacks), its
output must pass the reference's own correctness gate against the CPU path
(src/main.cu:257-261: relative L2 < 0.02 and max |err| < 2); the report also
gives this library's parity statistics for both kernels on the same inputs.

The reference kernel's mbarrier waits are unbounded, so every case runs in
a child process that is stopped after a time limit."""
import json
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _worker(q, M, N, K, grp):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    import oracle
    import sm_120__gemm_b200 as i4g
    from parity import gemm_report, make_inputs, oracle_case, u16

    R = oracle.ref_final_kernel()
    a, w = make_inputs(M, N, K, seed_a=401, seed_b=403)
    ad, wd = a.cuda(), w.cuda()
    packed = torch.empty(K * N // 2, dtype=torch.uint8, device="cuda")
    scales = torch.empty(K // grp, N, dtype=torch.float16, device="cuda")
    i4g.launch_quantize(wd, packed, scales, K, N, grp)
    b_ref = torch.empty_like(packed)
    if grp == 64:
        i4g.launch_repack_mma_128x32(packed, b_ref, K, N)
    else:
        i4g.launch_repack_mma_pair_128x32(packed, b_ref, K, N)
    s_ref = torch.empty_like(scales)
    i4g.launch_repack_scales_128(scales, s_ref, K, N, grp)
    c_ref = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    st = R.i4r_launch_final(ad.data_ptr(), b_ref.data_ptr(), s_ref.data_ptr(), c_ref.data_ptr(),
                            M, N, K, grp, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    lin = i4g.QuantizedLinear.from_weight(wd, grp)
    c_ours = lin(ad)
    torch.cuda.synchronize()
    rng = np.random.default_rng(M + N + K + grp)
    rows = np.unique(np.concatenate([np.arange(min(M, 4)), rng.choice(M, min(M, 12), False)]))
    exp, _ = oracle_case(u16(a), u16(w), M, N, K, grp, rows)
    ref16 = oracle.f2h(exp.ref32)
    got_ref = u16(c_ref)[rows]
    m = oracle.compare_half(got_ref, ref16)
    q.put(json.dumps({"status": st, "rel_l2": float(m.relative_l2), "max_abs": float(m.max_abs),
                      "reference_kernel": gemm_report(got_ref, exp),
                      "this_library": gemm_report(u16(c_ours)[rows], exp)}, default=float))


@pytest.mark.parametrize("M,N,K,grp", [(256, 256, 256, 32), (256, 256, 256, 64),
                                       (256, 256, 256, 128), (4096, 4096, 4096, 128)])
def test_reference_final_kernel_passes_its_own_gate(M, N, K, grp):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    sys.path.insert(0, ROOT)
    import oracle
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libi4g_reffinal.so")):
        pytest.skip("oracle/_ref/libi4g_reffinal.so not built (needs the reference checkout)")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_worker, args=(q, M, N, K, grp))
    p.start()
    p.join(180)
    if p.is_alive():
        p.kill()
        p.join()
        pytest.fail("the reference kernel did not finish within 180 s")
    assert p.exitcode == 0
    rep = json.loads(q.get(timeout=10))
    print("reference final kernel", M, N, K, grp, json.dumps(rep))
    assert rep["status"] == 0
    assert rep["rel_l2"] < 0.02 and rep["max_abs"] < 2.0, rep
    assert oracle is not None
