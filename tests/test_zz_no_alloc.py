"""i4g_gemm_static_scratch: the GEMM entry point that allocates nothing.

Its split-K scratch is a fixed static device array, so this file is collected
last (the scratch's module is loaded by the first call in the process) and its
tests must pass both alone and after every other test. The GPU tests call the
C ABI directly and compare with i4g_gemm_ws on a caller-owned workspace.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from parity import make_inputs, u16

_vp, _i = ctypes.c_void_p, ctypes.c_int


def lib():
    import sm_120__gemm_b200 as m
    L = m.load()
    L.i4g_gemm_static_scratch.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]
    L.i4g_gemm_static_scratch.restype = _i
    return L


def test_static_scratch_rejects_bad_shapes_without_a_gpu():
    L = lib()
    # shape checks come before any device access
    assert L.i4g_gemm_static_scratch(None, None, None, None, 0, 128, 64, 128, None) == -2
    assert L.i4g_gemm_static_scratch(None, None, None, None, 64, 100, 64, 128, None) == -2
    assert L.i4g_gemm_static_scratch(None, None, None, None, 64, 128, 96, 128, None) == -2


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,grp", [(4096, 4096, 4096, 128), (512, 1024, 4096, 64),
                                       (1024, 7168, 8192, 64), (300, 640, 2048, 32),
                                       (8, 4096, 4096, 128)])
def test_static_scratch_matches_workspace_entry_point(M, N, K, grp):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as i4g
    L = lib()
    a, w = make_inputs(M, N, K, seed_a=31, seed_b=37)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ad = a.cuda()
    stream = torch.cuda.current_stream()

    ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
    need = i4g.gemm_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    i4g.launch_final_ws(ad, lin.tiles, lin.scales, ref, M, N, K, grp, ws, stream)
    torch.cuda.synchronize()
    ref16 = u16(ref)

    for call in range(2):  # two calls in a row through the same static scratch
        c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        st = L.i4g_gemm_static_scratch(ad.data_ptr(), lin.tiles.data_ptr(), lin.scales.data_ptr(),
                                       c.data_ptr(), M, N, K, grp, stream.cuda_stream)
        assert st == 0, L.i4g_last_error().decode()
        torch.cuda.synchronize()
        assert i4g.device_status() == 0
        got = u16(c)
        # tolerance: at most 1 FP16 ulp from the workspace entry point (the
        # two run the same schedule, so they agree bit for bit in practice)
        ulp = oracle.ulp_distance(got, ref16)
        print(M, N, K, grp, "call", call, "max ulp", int(ulp.max()),
              "identical", bool(np.array_equal(got, ref16)))
        assert int(ulp.max()) <= 1
