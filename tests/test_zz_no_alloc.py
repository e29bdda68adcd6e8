"""i4g_gemm_static_scratch: the GEMM entry point that allocates nothing.

Some callers cannot allocate device memory: a host framework whose device
memory is fully pooled, or a plugin that is handed only A, B and C. This entry
point takes i4g_gemm's arguments and keeps its split-K scratch in a fixed
static device array instead of a caller workspace. The array is loaded on a
device by the first call in the process there, so this file is collected last
and its tests pass both alone and after every other test. The GPU tests call
the C ABI directly and require the output to equal, bit for bit, the output
of the workspace entry point (i4g_gemm_ws), which runs the same schedule, on
two calls in a row through the same scratch.
"""
import ctypes

import numpy as np
import pytest
import torch

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


def _check_two_calls(i4g, L, ad, lin, ref, M, N, K, grp):
    stream = torch.cuda.current_stream()
    ref16 = u16(ref)
    for call in range(2):  # two calls in a row through the same static scratch
        c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        st = L.i4g_gemm_static_scratch(ad.data_ptr(), lin.tiles.data_ptr(), lin.scales.data_ptr(),
                                       c.data_ptr(), M, N, K, grp, stream.cuda_stream)
        assert st == 0, L.i4g_last_error().decode()
        torch.cuda.synchronize()
        assert i4g.device_status() == 0
        got = u16(c)
        print(M, N, K, grp, "call", call, "identical", bool(np.array_equal(got, ref16)))
        # the same schedule as the workspace entry point: equal bit for bit
        np.testing.assert_array_equal(got, ref16)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,grp", [
    (4096, 4096, 4096, 128),   # tcgen05, two-way split of the last wave
    (512, 1024, 4096, 64),     # tcgen05, four-way split
    (1024, 7168, 8192, 64),    # tcgen05, split tail (stream-K with I4G_STREAMK=1)
    (300, 640, 2048, 32),      # tcgen05, ragged M
    (8, 4096, 4096, 128),      # decode, cluster schedule (no scratch)
    (1, 28672, 8192, 128),     # decode, stream-K schedule through the scratch
])
def test_static_scratch_matches_workspace_entry_point(M, N, K, grp):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as i4g
    L = lib()
    a, w = make_inputs(M, N, K, seed_a=31, seed_b=37)
    lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
    ad = a.cuda()
    ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
    need = i4g.gemm_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    i4g.launch_final_ws(ad, lin.tiles, lin.scales, ref, M, N, K, grp, ws)
    torch.cuda.synchronize()
    _check_two_calls(i4g, L, ad, lin, ref, M, N, K, grp)


@pytest.mark.gpu
def test_static_scratch_decode_falls_back_when_stream_k_does_not_fit():
    """Decode shape with the stream-K schedule forced and a workspace need
    above the 40 MiB scratch (M = 16, K = 64, 4832 column tiles): the call
    runs the cluster schedule, which needs no scratch, and equals i4g_gemm."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as i4g
    L = lib()
    M, N, K, grp = 16, 4832 * 128, 64, 64
    try:
        i4g.set_decode_schedule("streamk")
        assert i4g.gemm_workspace_size(M, N, K) > (40 << 20)
        a, w = make_inputs(M, N, K, seed_a=3, seed_b=4, a_dist="normal")
        lin = i4g.QuantizedLinear.from_weight(w.cuda(), grp)
        ad = a.cuda()
        ref = torch.empty(M, N, dtype=torch.float16, device="cuda")
        i4g.launch_final(ad, lin.tiles, lin.scales, ref, M, N, K, grp)  # cluster schedule
        torch.cuda.synchronize()
        _check_two_calls(i4g, L, ad, lin, ref, M, N, K, grp)
    finally:
        i4g.set_decode_schedule("auto")
