"""Decode calls launched as programmatic dependents of the previous kernel.

The cluster-schedule decode kernel may start while the kernel before it on
the stream still runs: it warms L2 with its weights, then waits for that
kernel before it reads A or writes C. These tests chain calls whose A is the
previous call's C (a read-after-write across kernels) and whose C buffers are
reused (write-after-write), captured in one CUDA graph so the launches
overlap, and require the result to equal, bit for bit, the same chain run
with a device synchronisation between calls.
"""
import numpy as np
import pytest
import torch

from parity import u16


@pytest.fixture(scope="module")
def i4g():
    import sm_120__gemm_b200 as m
    m.load()
    torch.cuda.set_device(0)
    return m


def _layers(i4g, n, K, grp, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [i4g.QuantizedLinear.from_weight(
        (torch.randn(K, K, generator=gen, device="cuda") * (1.0 / K ** 0.5)).half(), grp)
        for _ in range(n)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,grp", [(1, 128), (8, 64), (16, 32)])
def test_chained_decode_in_graph_equals_synchronised_chain(i4g, M, grp):
    K, L = 4096, 12
    layers = _layers(i4g, L, K, grp, seed=100 + M)
    gen = torch.Generator(device="cuda").manual_seed(M)
    x0 = torch.randn(M, K, generator=gen, device="cuda").half()
    bufs = [torch.empty(M, K, dtype=torch.float16, device="cuda") for _ in range(2)]

    # reference: one call at a time
    ref = []
    x = x0
    for i, lin in enumerate(layers):
        y = bufs[i % 2]
        lin(x, out=y)
        torch.cuda.synchronize()
        ref.append(u16(y).copy())
        x = y
    assert i4g.device_status() == 0

    # the same chain, back to back inside one CUDA graph, twice: (1) outputs
    # ping-pong between two buffers, so every call also overwrites the A its
    # predecessor reads (write-after-read); (2) every call writes a buffer
    # of its own, so every layer's output can be checked.
    outs = [torch.empty(M, K, dtype=torch.float16, device="cuda") for _ in range(L)]
    for pingpong in (True, False):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                x = x0
                for i, lin in enumerate(layers):
                    y = bufs[i % 2] if pingpong else outs[i]
                    lin(x, out=y, stream=side)
                    x = y
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(3):  # replays reuse every buffer
            for t in bufs + outs:
                t.fill_(float("nan"))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            assert i4g.device_status() == 0
            if pingpong:
                np.testing.assert_array_equal(u16(bufs[(L - 1) % 2]), ref[L - 1])
            else:
                for i in range(L):
                    np.testing.assert_array_equal(u16(outs[i]), ref[i], err_msg=f"layer {i}")
        del g


@pytest.mark.gpu
def test_decode_after_a_producer_kernel_reads_its_output(i4g):
    """A decode call right after a kernel that writes its A (an ordinary
    kernel, which never signals its dependents early) reads the new A."""
    K, M = 4096, 4
    lin = _layers(i4g, 1, K, 128, seed=5)[0]
    gen = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(M, K, generator=gen, device="cuda").half()
    expected = u16(lin(a)).copy()
    torch.cuda.synchronize()
    src = a.clone()
    a.zero_()
    c = torch.empty(M, K, dtype=torch.float16, device="cuda")
    for _ in range(5):
        a.zero_()
        torch.cuda.synchronize()
        a.copy_(src)          # the producer
        lin(a, out=c)         # its dependent
        torch.cuda.synchronize()
        np.testing.assert_array_equal(u16(c), expected)
