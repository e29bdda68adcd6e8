"""i4g_peer_barrier on one GPU: the flag arrays of a two-rank barrier are
both local buffers, so no peer is needed. A barrier whose peer flag is
already set passes at once; one whose peer never arrives (a flag nothing
sets) gives up after its limit and reports a timeout in the device status
word, without faulting the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def i4g():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as m
    m.load()
    assert m.device_status() == 0
    return m


def test_barrier_passes_when_the_peer_has_arrived(i4g):
    mine = torch.zeros(2, dtype=torch.int64, device="cuda")   # rank 0's flags
    peer = torch.zeros(2, dtype=torch.int64, device="cuda")   # "rank 1's" flags
    mine[1] = 5  # rank 1 already stored epoch 5 into rank 0's flag for it
    i4g.peer_barrier(mine.data_ptr(), [mine.data_ptr(), peer.data_ptr()], 2, 0, 5,
                     limit_ns=100_000_000)
    torch.cuda.synchronize()
    assert i4g.device_status() == 0
    assert int(peer[0]) == 5  # this rank told rank 1


def test_barrier_times_out_when_the_peer_never_arrives(i4g):
    mine = torch.zeros(2, dtype=torch.int64, device="cuda")
    peer = torch.zeros(2, dtype=torch.int64, device="cuda")
    i4g.peer_barrier(mine.data_ptr(), [mine.data_ptr(), peer.data_ptr()], 2, 0, 1,
                     limit_ns=1_000_000)
    torch.cuda.synchronize()
    assert i4g.device_status() == -8  # I4G_ERR_TIMEOUT, read and cleared
    assert int(peer[0]) == 1
    assert i4g.device_status() == 0
    # the context is still usable
    x = torch.ones(1024, device="cuda")
    assert float(x.sum()) == 1024.0
