"""HostPipeline: GEMMs on pinned host A/C with overlapped copies."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_host_pipeline_matches_device_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as i4g
    from sm_120__gemm_b200.host import HostPipeline
    g = torch.Generator().manual_seed(11)
    lins = [i4g.QuantizedLinear.from_weight((torch.randn(1024, 512, generator=g) * 0.02)
                                            .half().cuda(), grp) for grp in (32, 64, 128)]
    a_host = [(torch.rand(M, 1024, generator=g) * 2 - 1).half().pin_memory() for M in (300, 8, 1024)]
    c_host = [torch.empty(a.shape[0], 512, dtype=torch.float16).pin_memory() for a in a_host]
    pipe = HostPipeline("cuda", 1024, 1024, 512)
    jobs = [(lins[i % 3], a_host[i % 3], c_host[i % 3]) for i in range(7)]
    pipe.run(jobs).synchronize()
    for i in range(3):
        ref = lins[i](a_host[i].cuda()).cpu()
        assert torch.equal(c_host[i].view(torch.int16), ref.view(torch.int16))


def test_host_pipeline_back_to_back_runs():
    """Two run() calls with no synchronisation between them: the second
    call's jobs reuse the device slots only after the first call's copies and
    GEMMs on them are done, so every C is right."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import sm_120__gemm_b200 as i4g
    from sm_120__gemm_b200.host import HostPipeline
    g = torch.Generator().manual_seed(12)
    lin = i4g.QuantizedLinear.from_weight((torch.randn(2048, 1024, generator=g) * 0.02)
                                          .half().cuda(), 64)
    a_host = [(torch.rand(2048, 2048, generator=g) * 2 - 1).half().pin_memory() for _ in range(6)]
    c_host = [torch.empty(2048, 1024, dtype=torch.float16).pin_memory() for _ in range(6)]
    pipe = HostPipeline("cuda", 2048, 2048, 1024)
    pipe.run([(lin, a_host[i], c_host[i]) for i in range(3)])
    pipe.run([(lin, a_host[i], c_host[i]) for i in range(3, 6)]).synchronize()
    for i in range(6):
        ref = lin(a_host[i].cuda()).cpu()
        assert torch.equal(c_host[i].view(torch.int16), ref.view(torch.int16)), i
