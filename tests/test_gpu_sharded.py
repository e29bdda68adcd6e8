"""Column-parallel GEMM over NCCL on 2+ GPUs (skips on a single-GPU box).

Each rank quantizes the same seeded weight, keeps its column slice (a view
into the tile and scale layouts), runs the fused GEMM on it and all-gathers
the FP16 column blocks; the gathered C must equal the single-GPU C bit for bit
(every output column is computed by the same kernel in the same k order)."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, M, N, K, group):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    import sm_120__gemm_b200 as i4g
    from sm_120__gemm_b200.sharded import ColumnParallelLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(77)
        w = (torch.randn(K, N, generator=g) * 0.02).half().cuda()
        a = (torch.rand(M, K, generator=g) * 2 - 1).half().cuda()
        full = i4g.QuantizedLinear.from_weight(w, group)
        cp = ColumnParallelLinear.from_full(full)
        c = cp.forward(a, gather=True)
        # the all-gather fused into the GEMM: peer stores, then a barrier
        from sm_120__gemm_b200.sharded import PeerOutputs
        outs = PeerOutputs(M, N, a.device)
        c2 = cp.forward_to_peers(a, outs).clone()
        torch.cuda.synchronize()
        ref = full(a)
        torch.cuda.synchronize()
        ok = (bool(torch.equal(c.view(torch.int16), ref.view(torch.int16))) and
              bool(torch.equal(c2.view(torch.int16), ref.view(torch.int16))))
        # more calls through the same buffers (barrier epochs 2, 3, ...), each
        # with new activations, read right after the barrier
        for it in range(3):
            a_it = (torch.rand(M, K, generator=g) * 2 - 1).half().cuda()
            got = cp.forward_to_peers(a_it, outs).clone()
            ok = ok and bool(torch.equal(got.view(torch.int16), full(a_it).view(torch.int16)))
        torch.cuda.synchronize()
        ok = ok and i4g.device_status() == 0
        outs.close()
        # back-to-back calls with no host synchronisation while the last rank
        # reads each result late (a sleep kernel before its copy): the reuse
        # rule (two alternating buffers, or one buffer with an entry barrier)
        # keeps a fast rank's next peer stores off a buffer still being read
        for slots in (2, 1):
            outs = PeerOutputs(M, N, a.device, slots=slots)
            a_list = [(torch.rand(M, K, generator=g) * 2 - 1).half().cuda() for _ in range(4)]
            copies = []
            for a_it in a_list:
                view = cp.forward_to_peers(a_it, outs)
                if rank == world - 1:
                    torch.cuda._sleep(4_000_000)  # ~2 ms: this rank reads late
                copies.append(view.clone())
            torch.cuda.synchronize()
            for a_it, got in zip(a_list, copies):
                ok = ok and bool(torch.equal(got.view(torch.int16), full(a_it).view(torch.int16)))
            ok = ok and i4g.device_status() == 0
            outs.close()
        flags = [None] * world
        dist.all_gather_object(flags, ok)
        if rank == 0:
            q.put(all(flags))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K,group", [(512, 1024, 1024, 64), (8, 2048, 2048, 128),
                                         (300, 4096, 512, 32)])
def test_column_parallel_matches_single_gpu(M, N, K, group):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = min(torch.cuda.device_count(), 4)
    while N % (128 * world):
        world -= 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, M, N, K, group))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert q.get(timeout=10) is True
