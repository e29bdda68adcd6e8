"""Host logic of the column-parallel path on CPU ranks (gloo, world size 2).

No GPU: the per-rank "GEMM" is the oracle's dequantize + cpu_gemm on the
rank's column slice, cut out of the full weight with the same shard arithmetic
(shard_range) the GPU path uses; the gather/assemble code is the product's."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import oracle
    from sm_120__gemm_b200 import shard_range
    from sm_120__gemm_b200.sharded import gather_columns

    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        M, N, K, g = 8, 512, 128, 64
        rng = np.random.default_rng(7)
        a = oracle.f2h(rng.uniform(-1, 1, (M, K)).astype(np.float32))
        w = oracle.f2h(rng.standard_normal((K, N)).astype(np.float32) * np.float32(0.02))
        packed, scales = oracle.quantize(w, K, N, g)
        tiles = oracle.repack_umma(packed, K, N)
        rsc = oracle.repack_scales_128(scales, K, N, g)
        toff, soff, n0, n1 = shard_range(K, N, g, world, rank)
        nl = n1 - n0
        # the rank's slice of the tile layout decodes to its columns
        local_tiles = tiles[toff: toff + K * nl // 2]
        local_packed = oracle.inverse_repack_umma(local_tiles, K, nl)
        full_rows = packed.reshape(K, N // 2)
        np.testing.assert_array_equal(local_packed.reshape(K, nl // 2),
                                      full_rows[:, n0 // 2: n1 // 2])
        local_rsc = rsc[soff // 2: soff // 2 + (K // g) * nl]
        np.testing.assert_array_equal(local_rsc.reshape(-1, K // g, 128),
                                      rsc.reshape(-1, K // g, 128)[n0 // 128: n1 // 128])
        deq = oracle.dequantize(local_packed, scales[:, n0:n1].copy(), K, nl, g)
        c_local = torch.from_numpy(oracle.f2h(oracle.gemm_rows(a, deq, M, nl, K))
                                   .view(np.int16)).view(torch.float16)
        full = gather_columns(c_local)
        if rank == 0:
            deq_full = oracle.dequantize(packed, scales, K, N, g)
            ref = oracle.f2h(oracle.gemm_rows(a, deq_full, M, N, K))
            result_q.put(bool(np.array_equal(full.view(torch.int16).numpy().view(np.uint16),
                                             ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_column_parallel_gather_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=10) is True


def test_assemble_columns_layout():
    from sm_120__gemm_b200.sharded import assemble_columns
    world, M, nl = 4, 3, 5
    blocks = torch.arange(world * M * nl, dtype=torch.float32)
    full = assemble_columns(blocks, world, M, nl)
    for r in range(world):
        np.testing.assert_array_equal(full[:, r * nl:(r + 1) * nl].numpy(),
                                      blocks.view(world, M, nl)[r].numpy())
