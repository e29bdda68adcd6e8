"""Persisted repacked-weight format (sm_120__gemm_b200.weights)."""
import struct

import numpy as np
import pytest
import torch

import sm_120__gemm_b200 as i4g
from sm_120__gemm_b200 import weights


def random_linear(K, N, group, seed=0):
    g = torch.Generator().manual_seed(seed)
    tiles = torch.randint(0, 256, (K * N // 2,), generator=g, dtype=torch.uint8)
    scales = (torch.rand((K // group) * N, generator=g) * 0.01).half()
    return i4g.QuantizedLinear(tiles, scales, K, N, group)


@pytest.mark.parametrize("K,N,group", [(64, 128, 32), (256, 512, 64), (1024, 1024, 128)])
def test_roundtrip(tmp_path, K, N, group):
    lin = random_linear(K, N, group)
    p = tmp_path / "w.i4g"
    weights.save(lin, p)
    h = weights.read_header(p)
    assert (h["K"], h["N"], h["group"]) == (K, N, group)
    assert h["tile_offset"] % 256 == 0 and h["scale_offset"] % 256 == 0
    back = weights.load(p)
    assert (back.K, back.N, back.group) == (K, N, group)
    assert torch.equal(back.tiles, lin.tiles)
    assert torch.equal(back.scales.view(torch.int16), lin.scales.view(torch.int16))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_load_reads_the_rank_slice(tmp_path, world):
    K, N, group = 256, 1024, 64
    lin = random_linear(K, N, group, seed=world)
    p = tmp_path / "w.i4g"
    weights.save(lin, p)
    for rank in range(world):
        part = weights.load(p, world=world, rank=rank)
        ref = lin.shard(world, rank)
        assert part.N == N // world
        assert torch.equal(part.tiles, ref.tiles)
        assert torch.equal(part.scales.view(torch.int16), ref.scales.view(torch.int16))


def test_rejects_foreign_and_damaged_files(tmp_path):
    lin = random_linear(64, 128, 32)
    p = tmp_path / "w.i4g"
    weights.save(lin, p)
    raw = bytearray(p.read_bytes())
    bad = tmp_path / "bad.i4g"
    bad.write_bytes(b"NOPE" + bytes(raw[4:]))
    with pytest.raises(ValueError, match="magic"):
        weights.load(bad)
    wrong_layout = bytearray(raw)
    wrong_layout[8:12] = struct.pack("<I", 99)
    bad.write_bytes(bytes(wrong_layout))
    with pytest.raises(ValueError, match="layout version"):
        weights.load(bad)
    bad.write_bytes(bytes(raw[:-10]))
    with pytest.raises(ValueError, match="truncated"):
        weights.load(bad)


@pytest.mark.gpu
def test_saved_weight_gives_identical_gemm(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    K, N, group, M = 1024, 512, 128, 64
    w = (torch.randn(K, N, generator=torch.Generator().manual_seed(3)) * 0.02).half().cuda()
    lin = i4g.QuantizedLinear.from_weight(w, group)
    p = tmp_path / "w.i4g"
    weights.save(lin, p)
    back = weights.load(p, device="cuda")
    a = torch.randn(M, K, device="cuda").half()
    c0 = lin(a)
    c1 = back(a)
    torch.cuda.synchronize()
    assert torch.equal(c0.view(torch.int16), c1.view(torch.int16))
