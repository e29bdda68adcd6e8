"""A quantised weight held in the sm_100a layouts, and its GEMM.

Owns the two device buffers the fused GEMM reads: the tile-layout INT4 codes
(``launch_repack_umma``) and the 128-column scale layout
(``launch_repack_scales_128``). Column-parallel shards are zero-copy views:
a rank's columns are one contiguous byte range of each buffer.
"""
from __future__ import annotations

import torch

from . import (launch_final_fp32_ws, launch_final_ws, launch_quantize_repack,
               launch_repack_scales_128, launch_repack_umma, shard_range, workspace_for)


class QuantizedLinear:
    def __init__(self, tiles: torch.Tensor, scales: torch.Tensor, K: int, N: int, group: int):
        if tiles.dtype != torch.uint8 or scales.dtype != torch.float16:
            raise TypeError("tiles must be uint8 and scales float16")
        if tiles.numel() != K * N // 2 or scales.numel() != (K // group) * N:
            raise ValueError("buffer sizes do not match K, N, group")
        self.tiles, self.scales = tiles, scales
        self.K, self.N, self.group = K, N, group

    @classmethod
    def from_weight(cls, w: torch.Tensor, group: int, stream=None) -> "QuantizedLinear":
        """Quantise an fp16 [K, N] weight on the GPU (codes and scales
        bit-identical to the reference's quantize_cpu) straight into the GEMM
        layouts, in one pass."""
        if w.dtype != torch.float16 or w.dim() != 2 or not w.is_cuda:
            raise TypeError("weight must be a 2-D float16 CUDA tensor [K, N]")
        w = w.contiguous()
        K, N = w.shape
        dev = w.device
        tiles = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
        rscales = torch.empty((K // group) * N, dtype=torch.float16, device=dev)
        launch_quantize_repack(w, tiles, rscales, K, N, group, stream)
        return cls(tiles, rscales, K, N, group)

    @classmethod
    def from_packed(cls, packed: torch.Tensor, scales: torch.Tensor, K: int, N: int,
                    group: int, stream=None) -> "QuantizedLinear":
        """Repack reference-layout codes ([K][N] nibbles) and scales ([K/g][N])."""
        dev = packed.device
        tiles = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
        rscales = torch.empty((K // group) * N, dtype=torch.float16, device=dev)
        launch_repack_umma(packed, tiles, K, N, stream)
        launch_repack_scales_128(scales, rscales, K, N, group, stream)
        return cls(tiles, rscales, K, N, group)

    def shard(self, world: int, rank: int) -> "QuantizedLinear":
        """This rank's column slice of a world-way column-parallel split (a view)."""
        toff, soff, n0, n1 = shard_range(self.K, self.N, self.group, world, rank)
        n_local = n1 - n0
        tiles = self.tiles[toff: toff + self.K * n_local // 2]
        s0 = soff // 2
        scales = self.scales[s0: s0 + (self.K // self.group) * n_local]
        return QuantizedLinear(tiles, scales, self.K, n_local, self.group)

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None, fp32_out: bool = False,
                 stream=None) -> torch.Tensor:
        if a.dtype != torch.float16 or a.dim() != 2 or a.shape[1] != self.K:
            raise ValueError(f"A must be float16 [M, {self.K}]")
        a = a.contiguous()
        M = a.shape[0]
        if out is None:
            out = torch.empty(M, self.N, dtype=torch.float32 if fp32_out else torch.float16,
                              device=a.device)
        ws = workspace_for(M, self.N, self.K, a.device, stream)
        fn = launch_final_fp32_ws if fp32_out else launch_final_ws
        fn(a, self.tiles, self.scales, out, M, self.N, self.K, self.group, ws, stream)
        return out
