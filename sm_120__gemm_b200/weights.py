"""Persisted repacked-weight format: repack once per model, load many times.

A file holds one quantised weight in the GEMM's own layouts, so loading it is
a plain read with no quantise or repack step, and a column-parallel rank reads
only its slice (both sections are N-tile-major, so a rank's columns are one
contiguous byte range of each, the ranges i4g_shard_range gives).

Layout (little-endian):

    offset 0    header, 64 bytes:
                  magic b"I4GW", format version u32 (1), layout version u32
                  (i4g_layout_version of the tile layout), K u32, N u32,
                  group u32, tile bytes u64, scale bytes u64, 16 reserved zero
                  bytes
    offset 256  tiles:  K * N / 2 bytes (i4g_repack_umma layout)
    then        scales: (K / group) * N fp16 (i4g_repack_scales_128 layout),
                starting at the next multiple of 256 bytes

The reference has no counterpart (it requantises and repacks on every run,
src/main.cu:320-331).
"""
from __future__ import annotations

import os
import struct

import torch

from . import load as _load_lib
from . import shard_range
from .linear import QuantizedLinear

MAGIC = b"I4GW"
FORMAT_VERSION = 1
HEADER = struct.Struct("<4sIIIIIQQ16x")
DATA_OFFSET = 256


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def layout_version() -> int:
    return int(_load_lib().i4g_layout_version())


def save(lin: QuantizedLinear, path: str | os.PathLike) -> None:
    """Write `lin` (device or host tensors) to `path`."""
    tiles = lin.tiles.detach().contiguous().cpu()
    scales = lin.scales.detach().contiguous().cpu().view(torch.uint8)
    if tiles.numel() != lin.K * lin.N // 2 or scales.numel() != (lin.K // lin.group) * lin.N * 2:
        raise ValueError("tensor sizes do not match K, N, group")
    header = HEADER.pack(MAGIC, FORMAT_VERSION, layout_version(), lin.K, lin.N, lin.group,
                         tiles.numel(), scales.numel())
    scale_off = _align(DATA_OFFSET + tiles.numel())
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * (DATA_OFFSET - HEADER.size))
        f.write(tiles.numpy().tobytes())
        f.write(b"\0" * (scale_off - DATA_OFFSET - tiles.numel()))
        f.write(scales.numpy().tobytes())


def read_header(path: str | os.PathLike) -> dict:
    with open(path, "rb") as f:
        raw = f.read(HEADER.size)
    if len(raw) != HEADER.size:
        raise ValueError(f"{path}: truncated header")
    magic, ver, lver, K, N, group, tbytes, sbytes = HEADER.unpack(raw)
    if magic != MAGIC:
        raise ValueError(f"{path}: not a repacked-weight file (magic {magic!r})")
    if ver != FORMAT_VERSION:
        raise ValueError(f"{path}: format version {ver}, this library reads {FORMAT_VERSION}")
    if lver != layout_version():
        raise ValueError(f"{path}: tile layout version {lver}, this library uses "
                         f"{layout_version()}; repack the weight")
    if tbytes != K * N // 2 or sbytes != (K // group) * N * 2:
        raise ValueError(f"{path}: section sizes do not match K={K} N={N} group={group}")
    return {"K": K, "N": N, "group": group, "tile_bytes": tbytes, "scale_bytes": sbytes,
            "tile_offset": DATA_OFFSET, "scale_offset": _align(DATA_OFFSET + tbytes)}


def load(path: str | os.PathLike, device="cpu", world: int = 1, rank: int = 0) -> QuantizedLinear:
    """Read `path`, or only rank `rank`'s column slice of a `world`-way
    column-parallel split, into tensors on `device`."""
    h = read_header(path)
    K, N, group = h["K"], h["N"], h["group"]
    toff, soff, n0, n1 = shard_range(K, N, group, world, rank)
    n_local = n1 - n0
    tbytes = K * n_local // 2
    sbytes = (K // group) * n_local * 2
    tiles = torch.empty(tbytes, dtype=torch.uint8)
    scales = torch.empty(sbytes, dtype=torch.uint8)
    with open(path, "rb") as f:
        f.seek(h["tile_offset"] + toff)
        if f.readinto(tiles.numpy()) != tbytes:
            raise ValueError(f"{path}: truncated tile section")
        f.seek(h["scale_offset"] + soff)
        if f.readinto(scales.numpy()) != sbytes:
            raise ValueError(f"{path}: truncated scale section")
    dev = torch.device(device)
    if dev.type == "cuda":
        tiles = tiles.pin_memory().to(dev, non_blocking=True)
        scales = scales.pin_memory().to(dev, non_blocking=True)
    return QuantizedLinear(tiles, scales.view(torch.float16), K, n_local, group)
