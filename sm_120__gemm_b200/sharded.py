"""Column-parallel (N-sharded) W4A16 GEMM over torch.distributed.

Each rank owns an N/world slice of the packed weights and scales (a
contiguous byte range of the tile and scale layouts, see ``shard_range``);
the activations A are replicated. The GEMM itself needs no communication.
When a rank needs the full C, either an all-gather of the FP16 C column
blocks runs (NCCL over NVLink on GPUs, gloo on CPU in tests), which yields
the rank-major ``[world][M][N/world]`` buffer that ``assemble_columns`` turns
into row-major ``[M][N]``, or (``forward_to_peers``) every rank's GEMM
stores its columns straight into every rank's C over peer mappings and a
flag barrier (``i4g_peer_barrier``) orders the readers.

The reference has no multi-GPU path; this is the north star's harness for
configs 3 and 4 (M=8192, K=8192, N=28672; K=8192, N=57344, g64, 8 GPUs).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import (ipc_close, ipc_handle, ipc_open, launch_final_to_peers, peer_barrier,
               workspace_for)
from .linear import QuantizedLinear


def assemble_columns(gathered: torch.Tensor, world: int, M: int, n_local: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """[world * M * n_local] rank-major blocks -> row-major [M, world * n_local]."""
    blocks = gathered.view(world, M, n_local)
    if out is None:
        out = torch.empty(M, world * n_local, dtype=gathered.dtype, device=gathered.device)
    out.view(M, world, n_local).copy_(blocks.permute(1, 0, 2))
    return out


def gather_columns(c_local: torch.Tensor, group=None, out: torch.Tensor | None = None,
                   gathered: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather every rank's [M, n_local] block into the full [M, N] C."""
    world = dist.get_world_size(group)
    M, n_local = c_local.shape
    if gathered is None:
        gathered = torch.empty(world * M * n_local, dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(gathered, c_local.contiguous().view(-1), group=group)
    return assemble_columns(gathered, world, M, n_local, out)


class PeerOutputs:
    """Every rank's full C buffers ([max_m, N] FP16), mapped into every rank
    (CUDA IPC, plain peer-to-peer mappings), so that one GEMM launch per rank
    can write its column block into all of them: the all-gather fused into
    the GEMM epilogue. The same allocation holds this rank's barrier flags
    (one 64-bit flag per rank, after the C buffers), which the peers set
    through their mappings (``i4g_peer_barrier``). Collective: every rank of
    `group` constructs it, and every rank makes the same sequence of calls.

    Reuse rule. After call i's barrier a rank reads its C while its peers go
    on to call i+1, whose peer stores would overwrite C under the reader if
    both calls used one buffer (write after read). With ``slots=2`` (the
    default) consecutive calls alternate between two buffers: call i+2
    reuses call i's buffer, and no rank starts call i+2 before every rank has
    passed call i+1's barrier, which on each rank runs after everything that
    rank enqueued before call i+1. So call i's C may be read by work enqueued
    on the call's stream before the rank's call i+1. With ``slots=1`` each
    call first runs a barrier that waits for every rank to reach the call,
    i.e. to have finished reading the previous result (half the memory, one
    more barrier per call)."""

    FLAG_BYTES = 256  # room for 32 ranks; the barrier kernel takes up to 8

    def __init__(self, max_m: int, N: int, device, group=None, slots: int = 2):
        if slots not in (1, 2):
            raise ValueError("slots must be 1 or 2")
        self.max_m, self.N, self.group, self.slots = max_m, N, group, slots
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        c_bytes = max_m * N * 2
        slot_bytes = (c_bytes + 255) // 256 * 256
        self._flag_off = slots * slot_bytes
        self._raw = torch.empty(self._flag_off + self.FLAG_BYTES, dtype=torch.uint8,
                                device=device)
        self._raw[self._flag_off:].zero_()
        # the flags are zero before any peer can reach them (the handle
        # exchange below is the first point at which a peer could)
        torch.cuda.synchronize(device)
        self.bufs = [self._raw[i * slot_bytes: i * slot_bytes + c_bytes].view(torch.float16)
                     for i in range(slots)]
        mine = ipc_handle(self._raw)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self._opened = []
        peer_bases = []
        self._flag_ptrs = [0] * self.world
        for r in range(self.world):
            if r == self.rank:
                self._flag_ptrs[r] = self._raw.data_ptr() + self._flag_off
                continue
            h, off = handles[r]
            base = ipc_open(h)
            self._opened.append(base)
            peer_bases.append(base + off)
            self._flag_ptrs[r] = base + off + self._flag_off
        # per slot: this GPU's copy first, then the peers' (the kernel writes
        # them in order)
        local = self._raw.data_ptr()
        self.dsts_by_slot = [[local + i * slot_bytes] + [p + i * slot_bytes for p in peer_bases]
                             for i in range(slots)]
        self._epoch = 0
        self._calls = 0

    @property
    def dsts(self):
        """Destination pointers of the buffer the next call writes."""
        return self.dsts_by_slot[self._calls % self.slots]

    def view(self, M: int, slot: int | None = None) -> torch.Tensor:
        """[M, N] view of a buffer (default: the one the last call wrote)."""
        if slot is None:
            slot = (self._calls - 1) % self.slots
        return self.bufs[slot][: M * self.N].view(M, self.N)

    def begin_call(self, stream=None) -> list:
        """Destinations of the next call; with one slot, first a barrier that
        every rank's previous reads are ordered before."""
        if self.slots == 1 and self._calls > 0:
            self.barrier(stream)
        dsts = self.dsts
        self._calls += 1
        return dsts

    def barrier(self, stream=None) -> None:
        """Stream-ordered cross-rank barrier (a flag per rank pair over the
        peer mappings): after it, every rank's launches before it (and their
        peer stores) have completed. Every rank calls it the same number of
        times."""
        self._epoch += 1
        peer_barrier(self._flag_ptrs[self.rank], self._flag_ptrs, self.world, self.rank,
                     self._epoch, stream=stream)

    def close(self) -> None:
        torch.cuda.synchronize()
        for base in self._opened:
            ipc_close(base)
        self._opened = []


class ColumnParallelLinear:
    """This rank's column slice of a quantised weight, plus the optional gather."""

    def __init__(self, local: QuantizedLinear, world: int, rank: int, group=None):
        self.local = local
        self.world, self.rank, self.group = world, rank, group
        self.n0 = rank * local.N
        self.N = world * local.N

    @classmethod
    def from_full(cls, full: QuantizedLinear, group=None) -> "ColumnParallelLinear":
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        return cls(full.shard(world, rank), world, rank, group)

    def forward_local(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self.local(a, out=out)

    def forward(self, a: torch.Tensor, gather: bool = True) -> torch.Tensor:
        c_local = self.forward_local(a)
        if not gather or self.world == 1:
            return c_local
        return gather_columns(c_local, self.group)

    def forward_to_peers(self, a: torch.Tensor, outs: PeerOutputs, stream=None) -> torch.Tensor:
        """The full C on every rank with no separate collective: this rank's
        GEMM stores its columns into every rank's buffer over NVLink, then a
        barrier orders the readers. Returns this rank's [M, N] view, readable
        by work enqueued before this rank's next call (``PeerOutputs``'
        reuse rule)."""
        a = a.contiguous()
        M = a.shape[0]
        if M > outs.max_m or outs.N != self.N:
            raise ValueError("PeerOutputs too small for this call")
        loc = self.local
        ws = workspace_for(M, loc.N, loc.K, a.device, stream)
        dsts = outs.begin_call(stream)
        launch_final_to_peers(a, loc.tiles, loc.scales, dsts, self.N, self.n0, M, loc.N,
                              loc.K, loc.group, ws, stream)
        outs.barrier(stream)
        return outs.view(M)
