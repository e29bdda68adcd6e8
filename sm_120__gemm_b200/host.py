"""GEMMs on host-resident activations, with the PCIe copies overlapped.

A caller whose A and C live in pinned host memory pays a host-to-device copy
of A and a device-to-host copy of C around every GEMM, and PCIe (about 50
GB/s per direction) is far slower than the GEMM. ``HostPipeline`` runs a list
of such GEMMs on three streams (copy in, compute, copy out) over two device
buffer slots, so the copy of job i+1's A, the GEMM of job i and the copy of
job i-1's C run at the same time and both PCIe directions stay busy.
"""
from __future__ import annotations

import torch


class HostPipeline:
    def __init__(self, device, max_m: int, max_k: int, max_n: int, depth: int = 2,
                 fp32_out: bool = False):
        self.device = torch.device(device)
        self.depth = depth
        self.fp32_out = fp32_out
        cdt = torch.float32 if fp32_out else torch.float16
        self.a_dev = [torch.empty(max_m * max_k, dtype=torch.float16, device=self.device)
                      for _ in range(depth)]
        self.c_dev = [torch.empty(max_m * max_n, dtype=cdt, device=self.device)
                      for _ in range(depth)]
        self.h2d = torch.cuda.Stream(self.device)
        self.compute = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        ev = lambda: [torch.cuda.Event() for _ in range(depth)]  # noqa: E731
        self.a_ready, self.a_free, self.c_done, self.c_free = ev(), ev(), ev(), ev()
        # jobs enqueued over every run(): a slot is reused (and its events
        # must be waited for) from the depth-th job of the pipeline's life on,
        # whatever run() call it belongs to
        self._jobs = 0

    def run(self, jobs, after: torch.cuda.Event | None = None) -> torch.cuda.Event:
        """Enqueue `jobs`, a list of (QuantizedLinear, A host [M, K] fp16, C
        host [M, N]), after event `after` (if given). Returns an event that
        completes when every C has reached the host."""
        streams = (self.h2d, self.compute, self.d2h)
        if after is not None:
            for s in streams:
                s.wait_event(after)
        for lin, a_host, c_host in jobs:
            n = self._jobs
            self._jobs += 1
            slot = n % self.depth
            M, K = a_host.shape
            a = self.a_dev[slot][: M * K].view(M, K)
            c = self.c_dev[slot][: M * lin.N].view(M, lin.N)
            reuse = n >= self.depth
            with torch.cuda.stream(self.h2d):
                if reuse:
                    self.h2d.wait_event(self.a_free[slot])
                a.copy_(a_host, non_blocking=True)
                self.a_ready[slot].record(self.h2d)
            with torch.cuda.stream(self.compute):
                self.compute.wait_event(self.a_ready[slot])
                if reuse:
                    self.compute.wait_event(self.c_free[slot])
                lin(a, out=c, fp32_out=self.fp32_out, stream=self.compute)
                self.a_free[slot].record(self.compute)
                self.c_done[slot].record(self.compute)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.c_done[slot])
                c_host.copy_(c, non_blocking=True)
                self.c_free[slot].record(self.d2h)
        done = torch.cuda.Event()
        self.compute.wait_stream(self.h2d)
        self.compute.wait_stream(self.d2h)
        done.record(self.compute)
        return done
