"""Benchmark of the fused W4A16 GEMM (the reference's headline metric).

Metric: effective TFLOP/s (2*M*N*K / time) at M=N=K=4096 for
group 32, 64 and 128; decode-shaped HBM GB/s; fraction of peak.

A step is the headline workload of configs[1]: three fused GEMMs at
M=N=K=4096, one per group size (32, 64, 128), each on its own quantised
weight, FP16 C. Under torchrun every rank owns its own 4096-column slice of
a column-parallel weight (N_total = 4096 * world), so per-GPU work is fixed
("weak" scaling), and every GEMM delivers the full [4096, N_total] C to every
rank: by default its epilogue stores the rank's columns into every rank's C
over NVLink and a flag barrier ends the call (--gather nccl: plain GEMM, then
NCCL all-gather + permute). After the timing the gathered C is checked bit
for bit against an NCCL gather of per-rank GEMMs. Extra blocks time configs[3]
(prefill, strong scaling over the job's GPUs) and configs[4] (the M sweep with
the gather), and at N = 1 the end-to-end path, the decode shapes, the
reference's "separate" dequant + cuBLAS row and the CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The reference arm (--impl reference) times the reference's own CPU
implementation of the path (oracle/_ref: its unmodified src/reference.cu,
dequantize_cpu + cpu_gemm_fp32, one std::thread per host core over disjoint
row slices) on a bounded row sample of the same workload, extrapolated.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_HEAD = N_HEAD = K_HEAD = 4096
GROUPS = (32, 64, 128)
METRIC = "Effective TFLOP/s @4096^3 g32/64/128"
UNIT = "TFLOP/s"
WORKLOAD = "fused W4A16 GEMM, M=N=K=4096, groups 32/64/128 (one GEMM each per step)"


def flops(M, N, K):
    return 2.0 * M * N * K


def algorithmic_bytes(M, N, K, g):
    return 2 * M * K + K * N // 2 + 2 * N * (K // g) + 2 * M * N


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_profile_traffic():
    """dram bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML read every 2 ms from a thread (read-only queries), or
    nvidia-smi -lms 20 where NVML cannot be loaded."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.device_index = device_index
        self.period_s = period_s
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []  # (sm_mhz, max_mhz, reasons) from NVML
        self.first = 0
        self.stop = threading.Event()

    def _nvml_sample(self):
        n = self.nvml
        try:
            sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            self.samples.append((sm, self.max_mhz, {k for k, b in self.bits.items() if r & b}))
        except Exception:  # noqa: BLE001 - a failed read only loses a sample
            pass

    def _nvml_poll(self):
        while not self.stop.is_set():
            self._nvml_sample()
            self.stop.wait(self.period_s)

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = n = pynvml
            self.handle = n.nvmlDeviceGetHandleByIndex(self.device_index)
            self.max_mhz = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
            self.bits = {"hw_slowdown": n.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": n.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": n.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": n.nvmlClocksEventReasonSwPowerCap}
            self.thread = threading.Thread(target=self._nvml_poll, daemon=True)
            self.thread.start()
            # the poller is running before the timed region starts; samples
            # from here on are the region's (a short region still gets some:
            # the poller runs while the host waits in the final synchronize)
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:
                time.sleep(0.0005)
            self.first = len(self.samples)
            return self
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:
                time.sleep(0.01)
            self.first = len(self.lines)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._nvml_sample()  # as the region ends
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self.nvml.nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        if self.nvml is not None:
            for s_mhz, m_mhz, rs in self.samples[self.first:]:
                sm.append(float(s_mhz))
                mx = float(m_mhz)
                reasons |= rs
            source = f"NVML every {self.period_s * 1e3:.0f} ms"
        else:
            for line in self.lines[max(0, self.first - 1):]:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for name, val in zip(self.NAMES, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
            source = "nvidia-smi -lms 20"
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0,
                    "source": source}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": source}


# ------------------------------------------------------------ our arm

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import sm_120__gemm_b200 as i4g
    from sm_120__gemm_b200.sharded import PeerOutputs, gather_columns

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    M, K = M_HEAD, K_HEAD
    n_local = N_HEAD
    n_total = n_local * world
    n0 = rank * n_local
    peaks = load_peaks()
    gather = args.gather if world > 1 else "none"

    # Seeded synthetic inputs: A fp16 U[-1,1]; W fp32 N(0, 0.02) -> fp16 ->
    # quantised on the GPU (codes bit-identical to quantize_cpu). Each rank
    # builds only its own column slice of the full weight (seeded by rank).
    def weights(g, rep):
        gen = torch.Generator(device=dev).manual_seed(5678 + 1000 * rep + 17 * g + 7919 * rank)
        w = (torch.randn(K, n_local, generator=gen, device=dev) * 0.02).half()
        return i4g.QuantizedLinear.from_weight(w, g)

    # Rotating inputs keep each GEMM's operands out of L2 (126 MB) when the
    # GEMM runs: 4 activation buffers (32 MiB each) and 2 weight sets per group.
    # The activations are the same on every rank (replicated A), as in a
    # column-parallel layer.
    n_act, n_wset = 4, 2
    gen_a = torch.Generator(device=dev).manual_seed(1234)
    acts = [(torch.rand(M, K, generator=gen_a, device=dev) * 2 - 1).half() for _ in range(n_act)]
    lins = {g: [weights(g, r) for r in range(n_wset)] for g in GROUPS}
    outs = [torch.empty(M, n_local, dtype=torch.float16, device=dev) for _ in range(3)]
    # Split-K workspace for the last partial wave (None: whole tiles only).
    ws = i4g.workspace_for(M, n_local, K, dev, stream) if args.schedule == "split" else None
    # At N > 1 every GEMM also delivers the full [M, N_total] C to every rank:
    # "fused" stores each rank's columns straight into every rank's C from the
    # GEMM epilogue (i4g_gemm_to_peers) and ends with the flag barrier;
    # "nccl" runs the plain GEMM, then an NCCL all-gather and the permute.
    peer = PeerOutputs(M, n_total, dev) if gather == "fused" else None
    full = torch.empty(M, n_total, dtype=torch.float16, device=dev) if gather == "nccl" else None
    gbuf = (torch.empty(world * M * n_local, dtype=torch.float16, device=dev)
            if gather == "nccl" else None)
    torch.cuda.synchronize()

    def gemm(lin, a, g, j):
        if peer is not None:
            dsts = peer.begin_call(stream)
            i4g.launch_final_to_peers(a, lin.tiles, lin.scales, dsts, n_total, n0, M, n_local, K,
                                      g, ws, stream)
        else:
            i4g.launch_final_ws(a, lin.tiles, lin.scales, outs[j], M, n_local, K, g, ws, stream)

    def step(i, events=None):
        for j, g in enumerate(GROUPS):
            lin = lins[g][(i + j) % n_wset]
            a = acts[(3 * i + j) % n_act]
            if events is not None:
                events[j][0].record(stream)
            gemm(lin, a, g, j)
            if events is not None:
                events[j][1].record(stream)
            if peer is not None:
                peer.barrier(stream)
            elif gather == "nccl":
                gather_columns(outs[j], out=full, gathered=gbuf)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if i4g.device_status() != 0:
        raise RuntimeError("device-side wait timed out during warm-up")

    # The timed region holds the steps alone: events around every GEMM would
    # stretch each one by ~14 us (117 -> 132 us at 4096^3 on B200), so the
    # per-GEMM split is taken in a separate pass after it.
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(stop)
    if i4g.device_status() != 0:
        raise RuntimeError("device-side wait timed out during timing")
    # Per-GEMM event pairs (every rank takes the same steps, barriers included).
    split_steps = min(args.steps, 20)
    kernel_events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in GROUPS]
                     for _ in range(split_steps)]
    for i in range(split_steps):
        step(args.warmup + args.steps + i, kernel_events[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    per_group_ms = {g: [kernel_events[i][j][0].elapsed_time(kernel_events[i][j][1])
                        for i in range(split_steps)] for j, g in enumerate(GROUPS)}
    if i4g.device_status() != 0:
        raise RuntimeError("device-side wait timed out during the per-GEMM pass")

    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    # The gathered C of the last GEMM, checked bit for bit on every rank
    # against an NCCL all-gather of per-rank plain GEMMs (outside the timing).
    gather_check = None
    if gather != "none":
        last = args.warmup + args.steps + split_steps - 1  # the per-GEMM pass ran last
        g = GROUPS[-1]
        lin = lins[g][(last + len(GROUPS) - 1) % n_wset]
        a = acts[(3 * last + len(GROUPS) - 1) % n_act]
        got = (peer.view(M) if peer is not None else full).clone()
        ref = gather_columns(lin(a))
        same = torch.tensor([float(torch.equal(got.view(torch.int16), ref.view(torch.int16)))],
                            device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        gather_check = bool(same.item() == 1.0)

    step_flops_rank = sum(flops(M, n_local, K) for _ in GROUPS)
    value = step_flops_rank * world * args.steps / (ms_max * 1e-3) / 1e12
    kernel_ms = {g: statistics.mean(v) for g, v in per_group_ms.items()}
    if gather == "none":
        # the timed region holds only gemm_tc_kernel launches: its time per
        # step is the kernels' summed average launch duration (gaps included)
        kernel_total_ms = ms / args.steps
        duration_source = ("timed region / launches (the region holds only the "
                           f"{len(GROUPS) * args.steps} gemm_tc_kernel launches)")
    else:
        kernel_total_ms = sum(kernel_ms.values())
        duration_source = (f"CUDA events around each GEMM ({split_steps} steps after the "
                           "timed region; the region also holds the gather barriers)")
    achieved = step_flops_rank / (kernel_total_ms * 1e-3) / 1e12
    gather_desc = {"none": "none (one GPU)" if world == 1 else "none",
                   "fused": "fused: GEMM epilogue stores into every rank's C + flag barrier",
                   "nccl": "NCCL all_gather_into_tensor + permute after each GEMM"}[gather]
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded): A fp16 U[-1,1]; W fp32 N(0,0.02) -> fp16 -> INT4",
        "config": {"workload": WORKLOAD, "M": M, "N_per_gpu": n_local, "N_total": n_total,
                   "K": K, "groups": list(GROUPS), "parallelism": f"column-parallel x{world}",
                   "gather": gather_desc,
                   "l2": "rotating inputs: 4 x 32 MiB activations, 2 weight sets per group",
                   "schedule": args.schedule + (f" (workspace {ws.numel()} B)" if ws is not None
                                                else "")},
        "per_group": {str(g): {"kernel_ms": round(kernel_ms[g], 4),
                               "tflops": round(flops(M, n_local, K) / kernel_ms[g] / 1e9, 1)}
                      for g in GROUPS},
        "per_group_timing": f"CUDA events around each GEMM, {split_steps} steps after the "
                            "timed region (each pair adds a few us)",
        "gpu_launches": args.steps * len(GROUPS) * (2 if peer is not None else 1),
    }
    if gather_check is not None:
        result["gather_check"] = {"bitwise_equal_to_nccl_gather_on_every_rank": gather_check}
    traffic = load_profile_traffic().get("tc_4096_g128_bytes_per_launch")
    result["roofline"] = {
        "bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
        "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
        "traffic": traffic,
        "peak_source": f"{peaks['source']} (cuBLAS bf16 burst; fp16 dense runs at the bf16 rate)",
        "kernel": "gemm_tc_kernel (tcgen05, TMEM)" + (", with peer stores" if peer else ""),
        "duration_source": duration_source,
        "algorithmic_bytes_per_launch": algorithmic_bytes(M, n_local, K, 128),
    }
    result["clocks"] = clocks.summary()
    if peer is not None:
        peer.close()
    del outs, full, gbuf, peer
    torch.cuda.empty_cache()

    if not args.no_extras:
        result["prefill_strong"] = run_prefill(args, i4g, rank, world, dev)
        result["m_sweep"] = run_m_sweep(args, i4g, rank, world, dev)
    if rank == 0 and world == 1 and not args.no_extras:
        result["e2e"] = run_e2e(args, i4g, lins, dev)
        result["decode"] = run_decode(args, i4g, dev, peaks)
        result["separate_baseline"] = run_separate(args, i4g, lins, dev)
        result["cpu_baseline"] = cpu_baseline(args, sample_rows=args.cpu_rows)
    elif rank == 0:
        result["e2e"] = run_e2e(args, i4g, lins, dev)
    return result


def _time_max(fn, iters, dev, world):
    """Device time per call of fn (CUDA events on the current stream, after 3
    warm-ups), max over ranks. On one GPU the stream first runs a 2 ms spin
    kernel while the host enqueues every call, and the start event follows the
    spin: the calls then run back to back on the device, so a call shorter
    than its Python launch path (decode-sized M) is timed, not the host."""
    import torch
    import torch.distributed as dist
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if world == 1:
        # (with several ranks the spin would move the ranks' host skew into
        # the first call's cross-GPU barrier, so they start unqueued)
        clock_khz = getattr(torch.cuda.get_device_properties(dev), "clock_rate", 0) or 1965000
        torch.cuda._sleep(int(2e-3 * clock_khz * 1e3))
    b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    t = torch.tensor([b.elapsed_time(e) * 1e3 / iters], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _column_parallel(i4g, rank, world, dev, K, N, g, seed):
    import torch
    from sm_120__gemm_b200.sharded import ColumnParallelLinear
    n_local = N // world
    gen = torch.Generator(device=dev).manual_seed(seed + rank)
    w = (torch.randn(K, n_local, generator=gen, device=dev) * 0.02).half()
    lin = i4g.QuantizedLinear.from_weight(w, g)
    del w
    return ColumnParallelLinear(lin, world, rank), n_local


def run_prefill(args, i4g, rank, world, dev):
    """M=8192, K=8192, N=28672, g128, column-parallel over the job's
    G = world GPUs (N/G columns each; strong scaling across G). Per call: the
    GEMM alone and the GEMM with the full C delivered to every rank (fused
    gather) when G > 1; whole-job TFLOP/s from the max-over-ranks time."""
    import torch
    from sm_120__gemm_b200.sharded import PeerOutputs
    M, K, N, g = 8192, 8192, 28672, 128
    cp, n_local = _column_parallel(i4g, rank, world, dev, K, N, g, 777)
    a = (torch.rand(M, K, generator=torch.Generator(device=dev).manual_seed(31), device=dev)
         * 2 - 1).half()
    c = torch.empty(M, n_local, dtype=torch.float16, device=dev)
    gemm_us = _time_max(lambda: cp.forward_local(a, out=c), args.extra_iters, dev, world)
    out = {"workload": "configs[3]: M=8192 K=8192 N=28672 g128, column-parallel",
           "G": world, "N_per_gpu": n_local, "gemm_us": round(gemm_us, 1),
           "gemm_tflops": round(2.0 * M * N * K / (gemm_us * 1e-6) / 1e12, 1)}
    if world > 1:
        peer = PeerOutputs(M, N, dev)
        e2e_us = _time_max(lambda: cp.forward_to_peers(a, peer), args.extra_iters, dev, world)
        peer.close()
        out.update({"gemm_plus_fused_gather_us": round(e2e_us, 1),
                    "e2e_tflops": round(2.0 * M * N * K / (e2e_us * 1e-6) / 1e12, 1)})
        del peer
    del cp, a, c
    torch.cuda.empty_cache()
    return out


def run_m_sweep(args, i4g, rank, world, dev):
    """K=8192, N=57344 (fused gate+up), g64, each rank N/G columns
    (the config names G = 8); per M, the kernel the dispatcher picks, the GEMM
    alone and, when G > 1, the GEMM with the full C on every rank by the fused
    gather and by NCCL all-gather + permute (max-over-ranks device times)."""
    import torch
    from sm_120__gemm_b200.sharded import PeerOutputs, gather_columns
    K, N, g = 8192, 57344, 64
    cp, n_local = _column_parallel(i4g, rank, world, dev, K, N, g, 9000)
    gen = torch.Generator(device=dev).manual_seed(4321)
    res = {"workload": "configs[4]: K=8192 N=57344 g64, column-parallel", "G": world,
           "N_per_gpu": n_local}
    for M in (1, 16, 128, 1024, 4096, 16384):
        a = (torch.rand(M, K, generator=gen, device=dev) * 2 - 1).half()
        c = torch.empty(M, n_local, dtype=torch.float16, device=dev)
        p = i4g.plan(M, n_local, K, g, torch.cuda.get_device_properties(dev).multi_processor_count,
                     i4g.gemm_workspace_size(M, n_local, K))
        row = {"kernel": p["kernel"], "schedule": p["schedule"]}
        row["gemm_us"] = round(_time_max(lambda: cp.forward_local(a, out=c), args.extra_iters,
                                         dev, world), 2)
        if world > 1:
            peer = PeerOutputs(M, N, dev)
            row["fused_gather_us"] = round(_time_max(lambda: cp.forward_to_peers(a, peer),
                                                     args.extra_iters, dev, world), 2)
            full = torch.empty(M, N, dtype=torch.float16, device=dev)
            gbuf = torch.empty(world * M * n_local, dtype=torch.float16, device=dev)

            def nccl():
                cp.forward_local(a, out=c)
                gather_columns(c, out=full, gathered=gbuf)

            row["nccl_gather_us"] = round(_time_max(nccl, args.extra_iters, dev, world), 2)
            # each rank receives (G-1)/G of C over NVLink
            row["gather_bytes_in_per_rank"] = (world - 1) * M * n_local * 2
            peer.close()
            del peer, full, gbuf
        res[f"M{M}"] = row
        del a, c
        torch.cuda.empty_cache()
    del cp
    torch.cuda.empty_cache()
    return res


def run_separate(args, i4g, lins, dev):
    """The reference's "separate" comparison row (src/main.cu:319): the
    dequantize kernel materialises B in FP16, then cuBLAS (torch.matmul) runs
    the FP16 GEMM, at the headline shape, g128; beside the fused kernel."""
    import torch
    M, N, K, g = M_HEAD, N_HEAD, K_HEAD, 128
    gen = torch.Generator(device=dev).manual_seed(55)
    w = (torch.randn(K, N, generator=gen, device=dev) * 0.02).half()
    packed = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(K // g, N, dtype=torch.float16, device=dev)
    i4g.launch_quantize(w, packed, scales, K, N, g)
    lin = i4g.QuantizedLinear.from_packed(packed, scales, K, N, g)
    b16 = torch.empty(K, N, dtype=torch.float16, device=dev)
    a = (torch.rand(M, K, generator=gen, device=dev) * 2 - 1).half()
    c = torch.empty(M, N, dtype=torch.float16, device=dev)
    ws = i4g.workspace_for(M, N, K, dev)

    def separate():
        i4g.launch_dequantize(packed, scales, b16, K, N, g)
        torch.matmul(a, b16, out=c)

    def fused():
        i4g.launch_final_ws(a, lin.tiles, lin.scales, c, M, N, K, g, ws)

    out = {}
    for name, fn in (("dequant_plus_cublas_us", separate),
                     ("cublas_fp16_only_us", lambda: torch.matmul(a, b16, out=c)),
                     ("fused_us", fused)):
        out[name] = round(_time_max(fn, 50, dev, 1), 1)
    out["fused_speedup_vs_separate"] = round(out["dequant_plus_cublas_us"] / out["fused_us"], 3)
    out["note"] = ("M=N=K=4096 g128, warm L2 (same operands each call); the reference's "
                   "'separate' and 'cublas_fp16' rows")
    return out


def run_e2e(args, i4g, lins, dev):
    """Same metric through the public API with host buffers: every GEMM copies
    its A from pinned host memory and reads its C back, inside the timed loop
    (sm_120__gemm_b200.host.HostPipeline overlaps the two copy directions and
    the GEMMs on three streams)."""
    import torch

    from sm_120__gemm_b200.host import HostPipeline

    M, K, N = M_HEAD, K_HEAD, N_HEAD
    a_host = [(torch.rand(M, K, generator=torch.Generator().manual_seed(99 + j)) * 2 - 1)
              .half().pin_memory() for j in range(len(GROUPS))]
    c_host = [torch.empty(M, N, dtype=torch.float16).pin_memory() for _ in GROUPS]
    pipe = HostPipeline(dev, M, K, N)
    steps = max(3, args.steps // 2)

    def jobs(n):
        return [(lins[g][0], a_host[j], c_host[j]) for _ in range(n)
                for j, g in enumerate(GROUPS)]

    pipe.run(jobs(max(1, args.warmup))).synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(pipe.compute)
    done = pipe.run(jobs(steps), after=start)
    pipe.compute.wait_event(done)
    stop.record(pipe.compute)
    stop.synchronize()
    ms = start.elapsed_time(stop) / steps
    return {"value": round(sum(flops(M, N, K) for _ in GROUPS) / (ms * 1e-3) / 1e12, 2),
            "unit": UNIT, "h2d_bytes_per_step": len(GROUPS) * M * K * 2,
            "d2h_bytes_per_step": len(GROUPS) * M * N * 2, "ms_per_step": round(ms, 4),
            "path": "HostPipeline -> QuantizedLinear -> launch_final_ws (C ABI i4g_gemm_ws), "
                    "pinned host A and C, copies overlapped on separate streams"}


def run_decode(args, i4g, dev, peaks):
    """Decode-shaped HBM GB/s: M in {1,4,8,16}, g128, both MLP
    shapes, rotating weight sets whose total exceeds L2 (cold weights)."""
    import torch

    stream = torch.cuda.current_stream()
    out = {}
    for (K, N) in ((4096, 14336), (14336, 4096)):
        nsets = 6  # 6 x ~30 MB > 126 MB L2
        gen = torch.Generator(device=dev).manual_seed(4242 + K)
        lins = []
        for _ in range(nsets):
            w = (torch.randn(K, N, generator=gen, device=dev) * 0.02).half()
            lins.append(i4g.QuantizedLinear.from_weight(w, 128))
            del w
        for M in (1, 4, 8, 16):
            a = torch.randn(M, K, generator=gen, device=dev).half()
            c = torch.empty(M, N, dtype=torch.float16, device=dev)
            iters = 120
            for i in range(nsets):
                lins[i % nsets](a, out=c)
            torch.cuda.synchronize()
            # Back-to-back launches captured in one CUDA graph, so the host's
            # per-call cost is not in the device time.
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph, stream=side):
                    for i in range(iters):
                        lins[i % nsets](a, out=c, stream=side)
            torch.cuda.current_stream().wait_stream(side)
            graph.replay()
            torch.cuda.synchronize()
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            graph.replay()
            stop.record(stream)
            torch.cuda.synchronize()
            del graph
            us = start.elapsed_time(stop) * 1e3 / iters
            nbytes = algorithmic_bytes(M, N, K, 128)
            gbs = nbytes / (us * 1e-6) / 1e9
            out[f"M{M}_K{K}_N{N}"] = {"us": round(us, 2), "hbm_gbs": round(gbs, 1),
                                     "frac_hbm": round(gbs / peaks["hbm_gbs"], 3)}
        del lins
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------- CPU reference arm

def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


_CPU_CASES = {}


def _cpu_case(group):
    """Quantised 4096x4096 weight of the CPU arm (built once per group)."""
    import numpy as np

    import oracle

    if group not in _CPU_CASES:
        K, N = K_HEAD, N_HEAD
        rng = np.random.default_rng(5678 + group)
        w = oracle.f2h(rng.standard_normal((K, N)).astype(np.float32) * np.float32(0.02))
        _CPU_CASES[group] = oracle.quantize(w, K, N, group)  # bit-identical to quantize_cpu
    return _CPU_CASES[group]


def cpu_sample(rows, threads, group=128, seed=0):
    """Time the reference's CPU path (oracle/_ref if built, else the oracle
    port) on `rows` rows of the 4096^3 workload: dequantize_cpu of the whole
    weight, then cpu_gemm_fp32 on the row sample. Returns seconds and kind."""
    import numpy as np

    import oracle

    N, K = N_HEAD, K_HEAD
    rng = np.random.default_rng(seed)
    a = oracle.f2h(rng.uniform(-1, 1, (rows, K)).astype(np.float32))
    packed, scales = _cpu_case(group)
    if oracle.ref_available():
        kind = "reference"
        t0 = time.perf_counter()
        deq = oracle.ref_dequantize(packed, scales, K, N, group)
        t1 = time.perf_counter()
        oracle.ref_gemm_rows(a, deq, rows, N, K, threads=threads)
        t2 = time.perf_counter()
    else:
        kind = "port"
        t0 = time.perf_counter()
        deq = oracle.dequantize(packed, scales, K, N, group)
        t1 = time.perf_counter()
        oracle.gemm_rows(a, deq, rows, N, K, threads=threads)
        t2 = time.perf_counter()
    return t1 - t0, t2 - t1, kind


def cpu_baseline(args, sample_rows):
    """The reference's CPU path on a bounded row sample sized to about
    args.cpu_seconds of CPU work: a first sample of `sample_rows` rows
    calibrates the time per row, then the timed sample is taken."""
    threads = _cpu_threads()
    rows = max(sample_rows, threads)
    t_deq, t_rows, kind = cpu_sample(rows, threads)
    per_row = t_rows / rows
    want = max(rows, min(M_HEAD, int((args.cpu_seconds - t_deq) / max(per_row, 1e-9))))
    if want > rows:
        rows = want
        t_deq, t_rows, kind = cpu_sample(rows, threads, seed=1)
    t_full = t_deq + t_rows * (M_HEAD / rows)
    value = flops(M_HEAD, N_HEAD, K_HEAD) / t_full / 1e12
    # the reference as written runs on one thread: a smaller sample of that too
    rows1 = max(1, min(rows, int(0.5 * args.cpu_seconds / max(per_row * threads, 1e-9))))
    t_deq1, t_rows1, _ = cpu_sample(rows1, 1, seed=2)
    t_full1 = t_deq1 + t_rows1 * (M_HEAD / rows1)
    return {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"dequantize_cpu of the 4096x4096 g128 weight + cpu_gemm_fp32 on {rows} "
                      f"of 4096 rows ({threads} threads), extrapolated to the full GEMM",
            "seconds_measured": round(t_deq + t_rows, 3),
            "single_thread": {"value": flops(M_HEAD, N_HEAD, K_HEAD) / t_full1 / 1e12,
                              "unit": UNIT, "cores": 1,
                              "sample": f"the same path on {rows1} rows, one thread",
                              "seconds_measured": round(t_deq1 + t_rows1, 3)}}


def _reference_gpu_worker(q, iters):
    """Child process: the reference's final GPU kernel at the headline shape,
    per group, with rotating inputs as in run_ours (reference layouts made by
    this library's byte-exact quantize and repacks, outside the timing)."""
    import torch

    import oracle
    import sm_120__gemm_b200 as i4g

    R = oracle.ref_final_kernel()
    if R is None:
        q.put({"unavailable": "oracle/_ref/libi4g_reffinal.so not loadable"})
        return
    M, N, K = M_HEAD, N_HEAD, K_HEAD
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1234)
    acts = [(torch.rand(M, K, generator=gen, device=dev) * 2 - 1).half() for _ in range(4)]
    c = torch.empty(M, N, dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream()
    out = {}
    for g in GROUPS:
        sets = []
        for r in range(2):
            w = (torch.randn(K, N, generator=gen, device=dev) * 0.02).half()
            packed = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
            scales = torch.empty(K // g, N, dtype=torch.float16, device=dev)
            i4g.launch_quantize(w, packed, scales, K, N, g)
            b = torch.empty_like(packed)
            (i4g.launch_repack_mma_128x32 if g == 64 else i4g.launch_repack_mma_pair_128x32)(
                packed, b, K, N)
            s = torch.empty_like(scales)
            i4g.launch_repack_scales_128(scales, s, K, N, g)
            sets.append((b, s))

        def call(i):
            b, s = sets[i % 2]
            return R.i4r_launch_final(acts[(3 * i + 1) % 4].data_ptr(), b.data_ptr(), s.data_ptr(),
                                      c.data_ptr(), M, N, K, g, stream.cuda_stream)
        for i in range(3):
            if call(i) != 0:
                q.put({"unavailable": f"reference launch failed (group {g})"})
                return
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(iters)]
        for i, (e0, e1) in enumerate(ev):
            e0.record(stream)
            call(i)
            e1.record(stream)
        torch.cuda.synchronize()
        ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev)
        out[str(g)] = {"kernel_ms": round(ms, 4), "tflops": round(flops(M, N, K) / ms / 1e9, 1)}
    total = sum(v["kernel_ms"] for v in out.values())
    q.put({"per_group": out, "tflops": round(len(GROUPS) * flops(M, N, K) / total / 1e9, 1)})


def reference_gpu_row(iters=20, limit_s=240):
    """Context row (not the arm's value): the reference's own final GPU GEMM
    (kernels/gemm_final.cu:5-13 over kernels/gemm_v17_instruction.cu,
    compiled unmodified for sm_100a by oracle/Makefile) on this box, at the
    headline workload. Its waits are unbounded, so it runs in a child process
    stopped after `limit_s`."""
    import multiprocessing as mp

    import torch
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libi4g_reffinal.so")):
        return {"unavailable": "oracle/_ref/libi4g_reffinal.so not built (needs the reference)"}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_reference_gpu_worker, args=(q, iters))
    p.start()
    p.join(limit_s)
    if p.is_alive():
        p.kill()
        p.join()
        return {"unavailable": f"did not finish within {limit_s} s"}
    if p.exitcode != 0:
        return {"unavailable": f"child exited with {p.exitcode}"}
    row = q.get(timeout=10)
    row["kernel"] = ("the reference's final kernel (V18a g32 / V17b g64 / V18b g128, "
                     "mma.sync + TMA), built for sm_100a from its own source")
    row["inputs"] = ("reference layouts (mma pair / mma fragments, 128-column scales) from "
                     "this library's byte-exact quantize and repacks, outside the timing; "
                     "rotating inputs as in the main arm")
    return row


def run_reference(args):
    """Each step times the reference's CPU path on one bounded sample (one
    group per step, cycling 32/64/128: the full dequantize_cpu plus
    cpu_gemm_fp32 on a row sample); a 3-GEMM step's time is the sum of the
    per-group extrapolated times, averaged over the steps."""
    threads = _cpu_threads()
    rows = max(args.cpu_rows // 2, threads)
    for i in range(args.warmup):
        cpu_sample(threads, threads, group=GROUPS[i % len(GROUPS)], seed=100 + i)
    per_group = {g: [] for g in GROUPS}
    kind = "port"
    for i in range(args.steps):
        g = GROUPS[i % len(GROUPS)]
        t_deq, t_rows, kind = cpu_sample(rows, threads, group=g, seed=i)
        per_group[g].append(t_deq + t_rows * (M_HEAD / rows))
    ms_step = 1e3 * sum(statistics.mean(v) for v in per_group.values() if v) * (
        len(GROUPS) / max(1, sum(1 for v in per_group.values() if v)))
    value = sum(flops(M_HEAD, N_HEAD, K_HEAD) for _ in GROUPS) / (ms_step * 1e-3) / 1e12
    sample = (f"per step: one group's dequantize_cpu of the 4096x4096 weight + cpu_gemm_fp32 "
              f"on {rows} of 4096 rows ({threads} threads), extrapolated to the full GEMM; "
              f"groups cycle 32/64/128")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "reference",
        "data": "synthetic (seeded): A fp16 U[-1,1]; W fp32 N(0,0.02) -> fp16 -> INT4",
        "config": {"workload": WORKLOAD, "M": M_HEAD, "N_per_gpu": N_HEAD, "K": K_HEAD,
                   "groups": list(GROUPS), "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "reference_gpu_kernel": reference_gpu_row() if not args.no_extras else None,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=600)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work of the cpu_baseline sample (rows are chosen to fit it)")
    ap.add_argument("--schedule", choices=["split", "whole"], default="split",
                    help="split: split-K the last partial wave through a workspace; "
                         "whole: whole output tiles only (i4g_gemm)")
    ap.add_argument("--gather", choices=["fused", "nccl", "none"], default="fused",
                    help="at N > 1, how each GEMM's full C reaches every rank")
    ap.add_argument("--extra-iters", type=int, default=10,
                    help="calls timed per shape in the prefill / M-sweep blocks")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the prefill, M-sweep, e2e, decode and cpu-baseline legs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        result = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
