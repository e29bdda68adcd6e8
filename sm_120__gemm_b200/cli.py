"""Command-line harness of the library, mirroring the reference's int4_gemm
binary (src/main.cu:415-439): the same modes and options.

    python -m sm_120__gemm_b200.cli --hardware
    python -m sm_120__gemm_b200.cli --correctness --size 256 --group 32
    python -m sm_120__gemm_b200.cli --fp32-output-check --size 256 --group 64
    python -m sm_120__gemm_b200.cli --benchmark --size 4096 --group all \
        --warmup 20 --iters 100 --csv results.csv
    python -m sm_120__gemm_b200.cli --profile final --size 4096 --group 128 [--m M --n N --k K]
    python -m sm_120__gemm_b200.cli --configs [--iters 50] [--csv configs.csv]

Correctness gates are the reference's (src/main.cu:257-261): against cuBLAS
(torch.matmul) on the GPU-dequantised B, rel_l2 < 0.02 and max_abs < 2.0.
The CSV keeps the reference's 27 columns (src/main.cu:289-295) and appends
gpus, hbm_gbs and frac_peak.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

from . import (QuantizedLinear, launch_dequantize, launch_final, launch_final_fp32, plan,
               launch_inverse_repack_128x32, launch_inverse_repack_umma, launch_quantize,
               launch_repack_128x32, launch_repack_mma_128x32, launch_repack_mma_pair_128x32,
               launch_repack_scales_128, launch_repack_umma, launch_quantize_repack,
               launch_final_ws, workspace_for)

CSV_HEADER = ("version,description,M,N,K,group_size,BM,BN,BK,warp_tile_m,warp_tile_n,stages,"
              "threads,registers_per_thread,smem_bytes,occupancy,cache_mode,median_ms,mean_ms,"
              "min_ms,p95_ms,effective_tflops,speedup_vs_previous,speedup_vs_baseline,"
              "max_abs_error,rmse,notes,gpus,hbm_gbs,frac_peak")


def random_half(shape, seed, lo=-0.5, hi=0.5):
    """Seeded uniform [lo, hi) inputs rounded to fp16 (the distribution of the
    reference harness's random_half, src/main.cu:75-81; torch's generator)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(*shape, generator=g) * (hi - lo) + lo).half()


class Case:
    """Device buffers of one problem (the reference's CaseBuffers, main.cu:117-138)."""

    def __init__(self, M, N, K, group, dev="cuda"):
        self.M, self.N, self.K, self.group = M, N, K, group
        self.a = random_half((M, K), 1234).to(dev)
        self.b = random_half((K, N), 5678).to(dev)
        self.packed = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
        self.scales = torch.empty(K // group, N, dtype=torch.float16, device=dev)
        launch_quantize(self.b, self.packed, self.scales, K, N, group)
        self.lin = QuantizedLinear.from_packed(self.packed, self.scales, K, N, group)
        self.dequant = torch.empty(K, N, dtype=torch.float16, device=dev)
        launch_dequantize(self.packed, self.scales, self.dequant, K, N, group)
        self.c = torch.empty(M, N, dtype=torch.float16, device=dev)
        torch.cuda.synchronize()


def error_metrics(got: torch.Tensor, ref: torch.Tensor):
    d = (got.double() - ref.double()).abs()
    rs = (ref.double() ** 2).sum().item()
    se = (d ** 2).sum().item()
    return {"max_abs": d.max().item(), "mean_abs": d.mean().item(),
            "rmse": math.sqrt(se / d.numel()), "rel_l2": math.sqrt(se / max(rs, 1e-30))}


def validate_repack(x: Case):
    """Round trips of every layout (the GPU half of main.cu:140-208)."""
    K, N, g = x.K, x.N, x.group
    tile = torch.empty_like(x.packed)
    rsc = torch.empty(K // g * N, dtype=torch.float16, device="cuda")
    launch_repack_128x32(x.packed, x.scales, tile, rsc, K, N, g)
    inv = torch.empty_like(x.packed)
    launch_inverse_repack_128x32(tile, inv, K, N)
    back = torch.empty_like(x.packed)
    launch_inverse_repack_umma(x.lin.tiles, back, K, N)
    torch.cuda.synchronize()
    if not torch.equal(inv, x.packed):
        raise RuntimeError("GPU repack inverse test failed")
    if not torch.equal(back, x.packed):
        raise RuntimeError("GPU tile-layout inverse test failed")


def cublas_ref(x: Case, fp32=False):
    if fp32:
        return torch.matmul(x.a.float(), x.dequant.float())
    return torch.matmul(x.a, x.dequant)


def correctness(size, group, m=None, n=None, k=None):
    M, N, K = m or size, n or size, k or size
    print(f"correctness M={M} N={N} K={K} group={group}")
    x = Case(M, N, K, group)
    validate_repack(x)
    ref = cublas_ref(x)
    launch_final(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, group)
    torch.cuda.synchronize()
    e = error_metrics(x.c, ref)
    ok = e["rel_l2"] < 0.02 and e["max_abs"] < 2.0
    print(f"final max_abs={e['max_abs']} mean_abs={e['mean_abs']} rmse={e['rmse']} "
          f"rel_l2={e['rel_l2']} {'PASS' if ok else 'FAIL'}")
    if not ok:
        raise RuntimeError("final correctness failed")


def fp32_output_check(size, group):
    x = Case(size, size, size, group)
    validate_repack(x)
    ref = cublas_ref(x, fp32=True)
    got = torch.empty(size, size, dtype=torch.float32, device="cuda")
    launch_final_fp32(x.a, x.lin.tiles, x.lin.scales, got, size, size, size, group)
    torch.cuda.synchronize()
    e = error_metrics(got, ref)
    print(f"fp32_output size={size} group={group} max_abs={e['max_abs']} "
          f"mean_abs={e['mean_abs']} rmse={e['rmse']} rel_l2={e['rel_l2']}")
    if e["rel_l2"] >= 0.02 or e["max_abs"] >= 2.0:
        raise RuntimeError("FP32 output correctness failed")


def timing(fn, warmup, iters, flush=None):
    """CUDA-event timing: median / mean / min / p95 (include/benchmark.cuh:11-35).
    With `flush`, an L2-sized write runs before each (untimed) launch."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b.record()
        fn()
        e.record()
        e.synchronize()
        times.append(b.elapsed_time(e))
    times.sort()
    p95 = times[min(len(times) - 1, int(math.ceil(len(times) * 0.95)) - 1)]
    return {"median_ms": times[len(times) // 2], "mean_ms": sum(times) / len(times),
            "min_ms": times[0], "p95_ms": p95}


def peaks():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"]
    return 1590.0, 6650.0


def benchmark(size, groups, warmup, iters, csv_path, m=None, n=None, k=None):
    M, N, K = m or size, n or size, k or size
    pk_tf, pk_bw = peaks()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    trash = torch.empty(2 * l2 // 4, dtype=torch.int32, device="cuda")

    def flush():
        trash.add_(1)

    rows = []

    def tflops(ms):
        return 2.0 * M * N * K / (ms * 1e9)

    for g in groups:
        x = Case(M, N, K, g)
        validate_repack(x)
        nbytes = K * N // 2
        rep = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rsc = torch.empty(K // g * N, dtype=torch.float16, device="cuda")
        tq = timing(lambda: launch_quantize(x.b, x.packed, x.scales, K, N, g), warmup, iters)
        tr = timing(lambda: launch_repack_128x32(x.packed, x.scales, rep, rsc, K, N, g), warmup,
                    iters)
        tmma = timing(lambda: (launch_repack_mma_128x32(x.packed, rep, K, N),
                               launch_repack_scales_128(x.scales, rsc, K, N, g)), warmup, iters)
        tpair = timing(lambda: (launch_repack_mma_pair_128x32(x.packed, rep, K, N),
                                launch_repack_scales_128(x.scales, rsc, K, N, g)), warmup, iters)
        tumma = timing(lambda: (launch_repack_umma(x.packed, rep, K, N),
                                launch_repack_scales_128(x.scales, rsc, K, N, g)), warmup, iters)
        td = timing(lambda: launch_dequantize(x.packed, x.scales, x.dequant, K, N, g), warmup,
                    iters)
        tg = timing(lambda: torch.matmul(x.a, x.dequant, out=x.c), warmup, iters)
        tsep = timing(lambda: (launch_dequantize(x.packed, x.scales, x.dequant, K, N, g),
                               torch.matmul(x.a, x.dequant, out=x.c)), warmup, iters)

        def e2e():
            launch_quantize(x.b, x.packed, x.scales, K, N, g)
            launch_repack_umma(x.packed, rep, K, N)
            launch_repack_scales_128(x.scales, rsc, K, N, g)
            launch_final(x.a, rep, rsc, x.c, M, N, K, g)

        te2e = timing(e2e, warmup, iters)
        tqr = timing(lambda: launch_quantize_repack(x.b, rep, rsc, K, N, g), warmup, iters)

        def e2e_fused():
            launch_quantize_repack(x.b, rep, rsc, K, N, g)
            launch_final(x.a, rep, rsc, x.c, M, N, K, g)

        te2e_fused = timing(e2e_fused, warmup, iters)
        ref = cublas_ref(x)
        launch_final(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, g)
        torch.cuda.synchronize()
        err = error_metrics(x.c, ref)
        if err["rel_l2"] >= 0.02 or err["max_abs"] >= 2.0:
            raise RuntimeError("final benchmark correctness failed")
        tf = timing(lambda: launch_final(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, g), warmup,
                    iters)
        tcold = timing(lambda: launch_final(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, g),
                       warmup, iters, flush=flush)
        print(f"group={g} quant={tq['median_ms']:.4f}ms repack={tr['median_ms']:.4f}ms "
              f"mma_repack={tmma['median_ms']:.4f}ms pair_repack={tpair['median_ms']:.4f}ms "
              f"umma_repack={tumma['median_ms']:.4f}ms dequant={td['median_ms']:.4f}ms "
              f"cublas={tg['median_ms']:.4f}ms separate_total={tsep['median_ms']:.4f}ms "
              f"quantize_repack={tqr['median_ms']:.4f}ms end_to_end={te2e['median_ms']:.4f}ms "
              f"end_to_end_fused={te2e_fused['median_ms']:.4f}ms final={tf['median_ms']:.4f}ms "
              f"({tflops(tf['median_ms']):.1f} TFLOP/s) final_cold={tcold['median_ms']:.4f}ms")

        def row(version, desc, cache, t, notes="", tfl=0.0, err_=None, hbm=0.0):
            frac = tfl / pk_tf if tfl else (hbm / pk_bw if hbm else 0.0)
            e = err_ or {"max_abs": -1, "rmse": -1}
            return (f"{version},\"{desc}\",{M},{N},{K},{g},0,0,0,0,0,0,0,-1,0,-1,{cache},"
                    f"{t['median_ms']:.6f},{t['mean_ms']:.6f},{t['min_ms']:.6f},"
                    f"{t['p95_ms']:.6f},{tfl:.3f},0,0,{e['max_abs']},{e['rmse']},\"{notes}\","
                    f"1,{hbm:.1f},{frac:.4f}")

        def gbs(t, b):
            return b / (t["median_ms"] * 1e-3) / 1e9

        rows += [
            row("quantize", "GPU symmetric group quantization", "preprocess", tq,
                "bit-identical to quantize_cpu", hbm=gbs(tq, 2 * K * N + K * N // 2)),
            row("repack", "CTA tile-contiguous BN128 BK32", "preprocess", tr),
            row("repack_mma", "lane-native MMA fragments + tile-contiguous scales",
                "preprocess", tmma),
            row("repack_mma_pair", "two k16 fragments per uint32 + tile-contiguous scales",
                "preprocess", tpair),
            row("repack_umma", "sm_100a tile layout (128 cols x 64 k) + scales", "preprocess",
                tumma),
            row("quantize_repack", "one-pass quantize into the sm_100a tile + scale layouts",
                "preprocess", tqr, "bytes identical to quantize + repack_umma + scales",
                hbm=gbs(tqr, 2 * K * N + K * N // 2 + 2 * N * (K // g))),
            row("end_to_end", "quantize + tile repack + fused final GEMM", "one-shot", te2e,
                "preprocessing is normally amortized", tfl=tflops(te2e["median_ms"])),
            row("end_to_end_fused", "one-pass quantize_repack + fused final GEMM", "one-shot",
                te2e_fused, "preprocessing is normally amortized",
                tfl=tflops(te2e_fused["median_ms"])),
            row("dequant", "materialize packed INT4 B as FP16", "baseline-component", td),
            row("cublas_fp16", "cuBLAS FP16 on dequantized B", "steady", tg,
                "not workload-equivalent: B already materialized", tfl=tflops(tg["median_ms"])),
            row("separate", "dequant kernel + cuBLAS", "steady", tsep,
                tfl=tflops(tsep["median_ms"])),
            row("final", "tcgen05 TMEM fused W4A16 (sm_100a)", "steady", tf,
                tfl=tflops(tf["median_ms"]), err_=err),
            row("final_cold", "tcgen05 TMEM fused W4A16 (sm_100a)", "cold", tcold,
                f"{2 * l2 >> 20} MiB L2 flush before each untimed launch",
                tfl=tflops(tcold["median_ms"]), err_=err),
        ]
        del x
        torch.cuda.empty_cache()
    if csv_path:
        d = os.path.dirname(csv_path)
        if d:
            os.makedirs(d, exist_ok=True)
        with open(csv_path, "w") as f:
            f.write(CSV_HEADER + "\n")
            for r in rows:
                f.write(r + "\n")


def profile_one(size, group, version, m=None, n=None, k=None, launches=1, warmup=10):
    """10 warm-ups, then `launches` launches of one kernel between
    cudaProfilerStart/Stop (main.cu:397-410), for ncu --profile-from-start off
    or -k/-s/-c selection."""
    M, N, K = m or size, n or size, k or size
    x = Case(M, N, K, group)
    if version == "final":
        fn = lambda: launch_final(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, group)  # noqa
    elif version == "final_ws":
        ws = workspace_for(M, N, K)
        fn = lambda: launch_final_ws(x.a, x.lin.tiles, x.lin.scales, x.c, M, N, K, group, ws)  # noqa
    elif version == "quantize_repack":
        fn = lambda: launch_quantize_repack(x.b, x.lin.tiles, x.lin.scales, K, N, group)  # noqa
    elif version == "quantize":
        fn = lambda: launch_quantize(x.b, x.packed, x.scales, K, N, group)  # noqa
    elif version == "repack_umma":
        fn = lambda: launch_repack_umma(x.packed, x.lin.tiles, K, N)  # noqa
    elif version == "dequant":
        fn = lambda: launch_dequantize(x.packed, x.scales, x.dequant, K, N, group)  # noqa
    else:
        raise RuntimeError(f"unknown profile kernel: {version}")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(launches):
        fn()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"profiled {version} M={M} N={N} K={K} group={group}")


def config_shapes():
    """The shapes of the benchmark configurations on one GPU (a rank's slice
    for the column-parallel ones): decode MLP linears, the 70B-class prefill
    up-projection at G = 1/2/4/8, and the M sweep of the fused gate+up
    projection (one of 8 ranks: N = 57344 / 8)."""
    out = []
    for (K, N) in ((4096, 14336), (14336, 4096)):
        for M in (1, 4, 8, 16):
            out.append(("decode", M, N, K, 128))
    for G in (1, 2, 4, 8):
        out.append((f"prefill G={G}", 8192, 28672 // G, 8192, 128))
    for M in (1, 16, 128, 1024, 4096, 16384):
        out.append(("m-sweep rank 1/8", M, 7168, 8192, 64))
    return out


def configs(iters, csv_path=""):
    """Per shape: the kernel the dispatcher picks, the tcgen05 schedule, and
    the device time per call through QuantizedLinear (split-K workspace
    included), from a CUDA graph of back-to-back calls that rotate enough
    weight and activation sets to keep their operands out of L2."""
    pk_tf, pk_bw = peaks()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    lines = ["config,M,N,K,group,kernel,schedule,us_per_call,tflops,algorithmic_gbs,"
             "frac_tensor,frac_hbm"]
    import time
    for (label, M, N, K, g) in config_shapes():
        # let clocks and power recover from the previous row (the prefill
        # rows run the GPU at its power cap for a third of a second)
        time.sleep(1.0)
        wbytes = K * N // 2
        nw = max(1, min(8, -(-2 * l2 // wbytes)))
        na = max(1, min(4, -(-2 * l2 // (2 * M * K))))
        gen = torch.Generator(device="cuda").manual_seed(M * 131 + N * 7 + K)
        lins = []
        for _ in range(nw):
            w = (torch.randn(K, N, generator=gen, device="cuda") * 0.02).half()
            lins.append(QuantizedLinear.from_weight(w, g))
            del w
        acts = [(torch.rand(M, K, generator=gen, device="cuda") * 2 - 1).half() for _ in range(na)]
        c = torch.empty(M, N, dtype=torch.float16, device="cuda")
        ws = workspace_for(M, N, K)
        side = torch.cuda.Stream()
        for i in range(max(nw, na)):
            lins[i % nw](acts[i % na], out=c)
        torch.cuda.synchronize()
        ws = workspace_for(M, N, K, stream=side)
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                for i in range(iters):
                    lins[i % nw](acts[i % na], out=c, stream=side)
        torch.cuda.current_stream().wait_stream(side)
        graph.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b.record()
            graph.replay()
            e.record()
            e.synchronize()
            best = min(best, b.elapsed_time(e) * 1e3 / iters)
        del graph
        flops = 2.0 * M * N * K
        nbytes = 2 * M * K + K * N // 2 + 2 * N * (K // g) + 2 * M * N
        tf = flops / (best * 1e-6) / 1e12
        gbs = nbytes / (best * 1e-6) / 1e9
        # the kernel and schedule these calls ran (the planners, via i4g_plan)
        info = plan(M, N, K, g, torch.cuda.get_device_properties(0).multi_processor_count,
                    0 if ws is None else ws.numel())
        kernel = info["kernel"]
        sched = f'{info["schedule"]} ({info["param"]})'
        lines.append(f"{label},{M},{N},{K},{g},{kernel},{sched},{best:.2f},{tf:.1f},{gbs:.0f},"
                     f"{tf / pk_tf:.3f},{gbs / pk_bw:.3f}")
        print(lines[-1], flush=True)
        del lins, acts, c
        torch.cuda.empty_cache()
    if csv_path:
        with open(csv_path, "w") as f:
            f.write("\n".join(lines) + "\n")


def gather_sweep(iters):
    """The M sweep of the fused gate+up projection (K=8192, N=57344, g64),
    column-parallel over the ranks of a torchrun job, each rank owning
    N / world columns: per M, the GEMM alone and the GEMM plus the NCCL
    all-gather of C (end to end), max over ranks of CUDA-event times."""
    import datetime

    import torch.distributed as dist

    from .sharded import ColumnParallelLinear, PeerOutputs, gather_columns

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    K, N, g = 8192, 57344, 64
    n_local = N // world
    try:
        gen = torch.Generator(device=dev).manual_seed(9000 + rank)
        w = (torch.randn(K, n_local, generator=gen, device=dev) * 0.02).half()
        cp = ColumnParallelLinear(QuantizedLinear.from_weight(w, g), world, rank)
        del w
        if rank == 0:
            print("M,world,kernel,gemm_us,gemm_plus_nccl_gather_us,fused_peer_store_us,"
                  "nccl_gather_share,fused_equals_nccl")
        for M in (1, 16, 128, 1024, 4096, 16384):
            a = (torch.rand(M, K, generator=gen, device=dev) * 2 - 1).half()
            c_local = torch.empty(M, n_local, dtype=torch.float16, device=dev)
            gathered = torch.empty(world * M * n_local, dtype=torch.float16, device=dev)
            out = torch.empty(M, N, dtype=torch.float16, device=dev)

            def gemm():
                cp.forward_local(a, out=c_local)

            def e2e():
                cp.forward_local(a, out=c_local)
                if world > 1:
                    gather_columns(c_local, out=out, gathered=gathered)

            outs = PeerOutputs(M, N, dev) if world > 1 else None

            def fused():
                if outs is not None:
                    cp.forward_to_peers(a, outs)
                else:
                    cp.forward_local(a, out=c_local)

            res = []
            for fn in (gemm, e2e, fused):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                dist.barrier()
                b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                b.record()
                for _ in range(iters):
                    fn()
                e.record()
                e.synchronize()
                t = torch.tensor([b.elapsed_time(e) * 1e3 / iters], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                res.append(float(t.item()))
            # the fused path's C must be the NCCL-gathered C bit for bit, on
            # every rank
            same = torch.ones(1, device=dev)
            if outs is not None:
                e2e()
                fused()
                torch.cuda.synchronize()
                same[0] = float(torch.equal(outs.view(M).view(torch.int16), out.view(torch.int16)))
                dist.all_reduce(same, op=dist.ReduceOp.MIN)
                outs.close()
            if rank == 0:
                kern = "decode" if M <= 16 else "tcgen05"
                print(f"{M},{world},{kern},{res[0]:.2f},{res[1]:.2f},{res[2]:.2f},"
                      f"{(res[1] - res[0]) / res[1]:.3f},{int(same.item())}", flush=True)
            del a, c_local, gathered, out, outs
            torch.cuda.empty_cache()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def hardware():
    print(f"torch {torch.__version__}, CUDA runtime {torch.version.cuda}")
    for d in range(torch.cuda.device_count()):
        p = torch.cuda.get_device_properties(d)
        print(f"GPU {d}: {p.name}\ncompute capability: {p.major}.{p.minor}\n"
              f"SM count: {p.multi_processor_count}\nL2 bytes: {p.L2_cache_size}\n"
              f"global memory bytes: {p.total_memory}")


def main(argv=None):
    ap = argparse.ArgumentParser(prog="int4_gemm")
    mode = ap.add_mutually_exclusive_group()
    mode.add_argument("--hardware", action="store_true")
    mode.add_argument("--correctness", action="store_true")
    mode.add_argument("--fp32-output-check", action="store_true")
    mode.add_argument("--benchmark", action="store_true")
    mode.add_argument("--profile", metavar="VERSION")
    mode.add_argument("--configs", action="store_true")
    mode.add_argument("--gather-sweep", action="store_true")
    ap.add_argument("--size", type=int, default=256)
    ap.add_argument("--group", default="32")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--csv", default="")
    ap.add_argument("--m", type=int)
    ap.add_argument("--n", type=int)
    ap.add_argument("--k", type=int)
    ap.add_argument("--launches", type=int, default=1)
    a = ap.parse_args(argv)
    groups = [32, 64, 128] if a.group == "all" else [int(a.group)]
    try:
        if a.correctness:
            for g in groups:
                correctness(a.size, g, a.m, a.n, a.k)
        elif a.fp32_output_check:
            for g in groups:
                fp32_output_check(a.size, g)
        elif a.benchmark:
            benchmark(a.size, groups, a.warmup, a.iters, a.csv, a.m, a.n, a.k)
        elif a.profile:
            profile_one(a.size, groups[0], a.profile, a.m, a.n, a.k, a.launches)
        elif a.configs:
            configs(a.iters, a.csv)
        elif a.gather_sweep:
            gather_sweep(a.iters)
        else:
            hardware()
    except Exception as e:  # the reference prints ERROR and exits 1 (main.cu:437)
        print(f"ERROR: {e}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
