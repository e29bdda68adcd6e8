"""The reference's own harness and this library's CLI, on a GPU.

oracle/_ref/int4_gemm is the reference's src/main.cu (with the one layout
change of oracle/harness_patch.py) and its CPU checker, built against
include/reference_compat + int4gemm.hpp + libi4g.so on the build machine; it
runs its own correctness gates (src/main.cu:226-280: rel_l2 < 0.02 and
max_abs < 2.0 against cuBLAS, and at size <= 256 the CPU fp32 path) on this
library's "final". The CLI (sm_120__gemm_b200.cli) mirrors the same modes.
"""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

HARNESS = os.path.join(ROOT, "oracle", "_ref", "int4_gemm")


def _needs_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")


@pytest.mark.parametrize("group", [32, 64, 128])
def test_reference_harness_correctness(group):
    _needs_gpu()
    if not os.path.exists(HARNESS):
        pytest.skip("reference harness not built (needs the reference checkout)")
    r = subprocess.run([HARNESS, "--correctness", "--size", "256", "--group", str(group)],
                       capture_output=True, text=True, timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "cpu_fp32_vs_cublas" in r.stdout
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("final ")]
    assert len(lines) == 1 and lines[0].endswith("PASS"), r.stdout


@pytest.mark.parametrize("group", [32, 128])
def test_reference_harness_fp32_output(group):
    _needs_gpu()
    if not os.path.exists(HARNESS):
        pytest.skip("reference harness not built (needs the reference checkout)")
    r = subprocess.run([HARNESS, "--fp32-output-check", "--size", "256", "--group", str(group)],
                       capture_output=True, text=True, timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "fp32_output size=256" in r.stdout


def _cli(*args):
    r = subprocess.run([sys.executable, "-m", "sm_120__gemm_b200.cli", *args], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr)
    return r


def test_cli_correctness_all_groups():
    _needs_gpu()
    r = _cli("--correctness", "--size", "256", "--group", "all")
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("final ")]
    assert len(lines) == 3 and all(ln.endswith("PASS") for ln in lines), r.stdout


def test_cli_correctness_decode_shape():
    _needs_gpu()
    r = _cli("--correctness", "--group", "128", "--m", "4", "--n", "4096", "--k", "4096")
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr


def test_cli_fp32_output_check():
    _needs_gpu()
    r = _cli("--fp32-output-check", "--size", "512", "--group", "64")
    assert r.returncode == 0 and "fp32_output size=512" in r.stdout, r.stdout + r.stderr


def test_cli_benchmark_writes_the_reference_csv(tmp_path):
    _needs_gpu()
    csv = tmp_path / "b.csv"
    r = _cli("--benchmark", "--size", "1024", "--group", "64", "--warmup", "2", "--iters", "5",
             "--csv", str(csv))
    assert r.returncode == 0, r.stdout + r.stderr
    rows = csv.read_text().splitlines()
    header = rows[0].split(",")
    assert header[:27] == ("version,description,M,N,K,group_size,BM,BN,BK,warp_tile_m,"
                           "warp_tile_n,stages,threads,registers_per_thread,smem_bytes,"
                           "occupancy,cache_mode,median_ms,mean_ms,min_ms,p95_ms,"
                           "effective_tflops,speedup_vs_previous,speedup_vs_baseline,"
                           "max_abs_error,rmse,notes").split(",")
    versions = [ln.split(",")[0] for ln in rows[1:]]
    for v in ("quantize", "dequant", "cublas_fp16", "separate", "final"):
        assert v in versions, versions


def test_kernel_resources_on_the_device():
    _needs_gpu()
    import sm_120__gemm_b200 as m
    for variant, rows in ((m.VARIANT_TC, 256), (m.VARIANT_TC, 128), (m.VARIANT_DECODE, 8),
                          (m.VARIANT_DECODE, 16)):
        for g in (32, 64, 128):
            r = m.kernel_resources(variant, rows, g)
            c = m.kernel_config(variant, rows, g)
            print(variant, rows, g, r, c)
            assert 0 < r["registers_per_thread"] <= 255
            assert r["max_threads_per_block"] >= c["threads"]
            assert r["active_blocks_per_sm"] == (1 if variant == m.VARIANT_TC else 2)
