"""The C-ABI library without a GPU: it loads, exports every entry point that
include/i4g.h declares, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "i4g.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(i4g_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    import sm_120__gemm_b200 as m
    return m.load()


def test_header_declares_entry_points():
    names = declared_functions()
    for expected in ("i4g_quantize", "i4g_dequantize", "i4g_repack_umma", "i4g_gemm",
                     "i4g_gemm_fp32", "i4g_repack_mma_pair_128x32", "i4g_shard_range"):
        assert expected in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings(lib):
    for code in range(0, -10, -1):
        assert lib.i4g_status_string(code)
    assert lib.i4g_layout_version() == 1


def test_argument_checks_need_no_gpu(lib):
    vp = ctypes.c_void_p
    fake = vp(0x1000)  # never dereferenced: checks fail first
    # null pointers
    assert lib.i4g_gemm(None, fake, fake, fake, 64, 128, 128, 64, None) == -1
    # unsupported group (the reference silently used g128 for these)
    for g in (0, 16, 96, 256):
        assert lib.i4g_gemm(fake, fake, fake, fake, 64, 128, 128, g, None) == -3
    # K not a multiple of the group
    assert lib.i4g_gemm(fake, fake, fake, fake, 64, 128, 192, 128, None) == -3
    # shapes
    assert lib.i4g_gemm(fake, fake, fake, fake, 0, 128, 128, 64, None) == -2
    assert lib.i4g_gemm(fake, fake, fake, fake, 64, 100, 128, 64, None) == -2
    assert lib.i4g_gemm(fake, fake, fake, fake, 64, 128, 96, 32, None) == -2
    # alignment
    assert lib.i4g_gemm(vp(0x1002), fake, fake, fake, 64, 128, 128, 64, None) == -4
    # unknown variant / decode beyond M=16
    assert lib.i4g_gemm_variant(fake, fake, fake, fake, 64, 128, 128, 64, 7, None) == -9
    assert lib.i4g_gemm_variant(fake, fake, fake, fake, 17, 128, 128, 64, 2, None) == -9
    # preprocessing shapes
    assert lib.i4g_quantize(fake, fake, fake, 128, 127, 32, None) == -2
    assert lib.i4g_repack_umma(fake, fake, 96, 128, None) == -2
    assert lib.i4g_repack_128x32(fake, fake, fake, fake, 128, 100, 32, None) == -2
    # peer barrier argument checks come before any device access
    flags = (ctypes.c_void_p * 2)(fake, fake)
    assert lib.i4g_peer_barrier(None, flags, 2, 0, 1, 0, None) == -1
    assert lib.i4g_peer_barrier(fake, flags, 9, 0, 1, 0, None) == -2
    assert lib.i4g_peer_barrier(fake, flags, 2, 2, 1, 0, None) == -2
    assert lib.i4g_peer_barrier(fake, flags, 2, 0, 0, 0, None) == -2
    # plan query: no device needed, arguments checked
    k, sch, prm, b = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    ref = [ctypes.byref(x) for x in (k, sch, prm, b)]
    assert lib.i4g_plan(64, 128, 128, 64, 0, 148, 0, None, *ref[1:]) == -1
    assert lib.i4g_plan(64, 100, 128, 64, 0, 148, 0, *ref) == -2
    assert lib.i4g_plan(64, 128, 128, 96, 0, 148, 0, *ref) == -3
    assert lib.i4g_plan(64, 128, 128, 64, 0, 0, 0, *ref) == -2
    assert lib.i4g_plan(64, 128, 128, 64, 0, 148, 0, *ref) == 0
    # decode schedule selector: unknown values are refused, known ones taken
    assert lib.i4g_set_decode_schedule(4) == -9
    assert lib.i4g_set_decode_schedule(-1) == -9
    for mode in (3, 2, 1, 0):
        assert lib.i4g_set_decode_schedule(mode) == 0


def test_shard_range_arithmetic():
    import sm_120__gemm_b200 as m
    K, N, g = 8192, 28672, 128
    for world in (1, 2, 4, 8):
        prev_end = 0
        for rank in range(world):
            toff, soff, n0, n1 = m.shard_range(K, N, g, world, rank)
            assert n0 == prev_end and n1 - n0 == N // world
            assert toff == n0 * K // 2
            assert soff == (n0 // 128) * (K // g) * 128 * 2
            prev_end = n1
        assert prev_end == N
    with pytest.raises(m.I4GError):
        m.shard_range(K, 28672 + 128, g, 8, 0)


def test_cpp_wrappers_compile_and_throw(tmp_path):
    """include/int4gemm.hpp keeps the reference's C++ signatures and turns a
    non-zero status into std::runtime_error (checked without a GPU)."""
    import shutil
    import subprocess
    if shutil.which("g++") is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "t.cpp"
    src.write_text(r'''
#include "int4gemm.hpp"
#include <cstdio>
int main() {
  int4gemm::KernelLaunch fn = &int4gemm::launch_final;  // reference signature
  try { fn(nullptr, nullptr, nullptr, nullptr, 64, 128, 128, 64, nullptr); }
  catch (const std::runtime_error& e) { std::printf("threw: %s\n", e.what()); return 0; }
  return 1;
}
''')
    exe = tmp_path / "t"
    pkg = os.path.join(ROOT, "sm_120__gemm_b200")
    subprocess.run(["g++", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    "-I", "/usr/local/cuda/include", str(src), "-o", str(exe),
                    "-L", pkg, "-li4g", f"-Wl,-rpath,{pkg}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out
    assert "null pointer" in out.stdout


def test_kernel_config_needs_no_gpu():
    import sm_120__gemm_b200 as m
    c = m.kernel_config(m.VARIANT_TC, 256, 128)
    assert (c["rows"], c["cols"], c["bk"], c["mma_m"], c["mma_n"]) == (256, 128, 64, 128, 256)
    assert c["threads"] == 736 and 0 < c["dynamic_smem_bytes"] <= 232448
    d = m.kernel_config(m.VARIANT_DECODE, 16, 64)
    assert d["rows"] == 16 and d["cols"] == 128 and d["stages"] >= 2
    with pytest.raises(m.I4GError):
        m.kernel_config(m.VARIANT_TC, 64, 128)
    with pytest.raises(m.I4GError):
        m.kernel_config(m.VARIANT_DECODE, 8, 96)


def test_cpp_registry_matches_the_reference_interface(tmp_path):
    """kernel_registry() / KernelMetadata / query_resources() of
    include/int4gemm.hpp, used the way the reference's harness uses them
    (src/main.cu:247-249, 349-377); without a GPU the resource query throws."""
    import shutil
    import subprocess
    if shutil.which("g++") is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "r.cpp"
    src.write_text(r'''
#include "int4gemm.hpp"
#include <cstdio>
int main() {
  using namespace int4gemm;
  auto reg = kernel_registry();
  if (reg.size() != 1) return 2;
  const KernelMetadata& md = reg[0].first;
  KernelLaunch fn = reg[0].second;
  std::printf("%s BM=%d BN=%d BK=%d mma=%dx%d stages=%d threads=%d smem=%d\n", md.version,
              md.BM, md.BN, md.BK, md.warp_m, md.warp_n, md.stages, md.threads, md.smem_bytes);
  if (fn != &launch_final) return 3;
  try { KernelResources r = query_resources(md.version, 128); (void)r; }
  catch (const std::runtime_error& e) { std::printf("resources threw\n"); }
  try { query_resources("v17b", 128); return 4; } catch (const std::runtime_error&) {}
  return 0;
}
''')
    exe = tmp_path / "r"
    pkg = os.path.join(ROOT, "sm_120__gemm_b200")
    subprocess.run(["g++", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    "-I", "/usr/local/cuda/include", str(src), "-o", str(exe),
                    "-L", pkg, "-li4g", f"-Wl,-rpath,{pkg}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out
    assert out.stdout.startswith("final BM=256 BN=128 BK=64 mma=128x256"), out.stdout


def _reference_checkout():
    import json
    path = os.environ.get("I4G_REFERENCE")
    if not path:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            path = json.load(f).get("reference_path")
    return path if path and os.path.isfile(os.path.join(path, "src", "main.cu")) else None


def test_reference_harness_builds_against_the_library(tmp_path):
    """The reference's own harness (src/main.cu, with the one documented
    layout change of oracle/harness_patch.py) and its CPU checker compile and
    link against include/reference_compat + include/int4gemm.hpp +
    libi4g.so. Needs the reference checkout (skipped where it is absent)."""
    import subprocess
    ref = _reference_checkout()
    if ref is None:
        pytest.skip("reference checkout not present")
    out = tmp_path / "int4_gemm"
    r = subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "harness", f"REF={ref}",
                        f"HARNESS_OUT={out}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert out.exists()
    patched = open(f"{out}_main.cu").read()
    original = open(os.path.join(ref, "src", "main.cu")).read()
    # the patch only adds lines or swaps a repack call for the tile repack
    assert patched.count("use_tile_layout(x);") == 4
    assert len(patched.splitlines()) - len(original.splitlines()) == 12
