"""CPU oracle for the fused W4A16 INT4 GEMM path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` import this package: it is the checker, never the thing measured
or shipped. It binds two shared libraries with ctypes:

* ``liboracle.so``: the C restatement in ``oracle.c`` of the reference's CPU
  path (``src/reference.cu:6-64``) and of its weight layouts
  (``include/layout.cuh:8-48``, ``src/main.cu:140-208``).
* ``_ref/libi4g_ref.so``: ``ref_shim.cu`` compiled together with the
  reference's unmodified ``src/reference.cu`` (built only where the reference
  checkout exists; optional elsewhere).
* ``_ref/libi4g_refquant.so``: the reference's own GPU quantizer
  (``src/quantize.cu``) with its fast-math build flag, to measure where it
  departs from ``quantize_cpu`` (device pointers; needs a GPU to run).

Half-precision arrays travel as ``numpy.uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REF_LIB = os.path.join(HERE, "_ref", "libi4g_ref.so")
_lock = threading.Lock()
_lib = None
_ref = None

_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int


class ErrorMetrics(ctypes.Structure):
    _fields_ = [("max_abs", ctypes.c_double), ("mean_abs", ctypes.c_double),
                ("rmse", ctypes.c_double), ("relative_l2", ctypes.c_double)]


def build(ref_path: str | None = None) -> None:
    """Compile liboracle.so, and the reference checker (oracle/_ref) from the
    reference checkout at `ref_path` (default: the I4G_REFERENCE environment
    variable) when one is given and present."""
    subprocess.run(["make", "-C", HERE, "all"], check=True,
                   stdout=subprocess.DEVNULL)
    ref_src = ref_path or os.environ.get("I4G_REFERENCE")
    if ref_src and os.path.isfile(os.path.join(ref_src, "src", "reference.cu")):
        subprocess.run(["make", "-C", HERE, "ref", f"REF={ref_src}"], check=True,
                       stdout=subprocess.DEVNULL)
        # the reference's harness on this library (needs libi4g.so built)
        if os.path.exists(os.path.join(os.path.dirname(HERE), "sm_120__gemm_b200", "libi4g.so")):
            subprocess.run(["make", "-C", HERE, "harness", f"REF={ref_src}"], check=True,
                           stdout=subprocess.DEVNULL)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB):
                build()
            L = ctypes.CDLL(_LIB)
            L.i4o_h2f.restype = ctypes.c_float
            L.i4o_h2f.argtypes = [ctypes.c_uint16]
            L.i4o_f2h.restype = ctypes.c_uint16
            L.i4o_f2h.argtypes = [ctypes.c_float]
            L.i4o_sign_extend.restype = _i
            L.i4o_sign_extend.argtypes = [ctypes.c_uint8]
            L.i4o_h2f_array.argtypes = [_u16p, _f32p, ctypes.c_size_t]
            L.i4o_f2h_array.argtypes = [_f32p, _u16p, ctypes.c_size_t]
            L.i4o_quantize.argtypes = [_u16p, _u8p, _u16p, _i, _i, _i]
            L.i4o_dequantize.argtypes = [_u8p, _u16p, _u16p, _i, _i, _i]
            L.i4o_gemm_rows.argtypes = [_u16p, _u16p, _f32p, _i, _i, _i, _i, _i]
            L.i4o_gemm_rows_fb.argtypes = [_u16p, _f32p, _f32p, _i, _i, _i, _i, _i]
            L.i4o_gemm_rows_fb_noise.argtypes = [_u16p, _f32p, _f32p,
                                                 ctypes.POINTER(ctypes.c_double),
                                                 _i, _i, _i, _i, _i]
            L.i4o_gemm_rows_f64.argtypes = [_u16p, _f32p, ctypes.POINTER(ctypes.c_double),
                                            _i, _i, _i, _i, _i]
            L.i4o_abs_gemm_rows.argtypes = [_u16p, _u16p, _f32p, _i, _i, _i, _i, _i]
            L.i4o_compare_half.restype = ErrorMetrics
            L.i4o_compare_half.argtypes = [_u16p, _u16p, ctypes.c_size_t]
            L.i4o_ulp_distance.restype = _i
            L.i4o_ulp_distance.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
            for name in ("i4o_repack_128x32", "i4o_inverse_repack_128x32",
                         "i4o_repack_mma_128x32", "i4o_repack_mma_pair_128x32",
                         "i4o_repack_umma", "i4o_inverse_repack_umma"):
                getattr(L, name).argtypes = [_u8p, _u8p, _i, _i]
            L.i4o_repack_scales_128.argtypes = [_u16p, _u16p, _i, _i, _i]
            L.i4o_umma_nibble_index.restype = ctypes.c_size_t
            L.i4o_umma_nibble_index.argtypes = [_i, _i, _i]
            _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_LIB)


def ref_lib():
    """The reference's own CPU path (oracle/_ref); raises if it was not built."""
    global _ref
    with _lock:
        if _ref is None:
            if not os.path.exists(_REF_LIB):
                raise FileNotFoundError(f"{_REF_LIB} not built (make -C oracle ref)")
            R = ctypes.CDLL(_REF_LIB)
            R.i4r_quantize.argtypes = [_u16p, _u8p, _u16p, _i, _i, _i]
            R.i4r_dequantize.argtypes = [_u8p, _u16p, _u16p, _i, _i, _i]
            R.i4r_gemm_rows.argtypes = [_u16p, _u16p, _f32p, _i, _i, _i, _i, _i, _i]
            R.i4r_compare_half.argtypes = [_u16p, _u16p, ctypes.c_size_t,
                                           ctypes.POINTER(ctypes.c_double)]
            R.i4r_f2h.restype = ctypes.c_uint16
            R.i4r_f2h.argtypes = [ctypes.c_float]
            R.i4r_h2f.restype = ctypes.c_float
            R.i4r_h2f.argtypes = [ctypes.c_uint16]
            R.i4r_random_half.argtypes = [_u16p, ctypes.c_size_t, ctypes.c_uint64]
            for name in ("i4r_repack_128x32", "i4r_repack_mma_128x32",
                         "i4r_repack_mma_pair_128x32"):
                getattr(R, name).argtypes = [_u8p, _u8p, _i, _i]
            R.i4r_repack_scales_128.argtypes = [_u16p, _u16p, _i, _i, _i]
            _ref = R
    return _ref


_REFQ_LIB = os.path.join(HERE, "_ref", "libi4g_refquant.so")
_REFF_LIB = os.path.join(HERE, "_ref", "libi4g_reffinal.so")
_refq = None
_reff = None


def ref_gpu_quantizer():
    """The reference's GPU launch_quantize (fast-math build), as
    i4r_gpu_quantize(b, packed, scales, K, N, group, stream) on device
    pointers; None when it was not built."""
    global _refq
    with _lock:
        if _refq is None and os.path.exists(_REFQ_LIB):
            R = ctypes.CDLL(_REFQ_LIB)
            R.i4r_gpu_quantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           _i, _i, _i, ctypes.c_void_p]
            R.i4r_gpu_quantize.restype = _i
            _refq = R
    return _refq


def ref_final_kernel():
    """The reference's own final GPU GEMM (kernels/gemm_final.cu:5-13 over
    kernels/gemm_v17_instruction.cu, built for sm_100a), as
    i4r_launch_final(a, b, scales, c, M, N, K, group, stream) on device
    pointers in the reference's layouts; None when it was not built or no
    CUDA driver is present. Its
    waits are unbounded: run it under a host timeout."""
    global _reff
    with _lock:
        if _reff is None and os.path.exists(_REFF_LIB):
            try:
                R = ctypes.CDLL(_REFF_LIB)
            except OSError:  # no CUDA driver here (a CPU-only machine)
                return None
            R.i4r_launch_final.argtypes = [ctypes.c_void_p] * 4 + [_i] * 4 + [ctypes.c_void_p]
            R.i4r_launch_final.restype = _i
            _reff = R
    return _reff


def _p(arr, ptype):
    assert arr.flags["C_CONTIGUOUS"]
    return arr.ctypes.data_as(ptype)


def _u16(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


# ---------------------------------------------------------------- restatement

def f2h(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().i4o_f2h_array(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


def h2f(h) -> np.ndarray:
    h = _u16(h)
    out = np.empty(h.shape, np.float32)
    lib().i4o_h2f_array(_p(h, _u16p), _p(out, _f32p), h.size)
    return out


def quantize(b, K: int, N: int, group: int):
    """quantize_cpu (src/reference.cu:6-26): (packed uint8[K*N/2], scales u16[G,N])."""
    b = _u16(b)
    groups = (K + group - 1) // group
    packed = np.zeros(K * N // 2, np.uint8)
    scales = np.zeros((groups, N), np.uint16)
    lib().i4o_quantize(_p(b, _u16p), _p(packed, _u8p), _p(scales, _u16p), K, N, group)
    return packed, scales


def dequantize(packed, scales, K: int, N: int, group: int) -> np.ndarray:
    """dequantize_cpu (src/reference.cu:28-37): fp16 bits [K, N]."""
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = _u16(scales)
    out = np.empty((K, N), np.uint16)
    lib().i4o_dequantize(_p(packed, _u8p), _p(scales, _u16p), _p(out, _u16p), K, N, group)
    return out


def widen(b16) -> np.ndarray:
    """FP16 bit patterns -> flat binary32 array (exact), for reuse across calls."""
    return h2f(_u16(b16)).reshape(-1)


def _rows_parallel(fn, n_rows, threads):
    if threads <= 1 or n_rows <= 1:
        fn(0, n_rows)
        return
    chunks = np.array_split(np.arange(n_rows), threads)
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda c: fn(int(c[0]), int(c[-1]) + 1) if len(c) else None, chunks))


def gemm_rows(a, b16, M: int, N: int, K: int, rows=None, threads: int = 1,
              bf=None) -> np.ndarray:
    """cpu_gemm_fp32 (src/reference.cu:55-64) on the given A rows: fp32 [len(rows), N].

    ``rows`` is a range/array of row indices (default: all). Rows are
    independent, so they are split over ``threads`` host threads. ``bf`` is
    ``widen(b16)`` when the caller already has it.
    """
    a = _u16(a)
    bf = widen(b16) if bf is None else bf
    idx = np.arange(M) if rows is None else np.asarray(rows)
    out = np.empty((len(idx), N), np.float32)
    L = lib()

    def run(lo, hi):
        for j in range(lo, hi):
            L.i4o_gemm_rows_fb(_p(a, _u16p), _p(bf, _f32p),
                               out[j].ctypes.data_as(_f32p), M, N, K, int(idx[j]), 1)

    _rows_parallel(run, len(idx), threads)
    return out


def gemm_rows_noise(a, b16, M: int, N: int, K: int, rows=None, threads: int = 1, bf=None):
    """cpu_gemm_fp32 on the given rows (as gemm_rows) and, per output, the
    FP32 summation-noise scale 2^-24 * sqrt(sum_k p_k^2) of its running
    partial sums p_k: (fp32 [rows, N], float64 [rows, N])."""
    a = _u16(a)
    bf = widen(b16) if bf is None else bf
    idx = np.arange(M) if rows is None else np.asarray(rows)
    out = np.empty((len(idx), N), np.float32)
    p2 = np.empty((len(idx), N), np.float64)
    L = lib()
    dp = ctypes.POINTER(ctypes.c_double)

    def run(lo, hi):
        for j in range(lo, hi):
            L.i4o_gemm_rows_fb_noise(_p(a, _u16p), _p(bf, _f32p), out[j].ctypes.data_as(_f32p),
                                     p2[j].ctypes.data_as(dp), M, N, K, int(idx[j]), 1)

    _rows_parallel(run, len(idx), threads)
    return out, 2.0**-24 * np.sqrt(p2)


def gemm_rows_f64(a, b16, M: int, N: int, K: int, rows=None, threads: int = 1,
                  bf=None) -> np.ndarray:
    """The exact result of the same operands for the given A rows: FP16 x FP16
    products (exact in binary64) summed in binary64, float64 [len(rows), N].
    Rounded once to FP16 (``f64_to_h``) it is the best FP16 answer, the anchor
    the GEMM parity gate measures both this library and the reference from."""
    a = _u16(a)
    bf = widen(b16) if bf is None else bf
    idx = np.arange(M) if rows is None else np.asarray(rows)
    out = np.empty((len(idx), N), np.float64)
    L = lib()
    dp = ctypes.POINTER(ctypes.c_double)

    def run(lo, hi):
        for j in range(lo, hi):
            L.i4o_gemm_rows_f64(_p(a, _u16p), _p(bf, _f32p), out[j].ctypes.data_as(dp),
                                M, N, K, int(idx[j]), 1)

    _rows_parallel(run, len(idx), threads)
    return out


def f64_to_h(x) -> np.ndarray:
    """binary64 -> FP16 bit patterns, rounded once to nearest even."""
    return np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float16)).view(np.uint16)


def abs_gemm_rows(a, b16, M: int, N: int, K: int, rows=None) -> np.ndarray:
    """Per-output sum of |a|*|b| for the given rows (error-bound helper)."""
    a = _u16(a)
    b16 = _u16(b16)
    idx = np.arange(M) if rows is None else np.asarray(rows)
    out = np.empty((len(idx), N), np.float32)
    L = lib()
    for j, r in enumerate(idx):
        L.i4o_abs_gemm_rows(_p(a, _u16p), _p(b16, _u16p),
                            out[j].ctypes.data_as(_f32p), M, N, K, int(r), 1)
    return out


def compare_half(got, ref) -> ErrorMetrics:
    got = _u16(got)
    ref = _u16(ref)
    assert got.size == ref.size
    return lib().i4o_compare_half(_p(got, _u16p), _p(ref, _u16p), got.size)


def ulp_distance(a, b) -> np.ndarray:
    """Vectorised ordered-integer distance between half bit patterns."""
    a = _u16(a).astype(np.int32)
    b = _u16(b).astype(np.int32)
    oa = np.where(a & 0x8000, -(a & 0x7FFF), a)
    ob = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(oa - ob)


def _layout(name, packed, K, N):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.zeros(K * N // 2, np.uint8)
    getattr(lib(), name)(_p(packed, _u8p), _p(out, _u8p), K, N)
    return out


def repack_128x32(packed, K, N):
    return _layout("i4o_repack_128x32", packed, K, N)


def inverse_repack_128x32(repacked, K, N):
    return _layout("i4o_inverse_repack_128x32", repacked, K, N)


def repack_mma_128x32(packed, K, N):
    return _layout("i4o_repack_mma_128x32", packed, K, N)


def repack_mma_pair_128x32(packed, K, N):
    return _layout("i4o_repack_mma_pair_128x32", packed, K, N)


def repack_umma(packed, K, N):
    return _layout("i4o_repack_umma", packed, K, N)


def inverse_repack_umma(tiles, K, N):
    return _layout("i4o_inverse_repack_umma", tiles, K, N)


def repack_scales_128(scales, K, N, group):
    scales = _u16(scales)
    out = np.zeros((K // group) * N, np.uint16)
    lib().i4o_repack_scales_128(_p(scales, _u16p), _p(out, _u16p), K, N, group)
    return out


# ---------------------------------------------------------- reference itself

def ref_quantize(b, K, N, group):
    b = _u16(b)
    groups = (K + group - 1) // group
    packed = np.zeros(K * N // 2, np.uint8)
    scales = np.zeros((groups, N), np.uint16)
    ref_lib().i4r_quantize(_p(b, _u16p), _p(packed, _u8p), _p(scales, _u16p), K, N, group)
    return packed, scales


def ref_dequantize(packed, scales, K, N, group):
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = _u16(scales)
    out = np.empty((K, N), np.uint16)
    ref_lib().i4r_dequantize(_p(packed, _u8p), _p(scales, _u16p), _p(out, _u16p), K, N, group)
    return out


def ref_gemm_rows(a, b16, M, N, K, row0=0, rows=None, threads=1):
    a = _u16(a)
    b16 = _u16(b16)
    rows = M - row0 if rows is None else rows
    out = np.empty((rows, N), np.float32)
    ref_lib().i4r_gemm_rows(_p(a, _u16p), _p(b16, _u16p), _p(out, _f32p),
                            M, N, K, row0, rows, threads)
    return out


def ref_random_half(count, seed) -> np.ndarray:
    out = np.empty(count, np.uint16)
    ref_lib().i4r_random_half(_p(out, _u16p), count, seed)
    return out


def _ref_layout(name, packed, K, N):
    packed = np.ascontiguousarray(packed, np.uint8)
    out = np.zeros(K * N // 2, np.uint8)
    getattr(ref_lib(), name)(_p(packed, _u8p), _p(out, _u8p), K, N)
    return out


def ref_repack_128x32(packed, K, N):
    return _ref_layout("i4r_repack_128x32", packed, K, N)


def ref_repack_mma_128x32(packed, K, N):
    return _ref_layout("i4r_repack_mma_128x32", packed, K, N)


def ref_repack_mma_pair_128x32(packed, K, N):
    return _ref_layout("i4r_repack_mma_pair_128x32", packed, K, N)


def ref_repack_scales_128(scales, K, N, group):
    scales = _u16(scales)
    out = np.zeros((K // group) * N, np.uint16)
    ref_lib().i4r_repack_scales_128(_p(scales, _u16p), _p(out, _u16p), K, N, group)
    return out
