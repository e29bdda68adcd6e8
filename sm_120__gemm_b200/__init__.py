"""B200-native (sm_100a) fused W4A16 INT4 weight-only GEMM.

``C[M,N] = A_fp16[M,K] x dequant(B_int4[K,N], fp16 group scale)``, FP32
accumulation, FP16 (or FP32) output, group size 32 / 64 / 128.

This module is the Python host side of ``libi4g.so`` (the C ABI in
``include/i4g.h``). Its ``launch_*`` functions mirror the host API of
zichaowen8-prog/SM_120__GEMM one to one (``include/quant.cuh:6-21``,
``include/kernels.cuh:81-83``): same names, same argument order and meaning,
and an exception (``I4GError``, a ``RuntimeError``) where the reference
throws ``std::runtime_error``. Device buffers are ``torch`` CUDA tensors;
``stream`` is a ``torch.cuda.Stream``, a raw ``cudaStream_t`` integer, or
``None`` for the current torch stream.

The compute path is the CUDA library only: if ``libi4g.so`` is missing the
import of any launch function raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

__all__ = [
    "I4GError", "load", "launch_quantize", "launch_quantize_repack", "launch_dequantize",
    "launch_repack_128x32", "launch_inverse_repack_128x32", "launch_repack_mma_128x32",
    "launch_repack_mma_pair_128x32", "launch_repack_scales_128", "launch_repack_umma",
    "launch_inverse_repack_umma", "launch_final", "launch_final_fp32", "launch_gemm_variant",
    "gemm_workspace_size", "launch_final_ws", "launch_final_fp32_ws", "workspace_for",
    "launch_final_to_peers", "ipc_handle", "ipc_open", "ipc_close", "peer_barrier",
    "shard_range", "device_status", "selftest_wait_timeout", "plan", "set_decode_schedule",
    "kernel_config", "kernel_resources", "max_pairs",
    "QuantizedLinear", "VARIANT_AUTO", "VARIANT_TC", "VARIANT_DECODE", "DECODE_SCHEDULES",
    "PLAN_KERNELS", "PLAN_SCHEDULES", "LIB_PATH",
]

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libi4g.so")
VARIANT_AUTO, VARIANT_TC, VARIANT_DECODE = 0, 1, 2

_lock = threading.Lock()
_lib = None
_vp = ctypes.c_void_p
_i = ctypes.c_int


class I4GError(RuntimeError):
    """A non-zero status from libi4g (the reference throws std::runtime_error)."""

    def __init__(self, func: str, status: int, detail: str):
        self.status = status
        super().__init__(f"{func} failed: {detail} (status {status})")


_SIGNATURES = {
    "i4g_quantize": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "i4g_dequantize": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "i4g_quantize_repack": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "i4g_repack_128x32": [_vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "i4g_inverse_repack_128x32": [_vp, _vp, _i, _i, _vp],
    "i4g_repack_mma_128x32": [_vp, _vp, _i, _i, _vp],
    "i4g_repack_mma_pair_128x32": [_vp, _vp, _i, _i, _vp],
    "i4g_repack_scales_128": [_vp, _vp, _i, _i, _i, _vp],
    "i4g_repack_umma": [_vp, _vp, _i, _i, _vp],
    "i4g_inverse_repack_umma": [_vp, _vp, _i, _i, _vp],
    "i4g_gemm": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "i4g_gemm_fp32": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp],
    "i4g_gemm_variant": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp],
    "i4g_gemm_workspace_size": [_i, _i, _i, ctypes.POINTER(ctypes.c_size_t)],
    "i4g_gemm_ws": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, ctypes.c_size_t, _vp],
    "i4g_gemm_fp32_ws": [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, ctypes.c_size_t, _vp],
    "i4g_gemm_to_peers": [_vp, _vp, _vp, ctypes.POINTER(_vp), _i, _i, _i, _i, _i, _i, _i, _vp,
                          ctypes.c_size_t, _vp],
    "i4g_ipc_handle": [_vp, _vp, ctypes.POINTER(ctypes.c_size_t)],
    "i4g_ipc_open": [_vp, ctypes.POINTER(_vp)],
    "i4g_ipc_close": [_vp],
    "i4g_shard_range": [_i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_size_t),
                        ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(_i),
                        ctypes.POINTER(_i)],
    "i4g_device_status": [ctypes.POINTER(_i), _vp],
    "i4g_selftest_wait_timeout": [ctypes.c_ulonglong, _vp],
    "i4g_set_decode_schedule": [_i],
    "i4g_plan": [_i, _i, _i, _i, _i, _i, ctypes.c_size_t, ctypes.POINTER(_i), ctypes.POINTER(_i),
                 ctypes.POINTER(_i), ctypes.POINTER(ctypes.c_size_t)],
    "i4g_peer_barrier": [_vp, ctypes.POINTER(_vp), _i, _i, ctypes.c_ulonglong, ctypes.c_ulonglong,
                         _vp],
    "i4g_layout_version": [],
}


class _KernelConfig(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("rows", "cols", "bk", "mma_m", "mma_n", "stages", "threads",
                                  "dynamic_smem_bytes")]


class _KernelResources(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("registers_per_thread", "static_smem_bytes",
                                  "max_threads_per_block", "active_blocks_per_sm")]


_SIGNATURES["i4g_kernel_config"] = [_i, _i, _i, ctypes.POINTER(_KernelConfig)]
_SIGNATURES["i4g_max_pairs"] = [ctypes.POINTER(_i)]
_SIGNATURES["i4g_kernel_resources"] = [_i, _i, _i, ctypes.POINTER(_KernelResources)]


def load() -> ctypes.CDLL:
    """Load libi4g.so (built by ``make -C sm_120__gemm_b200``); raise if absent."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is not built; run `make -C {HERE}` "
                    "(the product has no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _i
            lib.i4g_status_string.argtypes = [_i]
            lib.i4g_status_string.restype = ctypes.c_char_p
            lib.i4g_last_error.argtypes = []
            lib.i4g_last_error.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def _check(func: str, status: int) -> None:
    if status != 0:
        lib = load()
        detail = lib.i4g_status_string(status).decode()
        extra = lib.i4g_last_error().decode()
        raise I4GError(func, status, f"{detail}: {extra}" if extra else detail)


def _stream(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(t) -> int:
    if t is None:
        return 0
    if not t.is_cuda:
        raise I4GError("argument check", -1, "tensors must be CUDA device tensors")
    return t.data_ptr()


def _call(name: str, *args) -> None:
    _check(name, getattr(load(), name)(*args))


# ------------------------------------------------- reference host API mirror

def launch_quantize(b, packed, scales, K: int, N: int, group_size: int, stream=None) -> None:
    """include/quant.cuh:6-7. Codes/scales bit-identical to quantize_cpu."""
    _call("i4g_quantize", _ptr(b), _ptr(packed), _ptr(scales), K, N, group_size, _stream(stream))


def launch_quantize_repack(b, tiles, scales_repacked, K: int, N: int, group_size: int,
                           stream=None) -> None:
    """One pass: launch_quantize + launch_repack_umma + launch_repack_scales_128
    (the one-shot path of src/main.cu:320-331), reading B once."""
    _call("i4g_quantize_repack", _ptr(b), _ptr(tiles), _ptr(scales_repacked), K, N, group_size,
          _stream(stream))


def launch_dequantize(packed, scales, b, K: int, N: int, group_size: int, stream=None) -> None:
    """include/quant.cuh:8-9."""
    _call("i4g_dequantize", _ptr(packed), _ptr(scales), _ptr(b), K, N, group_size,
          _stream(stream))


def launch_repack_128x32(packed, scales, repacked, repacked_scales, K: int, N: int,
                         group_size: int, stream=None) -> None:
    """include/quant.cuh:10-12."""
    _call("i4g_repack_128x32", _ptr(packed), _ptr(scales), _ptr(repacked),
          _ptr(repacked_scales), K, N, group_size, _stream(stream))


def launch_inverse_repack_128x32(repacked, packed, K: int, N: int, stream=None) -> None:
    """include/quant.cuh:13-14."""
    _call("i4g_inverse_repack_128x32", _ptr(repacked), _ptr(packed), K, N, _stream(stream))


def launch_repack_mma_128x32(packed, repacked, K: int, N: int, stream=None) -> None:
    """include/quant.cuh:15-16."""
    _call("i4g_repack_mma_128x32", _ptr(packed), _ptr(repacked), K, N, _stream(stream))


def launch_repack_mma_pair_128x32(packed, repacked, K: int, N: int, stream=None) -> None:
    """include/quant.cuh:17-18."""
    _call("i4g_repack_mma_pair_128x32", _ptr(packed), _ptr(repacked), K, N, _stream(stream))


def launch_repack_scales_128(scales, repacked_scales, K: int, N: int, group_size: int,
                             stream=None) -> None:
    """include/quant.cuh:19-21; also the scale layout of launch_final."""
    _call("i4g_repack_scales_128", _ptr(scales), _ptr(repacked_scales), K, N, group_size,
          _stream(stream))


def launch_repack_umma(packed, tiles, K: int, N: int, stream=None) -> None:
    """The weight layout launch_final consumes here (blocks of 128 cols x 64 k)."""
    _call("i4g_repack_umma", _ptr(packed), _ptr(tiles), K, N, _stream(stream))


def launch_inverse_repack_umma(tiles, packed, K: int, N: int, stream=None) -> None:
    _call("i4g_inverse_repack_umma", _ptr(tiles), _ptr(packed), K, N, _stream(stream))


def launch_final(a, b_repacked, scales_repacked, c, M: int, N: int, K: int, group: int,
                 stream=None) -> None:
    """include/kernels.cuh:83 (kernels/gemm_final.cu:5-13): fp16 C = A x dequant(B)."""
    _call("i4g_gemm", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), _ptr(c), M, N, K, group,
          _stream(stream))


def launch_final_fp32(a, b_repacked, scales_repacked, c, M: int, N: int, K: int, group: int,
                      stream=None) -> None:
    """include/kernels.cuh:81: the same product with an FP32 C."""
    _call("i4g_gemm_fp32", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), _ptr(c), M, N, K,
          group, _stream(stream))


def launch_gemm_variant(a, b_repacked, scales_repacked, c, M: int, N: int, K: int, group: int,
                        variant: int, stream=None) -> None:
    _call("i4g_gemm_variant", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), _ptr(c), M, N,
          K, group, variant, _stream(stream))


def gemm_workspace_size(M: int, N: int, K: int) -> int:
    """Bytes of split-K workspace the current device wants for this shape (0: none)."""
    b = ctypes.c_size_t()
    _call("i4g_gemm_workspace_size", M, N, K, ctypes.byref(b))
    return b.value


def launch_final_ws(a, b_repacked, scales_repacked, c, M: int, N: int, K: int, group: int,
                    workspace, stream=None) -> None:
    """launch_final with a split-K workspace: a zero-initialised uint8 CUDA
    tensor (``workspace_for``); calls sharing it must be stream-ordered."""
    _call("i4g_gemm_ws", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), _ptr(c), M, N, K,
          group, _ptr(workspace), 0 if workspace is None else workspace.numel(),
          _stream(stream))


def launch_final_fp32_ws(a, b_repacked, scales_repacked, c, M: int, N: int, K: int,
                         group: int, workspace, stream=None) -> None:
    _call("i4g_gemm_fp32_ws", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), _ptr(c), M, N,
          K, group, _ptr(workspace), 0 if workspace is None else workspace.numel(),
          _stream(stream))


_workspaces: dict = {}


def workspace_for(M: int, N: int, K: int, device=None, stream=None):
    """A zeroed split-K workspace for (device, stream), grown on demand.

    One buffer per stream keeps launches that share it ordered. The kernel
    leaves the workspace's counters at zero, so it is zeroed only when made.
    Returns None when the shape needs no workspace."""
    import torch
    need = gemm_workspace_size(M, N, K)
    if need == 0:
        return None
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    key = (dev.index, _stream(stream))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws


def launch_final_to_peers(a, b_repacked, scales_repacked, dsts, ldc: int, col0: int, M: int,
                          N: int, K: int, group: int, workspace=None, stream=None) -> None:
    """C ABI i4g_gemm_to_peers: this launch's columns [col0, col0 + N) of
    C = A x dequant(B), written into every matrix of `dsts` (device base
    pointers of row-major [M][ldc] FP16 matrices, this GPU's and peers')."""
    arr = (_vp * len(dsts))(*dsts)
    _call("i4g_gemm_to_peers", _ptr(a), _ptr(b_repacked), _ptr(scales_repacked), arr, len(dsts),
          ldc, col0, M, N, K, group, _ptr(workspace), 0 if workspace is None else workspace.numel(),
          _stream(stream))


def ipc_handle(t) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding tensor `t`, byte
    offset of t in it)."""
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_size_t()
    _call("i4g_ipc_handle", _ptr(t), h, ctypes.byref(off))
    return h.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map a peer's allocation (from ipc_handle) into this process; base pointer."""
    base = _vp()
    _call("i4g_ipc_open", ctypes.create_string_buffer(handle, 64), ctypes.byref(base))
    return base.value


def ipc_close(base: int) -> None:
    _call("i4g_ipc_close", base)


def shard_range(K: int, N: int, group: int, world: int, rank: int):
    """(tile_byte_offset, scale_byte_offset, n0, n1) of a column-parallel shard."""
    t = ctypes.c_size_t()
    s = ctypes.c_size_t()
    n0 = _i()
    n1 = _i()
    _call("i4g_shard_range", K, N, group, world, rank, ctypes.byref(t), ctypes.byref(s),
          ctypes.byref(n0), ctypes.byref(n1))
    return t.value, s.value, n0.value, n1.value


def device_status(stream=None) -> int:
    """Read and clear the device status word (0, or -8 after a wait timeout)."""
    out = _i()
    _call("i4g_device_status", ctypes.byref(out), _stream(stream))
    return out.value


def selftest_wait_timeout(limit_ns: int, stream=None) -> None:
    _call("i4g_selftest_wait_timeout", limit_ns, _stream(stream))


def peer_barrier(local_flags: int, peer_flags, world: int, rank: int, epoch: int,
                 limit_ns: int = 0, stream=None) -> None:
    """C ABI i4g_peer_barrier: device pointers of this rank's flag array and
    of every rank's array as mapped here (list indexed by rank)."""
    arr = (_vp * world)(*[p or 0 for p in peer_flags])
    _call("i4g_peer_barrier", local_flags, arr, world, rank, epoch, limit_ns, _stream(stream))


PLAN_KERNELS = {0: "tcgen05/256", 1: "tcgen05/128", 2: "decode"}
PLAN_SCHEDULES = {0: "whole", 1: "split", 2: "stream-k", 3: "cluster", 4: "slices"}


def plan(M: int, N: int, K: int, group: int, sm_count: int, workspace_bytes: int = 0,
         fp32_out: bool = False) -> dict:
    """C ABI i4g_plan: the kernel and schedule this shape would run with
    `workspace_bytes` of workspace on a device with `sm_count` SMs (no
    device needed)."""
    k, s, p = _i(), _i(), _i()
    b = ctypes.c_size_t()
    _call("i4g_plan", M, N, K, group, int(fp32_out), sm_count, workspace_bytes, ctypes.byref(k),
          ctypes.byref(s), ctypes.byref(p), ctypes.byref(b))
    return {"kernel": PLAN_KERNELS[k.value], "schedule": PLAN_SCHEDULES[s.value],
            "param": p.value, "workspace_bytes": b.value}


def kernel_config(variant: int, rows: int, group: int) -> dict:
    """C ABI i4g_kernel_config (the reference's KernelMetadata, kernels.cuh:6-14):
    tile, stages, threads and shared memory of one kernel instance; no device."""
    c = _KernelConfig()
    _call("i4g_kernel_config", variant, rows, group, ctypes.byref(c))
    return {n: getattr(c, n) for n, _ in _KernelConfig._fields_}


def kernel_resources(variant: int, rows: int, group: int) -> dict:
    """C ABI i4g_kernel_resources (the reference's KernelResources,
    kernels.cuh:16-22): registers, static shared memory, block limit and
    resident CTAs per SM of one kernel instance on the current device."""
    r = _KernelResources()
    _call("i4g_kernel_resources", variant, rows, group, ctypes.byref(r))
    return {n: getattr(r, n) for n, _ in _KernelResources._fields_}


def max_pairs() -> int:
    """C ABI i4g_max_pairs: CTA pairs of the paired tcgen05 kernel resident at
    once on the current device."""
    v = _i()
    _call("i4g_max_pairs", ctypes.byref(v))
    return v.value


DECODE_SCHEDULES = {"auto": 0, "cluster": 1, "streamk": 2, "slices": 3}


def set_decode_schedule(schedule: str) -> None:
    """C ABI i4g_set_decode_schedule: "auto", "slices", "cluster" or "streamk", for
    decode-shaped (M <= 16) launches issued after the call, process-wide."""
    _call("i4g_set_decode_schedule", DECODE_SCHEDULES[schedule])


from .linear import QuantizedLinear  # noqa: E402  (needs the launchers above)
