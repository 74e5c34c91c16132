"""ctypes binding of ``libscmp_b200.so`` (the C ABI declared in include/scmp_b200.h).

The library is loaded on first use; if it is missing or the process has no
CUDA device, every entry point raises instead of falling back to anything
else. Status codes map to the reference's exception types: invalid arguments
raise ``ValueError``, unsupported group sizes ``NotImplementedError``, CUDA
and device-side failures ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libscmp_b200.so")

SCMP_OK = 0
SCMP_ERR_INVALID_ARG = 1
SCMP_ERR_CUDA = 2
SCMP_ERR_TIMEOUT = 3
SCMP_ERR_UNSUPPORTED = 4
SCMP_ERR_WORKSPACE = 5

PER_TENSOR, PER_ROW, PER_HEAD = 0, 1, 2
BIPOLAR, UNIPOLAR = 0, 1
FLAG_FORCE_SIMT = 0x1
FLAG_NO_SPLIT = 0x2
FLAG_B_READY = 0x4
ABI_VERSION = 4
MAX_OUT_PEERS = 8

c_int, c_void_p, c_size_t, c_float, c_double = (ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                                ctypes.c_float, ctypes.c_double)


class MatmulDesc(ctypes.Structure):
    """Mirror of ``scmp_matmul_desc``."""
    _fields_ = [
        ("granularity", c_int), ("mode", c_int), ("sc_prec", c_int), ("stoc_len", c_int),
        ("rng_levels", c_int), ("chunk_d", c_int), ("group_a", c_int), ("group_b", c_int),
        ("batch", c_int), ("n", c_int), ("m", c_int), ("d", c_int),
        ("a", c_void_p), ("b", c_void_p), ("smooth_scales", c_void_p), ("out", c_void_p),
        ("ktab", c_void_p), ("pattern", c_void_p), ("amap", c_void_p), ("bmap", c_void_p),
        ("vcap", c_int), ("lp", c_int), ("flags", c_int), ("tensor_ranges", c_void_p),
        ("out_peers", c_void_p), ("n_out_peers", c_int), ("out_ld", c_int), ("out_offset", ctypes.c_longlong),
        ("pattern4", c_void_p), ("out_self", c_int),
    ]


class LevelDesc(ctypes.Structure):
    """Mirror of ``scmp_level_desc``."""
    _fields_ = [
        ("stoc_len", c_int), ("rng_levels", c_int), ("vcap", c_int), ("lp", c_int),
        ("ktab", c_void_p), ("pattern4", c_void_p), ("amap", c_void_p), ("bmap", c_void_p),
    ]


MAX_LEVELS = 4

# name -> (restype, argtypes); every symbol of include/scmp_b200.h
SIGNATURES = {
    "scmp_abi_version": (c_int, []),
    "scmp_launch_count": (ctypes.c_ulonglong, []),
    "scmp_set_profile_events": (c_int, [c_void_p, c_void_p]),
    "scmp_set_quant_profile_events": (c_int, [c_void_p, c_void_p]),
    "scmp_last_error": (ctypes.c_char_p, []),
    "scmp_device_error": (c_int, [ctypes.POINTER(c_int)]),
    "scmp_build_tables": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                  c_void_p, c_void_p, c_void_p]),
    "scmp_peer_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    "scmp_peer_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "scmp_peer_close": (c_int, [c_void_p]),
    "scmp_peer_free": (c_int, [c_void_p]),
    "scmp_sc_matmul_workspace_size": (c_int, [ctypes.POINTER(MatmulDesc), ctypes.POINTER(c_size_t)]),
    "scmp_sc_matmul": (c_int, [ctypes.POINTER(MatmulDesc), c_void_p, c_size_t, c_void_p]),
    "scmp_sc_matmul_noalloc": (c_int, [ctypes.POINTER(MatmulDesc), c_void_p]),
    "scmp_sc_matmul_levels_workspace_size": (c_int, [ctypes.POINTER(MatmulDesc), ctypes.POINTER(LevelDesc), c_int,
                                                     ctypes.POINTER(c_size_t)]),
    "scmp_sc_matmul_levels": (c_int, [ctypes.POINTER(MatmulDesc), ctypes.POINTER(LevelDesc), c_int, c_void_p,
                                      c_void_p, c_size_t, c_void_p]),
    "scmp_enable_matmul_workspace_size": (c_int, [c_int, c_int, c_int, ctypes.POINTER(c_size_t)]),
    "scmp_enable_matmul": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                   c_float, c_int, c_void_p, c_void_p, c_size_t, c_int, c_void_p]),
    "scmp_fused_quantize_bipolar": (c_int, [c_void_p, c_int, c_int, c_double, c_int, c_int,
                                            c_void_p, c_void_p, ctypes.POINTER(c_double), c_void_p]),
    "scmp_fused_quantize_bipolar_perrow": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                                   c_void_p, c_void_p, c_void_p]),
    "scmp_fused_quantize_unipolar": (c_int, [c_void_p, c_int, c_int, c_double, c_double, c_int,
                                             c_int, c_void_p, c_void_p, ctypes.POINTER(c_double),
                                             ctypes.POINTER(c_double), c_void_p]),
    "scmp_fused_quant_bipolar_batched": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int,
                                                 c_int, c_void_p, c_void_p, c_void_p]),
    "scmp_grouped_symmetric_quant": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                             c_void_p, c_void_p, c_void_p, c_void_p]),
    "scmp_grouped_asymmetric_quant": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                              c_void_p, c_void_p, c_void_p, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library (no CUDA call is made by loading)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"scmp_kernels_b200: native library {path} is missing; build it with "
                "`python -m scmp_kernels_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.scmp_abi_version() != ABI_VERSION:
            raise RuntimeError("scmp_kernels_b200: ABI version mismatch; rebuild the library")
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load()


def check(status: int, what: str = "") -> None:
    if status == SCMP_OK:
        return
    msg = lib().scmp_last_error().decode(errors="replace")
    if what and what not in msg:
        msg = f"{what}: {msg}"
    if status == SCMP_ERR_INVALID_ARG:
        raise ValueError(msg)
    if status == SCMP_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"scmp_kernels_b200 error {status}: {msg}")


def device_error() -> int:
    """Synchronise and return (and clear) the first error a kernel recorded."""
    code = c_int(0)
    check(lib().scmp_device_error(ctypes.byref(code)), "scmp_device_error")
    return code.value


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """Device buffer on the current device and its 64-byte IPC handle."""
    ptr, handle = c_void_p(), ctypes.create_string_buffer(64)
    check(lib().scmp_peer_alloc(nbytes, ctypes.byref(ptr), handle), "scmp_peer_alloc")
    return int(ptr.value), handle.raw


def peer_open(handle: bytes) -> int:
    """Map another process's scmp_peer_alloc buffer into this one."""
    ptr = c_void_p()
    check(lib().scmp_peer_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)), "scmp_peer_open")
    return int(ptr.value)


def launch_count() -> int:
    """Kernels the library has launched in this process so far."""
    return int(lib().scmp_launch_count())


def stream_handle(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda() -> None:
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError(
            "scmp_kernels_b200: a CUDA device (B200, sm_100a) is required; "
            "this package has no CPU implementation")
