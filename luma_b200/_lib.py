"""ctypes binding of ``libluma_b200.so`` (the C ABI in include/luma_b200.h).

The shared library is built in-tree (``luma_b200/_lib/libluma_b200.so``, see
``luma_b200/build.py``).  There is no fallback: if the library is missing or
its struct layout disagrees with the numpy mirrors below, ``lib()`` raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libluma_b200.so")

ABI_VERSION = 4

LUMA_OK = 0
LUMA_ERR_INVALID = 1
LUMA_ERR_CUDA = 2
LUMA_ERR_UNSUPPORTED = 3

F32, BF16, F16 = 0, 1, 2

# numpy mirrors of the C structs (include/luma_b200.h); offsets are explicit
# so a layout drift fails the size check in lib().
DESC_DTYPE = np.dtype({
    "names": ["param", "grad", "q_m", "q_w", "u_m", "u_w", "numel", "oct_begin", "rng_offset",
              "param_id", "row", "slot", "param_dtype", "grad_dtype", "vec_ok", "mc_local",
              "param_mc"],
    "formats": ["<u8", "<u8", "<u8", "<u8", "<u8", "<u8", "<i8", "<i8", "<i8",
                "<i4", "<i4", "<i4", "u1", "u1", "u1", "u1", "<u8"],
    "offsets": [0, 8, 16, 24, 32, 40, 48, 56, 64, 72, 76, 80, 84, 85, 86, 87, 88],
    "itemsize": 96,
})

ROW_DTYPE = np.dtype({
    "names": ["step", "eps", "beta1", "omb1", "beta2", "omb2", "decay", "neg_eta", "inv_bc2",
              "eps32", "w_max", "reserved"],
    "formats": ["<i8", "<f8"] + ["<f4"] * 10,
    "offsets": [0, 8, 16, 20, 24, 28, 32, 36, 40, 44, 48, 52],
    "itemsize": 56,
})

GRID_DTYPE = np.dtype({
    "names": ["S_m", "S_v", "eps", "dm", "inv_dm", "inv_zm", "s_m32", "w_min", "inv_wmin", "dw",
              "inv_dw", "inv_zw", "dw_pos"],
    "formats": ["<f8", "<f8", "<f8"] + ["<f4"] * 9 + ["<i4"],
    "offsets": [0, 8, 16, 24, 28, 32, 36, 40, 44, 48, 52, 56, 60],
    "itemsize": 64,
})

SLOT_DTYPE = np.dtype({
    "names": ["grid", "amax_m", "amax_v", "done"],
    "formats": [(GRID_DTYPE, (2,)), "<u4", "<u4", "<u8"],
    "offsets": [0, 128, 132, 136],
    "itemsize": 144,
})


class LumaStepArgs(ctypes.Structure):
    _fields_ = [
        ("descs", ctypes.c_void_p),
        ("slots", ctypes.c_void_p),
        ("rows", ctypes.c_void_p),
        ("n_desc", ctypes.c_int32),
        ("n_rows", ctypes.c_int32),
        ("total_octets", ctypes.c_int64),
        ("base_seed", ctypes.c_int64),
        ("events", ctypes.c_void_p * 3),
        ("max_ctas", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("step_counters", ctypes.c_void_p),
        ("grad_scale", ctypes.c_void_p),
        ("found_inf", ctypes.c_void_p),
    ]


EXPECTED_SIZES = (DESC_DTYPE.itemsize, ROW_DTYPE.itemsize, GRID_DTYPE.itemsize,
                  SLOT_DTYPE.itemsize, ctypes.sizeof(LumaStepArgs))

EXPORTED = ("luma_step", "luma_step_noalloc", "luma_decode", "luma_quantize",
            "luma_abi_version", "luma_struct_sizes", "luma_last_error", "luma_arith_selfcheck",
            "luma_ipc_export", "luma_ipc_open", "luma_ipc_close", "luma_copy_async",
            "luma_error_flags", "luma_launch_config", "luma_mc_copy",
            "luma_log_selfcheck")

KERR_ROW_RANGE = 1  # LUMA_KERR_ROW_RANGE

NOALLOC_MAX_DESCS = 4096  # LUMA_NOALLOC_MAX_DESCS

_lib = None
_lock = threading.Lock()


class LumaError(RuntimeError):
    """A call into libluma_b200 returned an error status."""


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library, checking ABI and layout."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libluma_b200.so not found at {LIB_PATH}; build it with "
                f"`python -m luma_b200.build` (nvcc, sm_100a)")
        h = ctypes.CDLL(LIB_PATH)
        h.luma_abi_version.restype = ctypes.c_int
        h.luma_abi_version.argtypes = []
        h.luma_struct_sizes.restype = ctypes.c_int
        h.luma_struct_sizes.argtypes = [ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
        h.luma_last_error.restype = ctypes.c_char_p
        h.luma_last_error.argtypes = []
        h.luma_arith_selfcheck.restype = ctypes.c_int
        h.luma_arith_selfcheck.argtypes = [ctypes.c_uint64, ctypes.c_uint64,
                                           ctypes.POINTER(ctypes.c_uint64), ctypes.c_void_p]
        h.luma_ipc_export.restype = ctypes.c_int
        h.luma_ipc_export.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                      ctypes.POINTER(ctypes.c_uint64)]
        h.luma_ipc_open.restype = ctypes.c_int
        h.luma_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        h.luma_ipc_close.restype = ctypes.c_int
        h.luma_ipc_close.argtypes = [ctypes.c_void_p]
        h.luma_copy_async.restype = ctypes.c_int
        h.luma_copy_async.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                      ctypes.c_void_p]
        h.luma_log_selfcheck.restype = ctypes.c_int
        h.luma_log_selfcheck.argtypes = [ctypes.POINTER(ctypes.c_uint64),
                                         ctypes.POINTER(ctypes.c_double), ctypes.c_void_p]
        h.luma_mc_copy.restype = ctypes.c_int
        h.luma_mc_copy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                   ctypes.c_void_p]
        h.luma_launch_config.restype = ctypes.c_int
        h.luma_launch_config.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int]
        h.luma_error_flags.restype = ctypes.c_int
        h.luma_error_flags.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
        h.luma_step.restype = ctypes.c_int
        h.luma_step.argtypes = [ctypes.POINTER(LumaStepArgs), ctypes.c_void_p]
        h.luma_step_noalloc.restype = ctypes.c_int
        h.luma_step_noalloc.argtypes = [ctypes.POINTER(LumaStepArgs), ctypes.c_void_p]
        h.luma_decode.restype = ctypes.c_int
        h.luma_decode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                  ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        h.luma_quantize.restype = ctypes.c_int
        h.luma_quantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p]
        v = h.luma_abi_version()
        if v != ABI_VERSION:
            raise ImportError(f"libluma_b200 ABI {v}, expected {ABI_VERSION}")
        sizes = (ctypes.c_int64 * 5)()
        h.luma_struct_sizes(sizes, 5)
        if tuple(sizes) != EXPECTED_SIZES:
            raise ImportError(f"libluma_b200 struct sizes {tuple(sizes)} != {EXPECTED_SIZES}")
        _lib = h
        return h


def arith_selfcheck(n: int, seed: int = 0, stream=None) -> tuple[int, int, int]:
    """Mismatch counts (rcp, sqrt, div) of the step's branch-free arithmetic
    against CUDA's IEEE intrinsics over n random operands each (synchronises)."""
    out = (ctypes.c_uint64 * 3)()
    st = 0 if stream is None else stream.cuda_stream
    check(lib().luma_arith_selfcheck(n, seed, out, ctypes.c_void_p(st)), "luma_arith_selfcheck")
    return tuple(int(v) for v in out)


def log_selfcheck(stream=None) -> tuple[tuple[int, int], tuple[float, float, float]]:
    """((log1p violations, log violations), (max log1p rel err, max log abs err
    near 1, max log rel err)) of the certified logarithms, every float of their
    domains checked against CUDA's log1pf / logf (synchronises)."""
    bad = (ctypes.c_uint64 * 2)()
    err = (ctypes.c_double * 3)()
    st = 0 if stream is None else stream.cuda_stream
    check(lib().luma_log_selfcheck(bad, err, ctypes.c_void_p(st)), "luma_log_selfcheck")
    return (int(bad[0]), int(bad[1])), (float(err[0]), float(err[1]), float(err[2]))


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(64-byte IPC handle of the allocation holding device pointer `ptr`, byte offset of ptr)."""
    buf = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64(0)
    check(lib().luma_ipc_export(ctypes.c_void_p(ptr), buf, ctypes.byref(off)), "luma_ipc_export")
    return buf.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map a peer's allocation into this process; returns its base address."""
    if len(handle) != 64:
        raise ValueError("IPC handle must be 64 bytes")
    base = ctypes.c_void_p(0)
    check(lib().luma_ipc_open(handle, ctypes.byref(base)), "luma_ipc_open")
    return int(base.value)


def ipc_close(base: int) -> None:
    check(lib().luma_ipc_close(ctypes.c_void_p(base)), "luma_ipc_close")


def copy_async(dst: int, src: int, nbytes: int, stream) -> None:
    """One cudaMemcpyAsync (copy engine) of nbytes from src to dst on `stream`."""
    check(lib().luma_copy_async(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes,
                                ctypes.c_void_p(stream.cuda_stream)), "luma_copy_async")


LAUNCH_KEYS = ("pass1_threads", "pass1_elems_per_thread", "pass1_stages", "pass2_threads",
               "pass2_elems_per_thread", "pass2_stages", "ctas_per_sm", "decode_table_min_elems")


def launch_config() -> dict[str, int]:
    """The step kernels' launch constants as compiled into the library."""
    out = (ctypes.c_int32 * len(LAUNCH_KEYS))()
    k = lib().luma_launch_config(out, len(LAUNCH_KEYS))
    return {key: int(out[i]) for i, key in enumerate(LAUNCH_KEYS[:k])}


def mc_copy(mc_dst: int, src: int, nbytes: int, stream) -> None:
    """Multicast (NVLS) copy of nbytes from src into a multicast mapping on `stream`."""
    check(lib().luma_mc_copy(ctypes.c_void_p(mc_dst), ctypes.c_void_p(src), nbytes,
                             ctypes.c_void_p(stream.cuda_stream)), "luma_mc_copy")


def kernel_error_flags(clear: bool = False) -> int:
    """LUMA_KERR_* flags the step kernels raised on the current device (synchronises)."""
    out = ctypes.c_uint32(0)
    check(lib().luma_error_flags(ctypes.byref(out), int(clear)), "luma_error_flags")
    return out.value


def check(status: int, what: str) -> None:
    if status != LUMA_OK:
        msg = lib().luma_last_error().decode(errors="replace")
        kind = {LUMA_ERR_INVALID: ValueError, LUMA_ERR_UNSUPPORTED: RuntimeError}.get(status, LumaError)
        raise kind(f"{what} failed (status {status}): {msg}")
