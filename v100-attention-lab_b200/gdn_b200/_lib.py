"""ctypes binding of the C ABI declared in include/gdn_b200.h.

Loading is strict: if ``libgdn_b200.so`` is missing or does not export the
expected symbols, ``load()`` raises.  There is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import _build

ABI_VERSION = 3

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_ALIGNMENT = 3
ERR_CUDA = 4
ERR_TIMEOUT = 5
ERR_NO_DEVICE = 6
ERR_SCRATCH_LIMIT = 7

# gdn_fwd_args.flags: input preparation inside the kernel
FLAG_QK_L2NORM = 1
FLAG_BETA_SIGMOID = 2
FLAG_G_LOGSIGMOID = 4
FLAG_SOLVER_NS = 8       # Newton-Schulz solve of (I + A)^-1 (gdn_triton_v2.py:58-68)
NS_ITERS_SHIFT = 8       # its iteration count, 1..15, in bits 8-11

# Scratch bytes of the two-kernel path per (batch, head, chunk of 64 steps);
# gdn_fwd_workspace_bytes() is the authority, this mirrors it for sizing.
PACKET_BYTES_PER_CHUNK = 98560
WORKSPACE_HEADER_BYTES = 256  # the prep's item counter, ahead of the state area and packets

# Every symbol include/gdn_b200.h declares.
EXPORTED_SYMBOLS = ("gdn_fwd_sm100", "gdn_fwd_sm100_noalloc", "gdn_fwd_workspace_bytes", "gdn_wy_prep_sm100",
                    "gdn_selftest_wait_timeout", "gdn_status_string", "gdn_abi_version")

_i64x3 = ctypes.c_int64 * 3


class GdnFwdArgs(ctypes.Structure):
    """Mirror of ``struct gdn_fwd_args`` (include/gdn_b200.h)."""

    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("B", ctypes.c_int32),
        ("T", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("V", ctypes.c_int32),
        ("chunk_size", ctypes.c_int32),
        ("in_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("block_v", ctypes.c_int32),
        ("q", ctypes.c_void_p),
        ("q_stride", _i64x3),
        ("k", ctypes.c_void_p),
        ("k_stride", _i64x3),
        ("v", ctypes.c_void_p),
        ("v_stride", _i64x3),
        ("beta", ctypes.c_void_p),
        ("beta_stride", _i64x3),
        ("g", ctypes.c_void_p),
        ("g_stride", _i64x3),
        ("h0", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("o_stride", _i64x3),
        ("ht", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64),
        ("scale", ctypes.c_float),
        ("flags", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return os.environ.get("GDN_B200_LIB", _build.LIB_PATH)


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load the shared library (building it first if asked and possible)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if build_if_missing:
                _build.build()
            else:
                raise RuntimeError(
                    f"gdn_b200: native library not found at {path}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` (needs nvcc)")
        lib = ctypes.CDLL(path)
        missing = [s for s in EXPORTED_SYMBOLS if not hasattr(lib, s)]
        if missing:
            raise RuntimeError(f"gdn_b200: {path} lacks symbols {missing}")
        lib.gdn_fwd_sm100.argtypes = [ctypes.POINTER(GdnFwdArgs), ctypes.c_void_p]
        lib.gdn_fwd_sm100.restype = ctypes.c_int
        lib.gdn_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(GdnFwdArgs), ctypes.c_void_p]
        lib.gdn_fwd_sm100_noalloc.restype = ctypes.c_int
        lib.gdn_fwd_workspace_bytes.argtypes = [ctypes.POINTER(GdnFwdArgs)]
        lib.gdn_fwd_workspace_bytes.restype = ctypes.c_uint64
        lib.gdn_wy_prep_sm100.argtypes = [ctypes.POINTER(GdnFwdArgs), ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p]
        lib.gdn_wy_prep_sm100.restype = ctypes.c_int
        lib.gdn_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
        lib.gdn_selftest_wait_timeout.restype = ctypes.c_int
        lib.gdn_status_string.argtypes = [ctypes.c_int]
        lib.gdn_status_string.restype = ctypes.c_char_p
        lib.gdn_abi_version.argtypes = []
        lib.gdn_abi_version.restype = ctypes.c_int
        if lib.gdn_abi_version() != ABI_VERSION:
            raise RuntimeError(f"gdn_b200: ABI version {lib.gdn_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().gdn_status_string(int(code)).decode()
