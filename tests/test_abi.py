"""C ABI checks that need no GPU: the library builds, loads, exports every
symbol include/gdn_b200.h declares, and its argument validation rejects bad
calls before any device work."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


@pytest.fixture(scope="module")
def lib():
    from gdn_b200 import _build, _lib
    _build.build()
    return _lib.load()


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|void|uint64_t)\s+(gdn_\w+)\s*\(", text, re.M)))


def test_header_declares_expected_entry_points():
    from gdn_b200 import _lib
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib):
    from gdn_b200 import _lib
    assert lib.gdn_abi_version() == _lib.ABI_VERSION
    for code in range(0, 8):
        assert len(lib.gdn_status_string(code)) > 0
    assert b"unknown" in lib.gdn_status_string(99)


def _args(**kw):
    from gdn_b200 import _lib
    a = _lib.GdnFwdArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V = 1, 64, 1, 128, 128
    a.chunk_size = 64
    a.in_dtype = _lib.DTYPE_BF16
    a.out_dtype = _lib.DTYPE_BF16
    fake = 0x10000  # 16-byte aligned, never dereferenced: validation fails or no device is found first
    for name in ("q", "k", "v", "o"):
        setattr(a, name, fake)
        st = getattr(a, name + "_stride")
        st[0], st[1], st[2] = 64 * 128, 128, 128
    for name in ("beta", "g"):
        setattr(a, name, fake)
        st = getattr(a, name + "_stride")
        st[0], st[1], st[2] = 64, 1, 1
    for key, val in kw.items():
        setattr(a, key, val)
    return a


@pytest.mark.parametrize("field,value,expected", [
    ("abi_version", 99, 1),
    ("B", 0, 1),
    ("T", 0, 1),
    ("in_dtype", 7, 1),
    ("in_dtype", 0, 2),          # fp32 inputs: valid request, not supported by this build
    ("K", 64, 2),
    ("chunk_size", 32, 2),
    ("block_v", 48, 2),
    ("q", 0x10008, 3),           # not 16-byte aligned
    ("flags", 16, 1),            # unknown flag
    ("flags", 8, 1),             # Newton-Schulz without an iteration count
    ("flags", 3 << 8, 1),        # an iteration count without Newton-Schulz
    ("scale", float("nan"), 1),
    ("beta", None, 1),
])
def test_validation_rejects_before_device_work(lib, field, value, expected):
    a = _args(**{field: value})
    rc = lib.gdn_fwd_sm100(ctypes.byref(a), None)
    assert rc == expected, (field, value, rc)


def test_null_input_pointer_rejected(lib):
    a = _args()
    a.v = None
    assert lib.gdn_fwd_sm100(ctypes.byref(a), None) == 1


def test_null_gate_is_accepted(lib):
    """g == NULL selects the DeltaNet recurrence (g == 0): validation passes and
    the call gets as far as the device check."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU tests")
    a = _args()
    a.g = None
    assert lib.gdn_fwd_sm100(ctypes.byref(a), None) == 6


def test_misaligned_stride_rejected(lib):
    a = _args()
    a.k_stride[1] = 129  # 258 bytes: not a multiple of 16
    assert lib.gdn_fwd_sm100(ctypes.byref(a), None) == 3


def test_valid_args_without_sm100_report_no_device(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU tests")
    a = _args()
    assert lib.gdn_fwd_sm100(ctypes.byref(a), None) == 6


def test_null_args_pointer(lib):
    assert lib.gdn_fwd_sm100(None, None) == 1


def test_workspace_query(lib):
    a = _args(B=2, T=4096, H=16)
    from gdn_b200 import _lib
    pk = _lib.PACKET_BYTES_PER_CHUNK
    # one packet per (b, h, chunk) plus one fp32 state per (b, h)
    hdr = _lib.WORKSPACE_HEADER_BYTES
    assert lib.gdn_fwd_workspace_bytes(ctypes.byref(a)) == hdr + 2 * 16 * (64 * pk + 128 * 128 * 4)
    a = _args(T=100)
    assert lib.gdn_fwd_workspace_bytes(ctypes.byref(a)) == hdr + 1 * 1 * (2 * pk + 128 * 128 * 4)
    assert lib.gdn_fwd_workspace_bytes(None) == 0
