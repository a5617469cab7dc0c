"""Out-of-bounds write detection without a sanitizer.

The output `o`, the final state and the two-kernel path's scratch are placed
inside larger buffers filled with a sentinel byte pattern; `o` is also given
a padded head stride, so it has holes between heads.  After the launch every
byte outside the elements the call owns must still hold the sentinel, and the
values inside must match the oracle.  Runs on both paths (fused kernel and
prep + scan), ragged T, and every output dtype, through the C ABI directly so
the test controls every pointer and stride.
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import STORE_ROUNDING, TOL, make, oracle, rel

pytestmark = pytest.mark.gpu

SENTINEL = 0x5A  # every byte; as fp32 / fp16 / bf16 this is an ordinary finite value
GUARD = 4096     # bytes before and after each region


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gdn_b200 import _lib
    return _lib.load()


def _guarded(nbytes, dev):
    buf = torch.full((GUARD + nbytes + GUARD,), SENTINEL, dtype=torch.uint8, device=dev)
    return buf


def _check_guards(buf, nbytes, what):
    host = buf.cpu().numpy()
    assert (host[:GUARD] == SENTINEL).all(), f"{what}: write below the region"
    assert (host[GUARD + nbytes:] == SENTINEL).all(), f"{what}: write above the region"


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [130, 256])
def test_writes_stay_inside_outputs(lib, fused, out_dtype, T):
    from gdn_b200 import _lib, ops
    dev = torch.device("cuda", 0)
    B, H, K, V = 2, 3, 128, 128
    qd, kd, vd, bd, gd, h0 = make(B, T, H, seed=T + 7, dtype=torch.bfloat16, h0_std=0.1)
    esz = torch.empty((), dtype=out_dtype).element_size()
    HP = V + 24  # padded head stride of o (elements): 24 unowned elements after each head's row
    o_elems = B * T * H * HP
    o_buf = _guarded(o_elems * esz, dev)
    o_full = o_buf[GUARD:GUARD + o_elems * esz].view(out_dtype).view(B, T, H, HP)
    o = o_full[..., :V]  # strided view: head stride HP
    ht_bytes = B * H * V * K * 4
    ht_buf = _guarded(ht_bytes, dev)
    ht = ht_buf[GUARD:GUARD + ht_bytes].view(torch.float32).view(B, H, V, K)

    status = torch.zeros(1, dtype=torch.int32, device=dev)
    args = ops._fill_args(qd, kd, vd, bd, gd, h0, o, ht, 64, 0, status)
    ws_buf = None
    if not fused:
        need = int(lib.gdn_fwd_workspace_bytes(ctypes.byref(args)))
        ws_buf = _guarded(need + 256, dev)
        base = ws_buf.data_ptr() + GUARD
        args.workspace = (base + 255) // 256 * 256
        args.workspace_bytes = need
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.gdn_fwd_sm100(ctypes.byref(args), ctypes.c_void_p(stream))
    assert rc == _lib.OK, _lib.status_string(rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0

    _check_guards(o_buf, o_elems * esz, "o")
    _check_guards(ht_buf, ht_bytes, "h_final")
    holes = o_full[..., V:].contiguous().view(torch.uint8).cpu().numpy()
    assert (holes == SENTINEL).all(), "o: write into the padding between heads"
    if ws_buf is not None:
        lo = args.workspace - ws_buf.data_ptr()
        host = ws_buf.cpu().numpy()
        assert (host[:lo] == SENTINEL).all(), "workspace: write below"
        assert (host[lo + args.workspace_bytes:] == SENTINEL).all(), "workspace: write above"

    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    assert rel(o, o_ref) < TOL + STORE_ROUNDING[out_dtype]
    assert rel(ht, h_ref) < TOL
