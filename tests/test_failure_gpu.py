"""Device-side failure detection, exercised without faulting the GPU: a
bounded wait on an mbarrier that nothing arrives at must expire, report
GDN_ERR_TIMEOUT through the status word, and leave the context usable."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_reports():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gdn_b200 import _lib, ops
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # ~2 ms at 1.9 GHz: short, so the test takes no time
    rc = lib.gdn_selftest_wait_timeout(ctypes.c_void_p(status.data_ptr()), 4_000_000, ctypes.c_void_p(stream))
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == (1 << _lib.ERR_TIMEOUT)
    # the context is still healthy: a real forward runs and checks clean
    from gpu_util import make
    qd, kd, vd, bd, gd, _ = make(1, 64, 1, seed=3, dtype=torch.float16)
    o, h = ops.gdn_chunk_fwd(qd, kd, vd, bd, gd, check=True)
    assert torch.isfinite(o.float()).all()


def test_status_word_maps_to_exception():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gdn_b200 import _lib, ops
    w = ops._status_word(torch.device("cuda", torch.cuda.current_device()))
    w.fill_(1 << _lib.ERR_TIMEOUT)
    with pytest.raises(ops.GdnError, match="timed out"):
        ops.check_status()
    assert int(w.item()) == 0
