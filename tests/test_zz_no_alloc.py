"""The allocation-free entry point gdn_fwd_sm100_noalloc, through the C ABI.

It exists for callers that may not allocate device memory at call time
(memory planned once at start-up, a host framework that owns the pool, or no
tolerance for cudaMalloc's device-wide synchronisation).  It keeps its scratch
in a fixed array inside the library.  These tests check that it computes what
the regular entry point computes, twice in a row (the array keeps the previous
call's contents), and that requests beyond the array's size are refused.

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gdn_b200
    from gdn_b200 import _lib, ops
    return gdn_b200, _lib, ops, _lib.load()


def _noalloc(env, q, k, v, beta, g, h0):
    _, _lib, ops, lib = env
    B, T, H, K = q.shape
    V = v.shape[-1]
    o = torch.empty(B, T, H, V, dtype=torch.float32, device=q.device)
    ht = torch.empty(B, H, V, K, dtype=torch.float32, device=q.device)
    args = ops._fill_args(q, k, v, beta, g, h0, o, ht, 64, 0, ops._status_word(q.device))
    rc = lib.gdn_fwd_sm100_noalloc(ctypes.byref(args),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, o, ht


def test_noalloc_matches_regular_entry_point_twice(env):
    from gpu_util import TOL, make, rel
    gdn, _lib, ops, _ = env
    # B*H = 32 heads and 32 chunks need ~103 MB of scratch in one piece, so
    # the 32 MiB array is used in four segments with the state carried over
    for call, seed in enumerate((51, 52)):
        qd, kd, vd, bd, gd, h0 = make(2, 2048, 16, seed=seed, dtype=torch.bfloat16, h0_std=0.1)
        rc, o, ht = _noalloc(env, qd, kd, vd, bd, gd, h0)
        assert rc == _lib.OK, (call, _lib.status_string(rc))
        ops.check_status()
        o_ref, h_ref = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0,
                                         output_dtype=torch.float32, check=True)
        assert rel(o, o_ref.cpu().numpy()) < TOL, call
        assert rel(ht, h_ref.cpu().numpy()) < TOL, call


def test_noalloc_refuses_requests_beyond_its_scratch(env):
    _, _lib, _, _ = env
    # 64 x 32 (batch, head) pairs need ~336 MB for one chunk each
    q = torch.zeros(64, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    beta = torch.zeros(64, 1, 32, device="cuda")
    rc, _, _ = _noalloc(env, q, q.clone(), q.clone(), beta, beta.clone(), None)
    assert rc == _lib.ERR_SCRATCH_LIMIT
    assert "no-alloc scratch" in _lib.status_string(rc)
