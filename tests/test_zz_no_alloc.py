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


def _sampled_oracle(qd, kd, vd, bd, gd, h0, pairs):
    """fp64 step recurrence of the CPU oracle on single (batch, head) pairs."""
    from gpu_util import oracle
    sl = lambda x, b, h: x[b:b + 1, :, h:h + 1]
    return [oracle(sl(qd, b, h), sl(kd, b, h), sl(vd, b, h), sl(bd, b, h), sl(gd, b, h),
                   h0[b:b + 1, h:h + 1]) for b, h in pairs]


def test_noalloc_matches_regular_entry_point_twice(env):
    from gpu_util import TOL, make, rel
    gdn, _lib, ops, _ = env
    # B*H = 32 heads and 32 chunks need ~103 MB of scratch in one piece, so
    # the 32 MiB array is used in four segments with the state carried over
    pairs = [(0, 3), (1, 14)]
    for call, seed in enumerate((51, 52)):
        qd, kd, vd, bd, gd, h0 = make(2, 2048, 16, seed=seed, dtype=torch.bfloat16, h0_std=0.1)
        rc, o, ht = _noalloc(env, qd, kd, vd, bd, gd, h0)
        assert rc == _lib.OK, (call, _lib.status_string(rc))
        ops.check_status()
        o_ref, h_ref = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0,
                                         output_dtype=torch.float32, check=True)
        assert rel(o, o_ref.cpu().numpy()) < TOL, call
        assert rel(ht, h_ref.cpu().numpy()) < TOL, call
        # and against the CPU oracle itself, on two sampled (batch, head) pairs
        for (b, h), (o_or, h_or) in zip(pairs, _sampled_oracle(qd, kd, vd, bd, gd, h0, pairs)):
            assert rel(o[b:b + 1, :, h:h + 1], o_or) < TOL, (call, b, h)
            assert rel(ht[b:b + 1, h:h + 1], h_or) < TOL, (call, b, h)


def test_noalloc_reports_unsupported_shapes_before_the_size_limit(env):
    """A shape this build does not handle (K = V = 64) is refused as
    unsupported, even when B*H alone would also exceed the scratch."""
    _, _lib, _, _ = env
    for B, H in ((1, 2), (64, 32)):
        q = torch.zeros(B, 64, H, 64, dtype=torch.bfloat16, device="cuda")
        beta = torch.zeros(B, 64, H, device="cuda")
        rc, _, _ = _noalloc(env, q, q.clone(), q.clone(), beta, beta.clone(), None)
        assert rc == _lib.ERR_UNSUPPORTED, (B, H, _lib.status_string(rc))


def test_noalloc_refuses_requests_beyond_its_scratch(env):
    _, _lib, _, _ = env
    # 64 x 32 (batch, head) pairs need ~336 MB for one chunk each
    q = torch.zeros(64, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    beta = torch.zeros(64, 1, 32, device="cuda")
    rc, _, _ = _noalloc(env, q, q.clone(), q.clone(), beta, beta.clone(), None)
    assert rc == _lib.ERR_SCRATCH_LIMIT
    assert "no-alloc scratch" in _lib.status_string(rc)
