"""GPU parity of the fused sm_100a forward against the CPU oracle (fp64).

Every case calls the product path (gdn_b200 -> C ABI -> sm_100a kernel) and
compares with oracle/gdn_oracle.py on the same inputs.
"""

import pytest
import torch

from gpu_util import STORE_ROUNDING, TOL, make, oracle, rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gdn():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gdn_b200
    return gdn_b200


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [64, 128, 200])
@pytest.mark.parametrize("with_h0", [False, True])
def test_small_fp32_out(gdn, dtype, T, with_h0, fused):
    qd, kd, vd, bd, gd, h0 = make(1, T, 2, seed=T + with_h0, dtype=dtype, h0_std=0.1 if with_h0 else None)
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, check=True,
                              fused=fused)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    assert rel(o, o_ref) < TOL
    assert rel(ht, h_ref) < TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_output_in_input_dtype(gdn, dtype):
    qd, kd, vd, bd, gd, h0 = make(2, 256, 3, seed=11, dtype=dtype, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, check=True)
    assert o.dtype == dtype and ht.dtype == torch.float32
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    assert rel(o, o_ref) < TOL + STORE_ROUNDING[dtype]
    assert rel(ht, h_ref) < TOL


def test_wy_prep_stage(gdn):
    """W and U of every chunk (gdn_ref.py:84-85) from the chunk-parallel stage."""
    import numpy as np
    from oracle import gdn_oracle as ora
    qd, kd, vd, bd, gd, _ = make(1, 192, 2, seed=5, dtype=torch.float16)
    W, U = gdn.gdn_wy_prep(qd, kd, vd, bd, gd)
    f = lambda x: x.float().cpu().numpy()
    k, v, b, g = f(kd), f(vd), f(bd), f(gd)
    B, T, H, _ = k.shape
    for c in range(T // 64):
        sl = slice(64 * c, 64 * c + 64)
        st = ora.chunk_stages(k[:, sl].transpose(0, 2, 1, 3), v[:, sl].transpose(0, 2, 1, 3),
                              b[:, sl].transpose(0, 2, 1), g[:, sl].transpose(0, 2, 1))
        assert ora.max_rel(f(W[:, :, c]), st["W"]) < 5e-3   # W uses input-dtype operands
        assert ora.max_rel(f(U[:, :, c]), st["U"]) < 1e-4   # U uses the hi+lo split


def test_two_kernel_and_fused_paths_both_match_oracle(gdn):
    """The two-kernel path (state update regrouped as e^{b_C} S + N S + c) and
    the fused single-kernel path round differently; each meets the tolerance
    against the oracle on the same inputs, and they agree with each other to
    within twice that."""
    qd, kd, vd, bd, gd, h0 = make(2, 700, 3, seed=41, dtype=torch.bfloat16, h0_std=0.1)
    o1, h1 = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, check=True)
    o2, h2 = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, check=True,
                               fused=True)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    for o, h in ((o1, h1), (o2, h2)):
        assert rel(o, o_ref) < TOL
        assert rel(h, h_ref) < TOL
    assert rel(o1, o2.float().cpu().numpy()) < 2 * TOL


@pytest.mark.parametrize("cap_chunks", [1, 3])
def test_segmented_workspace(gdn, cap_chunks, monkeypatch):
    """A workspace smaller than the sequence: several prep/scan segments with
    the state carried between them."""
    from gdn_b200 import _lib, ops
    B, H = 1, 2
    cap = _lib.WORKSPACE_HEADER_BYTES + B * H * (cap_chunks * _lib.PACKET_BYTES_PER_CHUNK + 128 * 128 * 4)
    monkeypatch.setattr(ops, "WORKSPACE_CAP_BYTES", cap)
    monkeypatch.setattr(ops, "_workspaces", {})
    qd, kd, vd, bd, gd, h0 = make(B, 450, H, seed=42, dtype=torch.float16, h0_std=0.1)
    for want_state in (True, False):
        o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32,
                                  output_final_state=want_state, check=True)
        o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
        assert rel(o, o_ref) < TOL
        if want_state:
            assert rel(ht, h_ref) < TOL
        else:
            assert ht is None


def test_two_streams_at_once(gdn):
    """Forwards queued on two streams at the same time: each stream has its own
    scratch, so the prep of one and the scan of the other may overlap on the
    GPU without touching each other's packets.  Both match the oracle, and
    equal (bit for bit) the same forwards run one after the other."""
    from gdn_b200 import ops
    a = make(1, 1000, 4, seed=61, dtype=torch.bfloat16, h0_std=0.1)
    b = make(2, 640, 3, seed=62, dtype=torch.float16, h0_std=0.1)
    seq = [gdn.gdn_chunk_fwd(*x[:5], initial_state=x[5], output_dtype=torch.float32, check=True) for x in (a, b)]
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    res = []
    for _ in range(4):  # several rounds, so that kernels of the two streams interleave
        with torch.cuda.stream(s1):
            ra = gdn.gdn_chunk_fwd(*a[:5], initial_state=a[5], output_dtype=torch.float32)
        with torch.cuda.stream(s2):
            rb = gdn.gdn_chunk_fwd(*b[:5], initial_state=b[5], output_dtype=torch.float32)
        res.append((ra, rb))
    torch.cuda.synchronize()
    ops.check_status()
    keys = [k for k in ops._workspaces if k[1] in (s1.cuda_stream, s2.cuda_stream)]
    assert len(keys) == 2  # one scratch buffer per stream
    for x, (o_seq, h_seq), k in ((a, seq[0], 0), (b, seq[1], 1)):
        o_ref, h_ref = oracle(*x)
        for r in res:
            o, h = r[k]
            assert torch.equal(o, o_seq) and torch.equal(h, h_seq)
        assert rel(o_seq, o_ref) < TOL and rel(h_seq, h_ref) < TOL
