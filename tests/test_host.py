"""Host-side argument handling of gdn_b200.gdn_chunk_fwd (no GPU needed):
bad shapes, dtypes and devices raise before any launch, as the reference's
callers expect Python exceptions (gdn_ref.py:62, bench_gdn.py:76-80)."""

import pytest
import torch

import gdn_b200


def inputs(B=1, T=64, H=2, K=128, V=128, dtype=torch.bfloat16):
    q = torch.zeros(B, T, H, K, dtype=dtype)
    k = torch.zeros(B, T, H, K, dtype=dtype)
    v = torch.zeros(B, T, H, V, dtype=dtype)
    beta = torch.zeros(B, T, H)
    g = torch.zeros(B, T, H)
    return q, k, v, beta, g


def test_cpu_tensors_rejected():
    with pytest.raises(ValueError, match="CUDA"):
        gdn_b200.gdn_chunk_fwd(*inputs())


def test_shape_mismatch_rejected():
    q, k, v, beta, g = inputs()
    with pytest.raises(ValueError, match="k shape"):
        gdn_b200.gdn_chunk_fwd(q, k[:, :32], v, beta, g)
    with pytest.raises(ValueError, match="v shape"):
        gdn_b200.gdn_chunk_fwd(q, k, v[:, :, :1], beta, g)
    with pytest.raises(ValueError, match="beta and g"):
        gdn_b200.gdn_chunk_fwd(q, k, v, beta[:, :, :1], g)


def test_rank_and_dtype_checks():
    q, k, v, beta, g = inputs()
    with pytest.raises(ValueError):
        gdn_b200.gdn_chunk_fwd(q[0], k, v, beta, g)
    with pytest.raises(ValueError, match="share a dtype"):
        gdn_b200.gdn_chunk_fwd(q, k.half(), v, beta, g)
    with pytest.raises(NotImplementedError):
        gdn_b200.gdn_chunk_fwd(q.float(), k.float(), v.float(), beta, g)


def test_noncontiguous_last_dim_rejected():
    q, k, v, beta, g = inputs()
    qt = q.transpose(2, 3).contiguous().transpose(2, 3)
    with pytest.raises(ValueError, match="contiguous last"):
        gdn_b200.gdn_chunk_fwd(qt, k, v, beta, g)


def test_not_tensor_rejected():
    q, k, v, beta, g = inputs()
    with pytest.raises(TypeError):
        gdn_b200.gdn_chunk_fwd(q, k, v, beta, g.numpy())


def test_v2_signature_is_keyword_compatible():
    """gdn_chunk_fwd_v2(q,k,v,beta,g,C,BV,num_warps,num_stages,iters) (gdn_triton_v2.py:92)."""
    import inspect
    params = list(inspect.signature(gdn_b200.gdn_chunk_fwd_v2).parameters)
    assert params[:10] == ["q", "k", "v", "beta", "g", "C", "BV", "num_warps", "num_stages", "iters"]
    with pytest.raises(ValueError, match="CUDA"):
        gdn_b200.gdn_chunk_fwd_v2(*inputs(), C=64, BV=32, num_warps=4, num_stages=1, iters=2)


def test_fixed_signature_matches_reference():
    """gdn_chunk_fwd_fixed(q,k,v,beta,g,C=32,BV=32,num_warps=4,num_stages=1) (bench_gdn.py:43)."""
    import inspect
    sig = inspect.signature(gdn_b200.gdn_chunk_fwd_fixed)
    params = list(sig.parameters)
    assert params[:9] == ["q", "k", "v", "beta", "g", "C", "BV", "num_warps", "num_stages"]
    assert sig.parameters["C"].default == 32 and sig.parameters["BV"].default == 32
    assert inspect.signature(gdn_b200.gdn_chunk_fwd_v2).parameters["C"].default == 32
    with pytest.raises(ValueError, match="CUDA"):
        gdn_b200.gdn_chunk_fwd_fixed(*inputs())
