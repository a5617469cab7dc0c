"""Host-side behaviour of the FLA-compatible entries and the input-prep
options: argument errors raised before any device work."""

import pytest
import torch


def _inputs(H=2, HV=2, B=1, T=8, K=128, V=128):
    q = torch.zeros(B, T, H, K, dtype=torch.bfloat16)
    v = torch.zeros(B, T, HV, V, dtype=torch.bfloat16)
    b = torch.zeros(B, T, HV)
    return q, q.clone(), v, b.clone(), b


def test_prep_flags():
    from gdn_b200 import _lib, ops
    assert ops._prep_flags(False, None, None) == 0
    assert ops._prep_flags(True, "sigmoid", "logsigmoid") == (_lib.FLAG_QK_L2NORM | _lib.FLAG_BETA_SIGMOID
                                                              | _lib.FLAG_G_LOGSIGMOID)
    with pytest.raises(ValueError):
        ops._prep_flags(False, "relu", None)
    with pytest.raises(ValueError):
        ops._prep_flags(False, None, "softplus")
    assert ops._prep_flags(False, None, None, "newton_schulz", 3) == _lib.FLAG_SOLVER_NS | (3 << _lib.NS_ITERS_SHIFT)
    with pytest.raises(ValueError):
        ops._prep_flags(False, None, None, "newton_schulz", 0)
    with pytest.raises(ValueError):
        ops._prep_flags(False, None, None, "cholesky")


def test_grouped_value_heads_not_supported():
    from gdn_b200 import chunk_gated_delta_rule
    q, k, v, g, b = _inputs(H=2, HV=4)
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(q, k, v, g, b)


def test_unsupported_keywords():
    from gdn_b200 import chunk_delta_rule, chunk_gated_delta_rule
    q, k, v, g, b = _inputs()
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(q, k, v, g, b, use_gate_in_kernel=True)
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(q, k, v, g, b, head_first=True)
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(q, k, v, g, b, cp_context=object())
    with pytest.raises(TypeError):
        chunk_delta_rule(q, k, v, b, bogus=1)


def test_cpu_tensors_rejected_before_device_work():
    from gdn_b200 import chunk_delta_rule, gdn_chunk_fwd
    q, k, v, g, b = _inputs()
    with pytest.raises(ValueError):
        gdn_chunk_fwd(q, k, v, b, None)
    with pytest.raises(ValueError):
        chunk_delta_rule(q, k, v, b)


def test_varlen_needs_batch_one():
    from gdn_b200 import chunk_gated_delta_rule
    q, k, v, g, b = _inputs(B=2)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q, k, v, g, b, cu_seqlens=torch.tensor([0, 4, 8]))
