"""The CPU oracle pinned against the reference's own outputs (tests/golden).

The fixtures were produced by running the reference's gdn_ref.py
(tests/golden/make_golden.py); these tests check that oracle/gdn_oracle.py,
the checker every GPU parity test uses, reproduces them.
"""

import os

import numpy as np
import pytest

from oracle import gdn_oracle as ora

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def test_selfcheck_case_matches_reference():
    """gdn_ref.py:117-132 inputs: recurrence and chunked path of the reference."""
    d = load("selfcheck")
    o, h = ora.recurrent(d["q"], d["k"], d["v"], d["beta"], d["g"], dtype=np.float64)
    assert np.abs(o - d["o_rec"]).max() < 1e-5
    assert np.abs(h - d["h_rec"]).max() < 1e-5
    o2, h2 = ora.chunked(d["q"], d["k"], d["v"], d["beta"], d["g"], C=int(d["C"]), dtype=np.float64)
    assert np.abs(o2 - d["o_chunk"]).max() < 1e-5
    assert np.abs(h2 - d["h_chunk"]).max() < 1e-5
    # the reference's own acceptance bound for chunked vs recurrent (gdn_ref.py:130-131)
    assert np.abs(d["o_rec"] - d["o_chunk"]).max() < 1e-3


def test_config0_matches_reference():
    d = load("cfg0")
    o, h = ora.recurrent(d["q"], d["k"], d["v"], d["beta"], d["g"], dtype=np.float64)
    assert ora.max_rel(o, d["o_rec"]) < 1e-5 and ora.max_rel(h, d["h_rec"]) < 1e-5
    o2, h2 = ora.chunked(d["q"], d["k"], d["v"], d["beta"], d["g"], C=32, dtype=np.float32)
    assert ora.max_rel(o2, d["o_chunk"]) < 1e-5 and ora.max_rel(h2, d["h_chunk"]) < 1e-5


def test_initial_state_case():
    d = load("h0_f16")
    o, h = ora.recurrent(d["q"], d["k"], d["v"], d["beta"], d["g"], initial_state=d["h0"], dtype=np.float64)
    assert ora.max_rel(o, d["o_rec"]) < 1e-9 and ora.max_rel(h, d["h_rec"]) < 1e-9
    o2, h2 = ora.chunked(d["q"], d["k"], d["v"], d["beta"], d["g"], C=64, initial_state=d["h0"])
    assert ora.max_rel(o2, d["o_chunk"]) < 1e-5 and ora.max_rel(h2, d["h_chunk"]) < 1e-5


def test_ragged_T_padding_rule():
    """pad_to_multiple (gdn_ref.py:102-114): padded steps leave the state alone."""
    d = load("bf16_ragged")
    q, k, v, b, g = ora.pad_to_multiple(d["q"], d["k"], d["v"], d["beta"], d["g"], 64)
    assert q.shape[1] == 128
    o, h = ora.chunked(q, k, v, b, g, C=64)
    assert ora.max_rel(o, d["o_chunk_padded"]) < 1e-5
    assert ora.max_rel(h, d["h_chunk"]) < 1e-5
    T = d["q"].shape[1]
    assert ora.max_rel(o[:, :T], d["o_rec"]) < 1e-5
    assert ora.max_rel(h, d["h_rec"]) < 1e-5
    assert np.abs(o[:, T:]).max() < 1e-6   # padded q = 0 -> o = 0


def test_stage_intermediates():
    """U and W captured from the reference's two solve_triangular calls."""
    d = load("stages")
    q, k, v, b, g = (d[n] for n in ("q", "k", "v", "beta", "g"))
    for c in range(d["U"].shape[0]):
        sl = slice(64 * c, 64 * c + 64)
        st = ora.chunk_stages(k[:, sl].transpose(0, 2, 1, 3), v[:, sl].transpose(0, 2, 1, 3),
                              b[:, sl].transpose(0, 2, 1), g[:, sl].transpose(0, 2, 1))
        assert ora.max_rel(st["U"], d["U"][c]) < 1e-5
        assert ora.max_rel(st["W"], d["W"][c]) < 1e-5
        # (I + A) is unit lower triangular and Tinv really inverts it
        eye = np.eye(64)
        assert np.abs((eye + st["A"]) @ st["Tinv"] - eye).max() < 1e-9


def test_state_update_forms_agree():
    """The folded update h' = e^{b_C} h + (e^{b_C-b} u)^T K equals the
    reference's h (e^{b_C} I - Wbar^T K) + Ubar^T K (gdn_ref.py:92-98)."""
    q, k, v, b, g, h0 = ora.make_inputs(1, 128, 2, 32, 48, seed=4, h0_std=0.3)
    o1, h1 = ora.chunked(q, k, v, b, g, C=32, initial_state=h0, fold_state=True)
    o2, h2 = ora.chunked(q, k, v, b, g, C=32, initial_state=h0, fold_state=False)
    assert ora.max_rel(o1, o2) < 1e-12 and ora.max_rel(h1, h2) < 1e-12


@pytest.mark.parametrize("C", [16, 32, 64])
def test_chunk_size_invariance(C):
    q, k, v, b, g, h0 = ora.make_inputs(1, 128, 1, 16, 16, seed=C, h0_std=0.1)
    o_r, h_r = ora.recurrent(q, k, v, b, g, initial_state=h0)
    o_c, h_c = ora.chunked(q, k, v, b, g, C=C, initial_state=h0)
    assert ora.max_rel(o_c, o_r) < 1e-10 and ora.max_rel(h_c, h_r) < 1e-10


def test_state_chaining_property():
    """Splitting the sequence and passing the state gives the same result."""
    q, k, v, b, g, h0 = ora.make_inputs(1, 96, 2, 16, 16, seed=9, h0_std=0.1)
    o, h = ora.recurrent(q, k, v, b, g, initial_state=h0)
    oa, ha = ora.recurrent(q[:, :40], k[:, :40], v[:, :40], b[:, :40], g[:, :40], initial_state=h0)
    ob, hb = ora.recurrent(q[:, 40:], k[:, 40:], v[:, 40:], b[:, 40:], g[:, 40:], initial_state=ha)
    assert ora.max_rel(np.concatenate([oa, ob], 1), o) < 1e-12 and ora.max_rel(hb, h) < 1e-12


def test_planted_mistake_is_caught():
    """A deliberately wrong oracle variant (decay off by one step) must fail the bar."""
    q, k, v, b, g, _ = ora.make_inputs(1, 64, 1, 16, 16, seed=1)
    o_r, _ = ora.recurrent(q, k, v, b, g)
    g_shift = np.roll(g, 1, axis=1)
    o_bad, _ = ora.recurrent(q, k, v, b, g_shift)
    assert ora.max_rel(o_bad, o_r) > 1e-3


def test_newton_schulz_restatement():
    """ns_inverse follows gdn_triton_v2.py:58-63: X0 = I - A and
    X <- X (2I - (I + A) X), so after one step I - (I + A) X = A^4 and after n
    steps A^(2^(n+1)), up to the fp16 roundings; the error vs the exact
    inverse falls until those roundings bound it."""
    q, k, v, b, g, _ = ora.make_inputs(1, 128, 2, 128, 16, seed=5, key_corr=2.0)
    st = ora.chunk_stages(k[:, :64].transpose(0, 2, 1, 3), v[:, :64].transpose(0, 2, 1, 3),
                          b[:, :64].transpose(0, 2, 1), g[:, :64].transpose(0, 2, 1))
    A, Tinv = st["A"], st["Tinv"]
    eye = np.eye(64)
    assert np.abs(A).max() > 0.3            # large enough for the iterations to matter
    x1 = ora.ns_inverse(A, 1)
    a4 = np.linalg.matrix_power(A[0, 0], 4)
    assert np.abs((eye - (eye + A[0, 0]) @ x1[0, 0]) - a4).max() < 4e-3 * np.abs(a4).max() + 2e-3
    errs = [ora.max_rel(ora.ns_inverse(A, n), Tinv) for n in range(1, 7)]
    assert errs[0] > 10 * errs[1] > 10 * errs[2]
    assert max(errs[2:]) < 1e-3              # fp16 floor from the third step on (A^16 is below it)
    # exact solver path of the chunked oracle unchanged; NS path converges to it
    o_ex, _ = ora.chunked(q, k, v, b, g)
    o_ns, _ = ora.chunked(q, k, v, b, g, ns_iters=5)
    assert 0 < ora.max_rel(o_ns, o_ex) < 1e-3


@pytest.mark.parametrize("pairs", [False, True])
@pytest.mark.parametrize("T", [256, 192])  # 4 chunks; 3 chunks (a single step at the end)
def test_affine_scan_equals_recurrence(pairs, T):
    """The two-kernel path's regrouped per-chunk affine form, and the same with
    two chunks composed per state step, are the step recurrence."""
    q, k, v, b, g, h0 = ora.make_inputs(2, T, 2, 32, 24, seed=T + pairs, h0_std=0.3, key_corr=1.0)
    o_r, h_r = ora.recurrent(q, k, v, b, g, initial_state=h0)
    o_a, h_a = ora.scan_affine(q, k, v, b, g, C=64, initial_state=h0, pairs=pairs)
    assert ora.max_rel(o_a, o_r) < 1e-10 and ora.max_rel(h_a, h_r) < 1e-10


@pytest.mark.parametrize("name", ["selfcheck", "cfg0", "h0_f16", "stages"])
def test_torch_chunked_restatement_matches_reference(name):
    """The CPU baseline (oracle/gdn_chunk_torch.py, the reference's chunked
    path restated in torch fp32) reproduces the reference's own chunked outputs."""
    import torch
    from oracle.gdn_chunk_torch import chunked_fp32
    d = load(name)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x))
    h0 = t(d["h0"]) if "h0" in d else None
    o, h = chunked_fp32(t(d["q"]), t(d["k"]), t(d["v"]), t(d["beta"]), t(d["g"]), C=int(d["C"]), initial_state=h0)
    assert o.dtype == torch.float32 and h.dtype == torch.float32
    assert ora.max_rel(o.numpy(), d["o_chunk"]) < 1e-5
    assert ora.max_rel(h.numpy(), d["h_chunk"]) < 1e-5


def test_torch_chunked_restatement_needs_whole_chunks():
    import torch
    from oracle.gdn_chunk_torch import chunked_fp32
    x = torch.zeros(1, 100, 1, 64)
    b = torch.zeros(1, 100, 1)
    with pytest.raises(ValueError):
        chunked_fp32(x, x, x, b, b, C=64)
