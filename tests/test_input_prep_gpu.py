"""The q scale, the DeltaNet case (g == 0), input preparation inside the
kernel (q/k L2 norm, beta / g activations) and the FLA-compatible entries,
against the oracle on the same inputs; plus a cross-check with FLA itself
(the reference's comparator, bench_gdn.py:167-179, bench_zoo.py:107-116)
when it runs on this machine."""

import math

import numpy as np
import pytest
import torch

from gpu_util import STORE_ROUNDING, TOL, make, oracle, rel

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def gdn():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gdn_b200
    return gdn_b200


def _l2norm(x):
    """gdn_ref.py:24-25 in fp32, rounded back to the input dtype."""
    xf = x.float()
    return (xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)).to(x.dtype)


def test_scale_multiplies_q(gdn):
    qd, kd, vd, bd, gd, h0 = make(1, 300, 2, seed=61, dtype=BF16, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, scale=0.37,
                              check=True)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    assert rel(o, 0.37 * o_ref) < TOL
    assert rel(ht, h_ref) < TOL


@pytest.mark.parametrize("fused", [False, True])
def test_no_gate_is_the_deltanet_recurrence(gdn, fused):
    qd, kd, vd, bd, _, h0 = make(2, 200, 2, seed=62, dtype=torch.float16, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, None, initial_state=h0, output_dtype=torch.float32, check=True,
                              fused=fused)
    o_ref, h_ref = oracle(qd, kd, vd, bd, torch.zeros_like(bd), h0)
    assert rel(o, o_ref) < TOL
    assert rel(ht, h_ref) < TOL


@pytest.mark.parametrize("fused,T", [(False, 256), (False, 2048), (True, 256)])
def test_no_gate_bf16_long(gdn, fused, T):
    """No decay keeps every chunk's rounding in the state: the hardest case for
    the T operand precision (bf16 inputs).  The two-kernel path splits both T
    operands hi + lo and holds 4e-4 at T = 2048; the fused fallback keeps a
    single bf16 copy of T diag(beta e^b) (its shared memory is full) and
    reaches 1.1e-3 on the final state at T = 2048, so it is checked at 256."""
    qd, kd, vd, bd, _, h0 = make(1, T, 2, seed=68, dtype=BF16, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, bd, None, initial_state=h0, output_dtype=torch.float32, check=True,
                              fused=fused)
    o_ref, h_ref = oracle(qd, kd, vd, bd, torch.zeros_like(bd), h0)
    assert rel(o, o_ref) < TOL
    assert rel(ht, h_ref) < TOL


@pytest.mark.parametrize("fused", [False, True])
def test_beta_and_g_activations_in_kernel(gdn, fused):
    rng = np.random.default_rng(63)
    qd, kd, vd, _, _, h0 = make(1, 260, 3, seed=63, dtype=BF16, h0_std=0.1)
    logits = lambda: torch.from_numpy(rng.standard_normal((1, 260, 3), dtype=np.float32)).cuda()
    beta_logit, g_logit = logits(), logits()
    o, ht = gdn.gdn_chunk_fwd(qd, kd, vd, beta_logit, g_logit, initial_state=h0, output_dtype=torch.float32,
                              beta_activation="sigmoid", g_activation="logsigmoid", check=True, fused=fused)
    o_ref, h_ref = oracle(qd, kd, vd, torch.sigmoid(beta_logit), torch.nn.functional.logsigmoid(g_logit), h0)
    assert rel(o, o_ref) < TOL
    assert rel(ht, h_ref) < TOL


def test_qk_l2norm_in_kernel(gdn):
    gen = torch.Generator().manual_seed(64)
    B, T, H = 1, 330, 2
    raw_q = (3.0 * torch.randn(B, T, H, 128, generator=gen)).to(BF16).cuda()
    raw_k = (0.5 * torch.randn(B, T, H, 128, generator=gen)).to(BF16).cuda()
    _, _, vd, bd, gd, h0 = make(B, T, H, seed=64, dtype=BF16, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(raw_q, raw_k, vd, bd, gd, initial_state=h0, output_dtype=torch.float32,
                              use_qk_l2norm_in_kernel=True, check=True)
    o_ref, h_ref = oracle(_l2norm(raw_q), _l2norm(raw_k), vd, bd, gd, h0)
    assert rel(o, o_ref) < TOL
    assert rel(ht, h_ref) < TOL
    with pytest.raises(NotImplementedError):
        gdn.gdn_chunk_fwd(raw_q, raw_k, vd, bd, gd, use_qk_l2norm_in_kernel=True, fused=True)


def test_fla_entry_layouts_and_default_scale(gdn):
    qd, kd, vd, bd, gd, h0 = make(2, 200, 2, seed=65, dtype=BF16, h0_std=0.1)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    # FLA's state layout [N, H, K, V] and the reference's scale 1.0
    o, ht = gdn.chunk_gated_delta_rule(qd, kd, vd, gd, bd, scale=1.0, initial_state=h0.transpose(-1, -2).contiguous(),
                                       output_final_state=True)
    assert o.dtype == BF16 and tuple(ht.shape) == (2, 2, 128, 128)
    assert rel(o, o_ref) < TOL + STORE_ROUNDING[BF16]
    assert rel(ht.transpose(-1, -2), h_ref) < TOL
    # default scale 1/sqrt(K), gdn_ref's state layout, no final state
    o2, ht2 = gdn.chunk_gated_delta_rule(qd, kd, vd, gd, bd, initial_state=h0, transpose_state_layout=True)
    assert ht2 is None
    assert rel(o2, o_ref / math.sqrt(128)) < TOL + STORE_ROUNDING[BF16]


@pytest.mark.parametrize("lens", [[150, 77, 64], [96, 40, 96, 0, 40, 96]])
def test_fla_entry_variable_lengths(gdn, lens):
    parts = [make(1, L, 2, seed=70 + i, dtype=BF16, h0_std=0.1) for i, L in enumerate(lens)]
    cat = lambda j: torch.cat([p[j] for p in parts], dim=1)
    q, k, v, b, g = (cat(j) for j in range(5))
    h0 = torch.cat([p[5] for p in parts], dim=0)  # [N, H, V, K]
    cu = torch.tensor([0] + list(np.cumsum(lens)), device="cuda")
    o, ht = gdn.chunk_gated_delta_rule(q, k, v, g, b, scale=1.0, initial_state=h0, output_final_state=True,
                                       cu_seqlens=cu, transpose_state_layout=True)
    s = 0
    for i, p in enumerate(parts):
        if lens[i] == 0:  # an empty sequence keeps its state
            assert torch.equal(ht[i], h0[i])
            continue
        o_ref, h_ref = oracle(*p)
        assert rel(o[:, s:s + lens[i]], o_ref) < TOL + STORE_ROUNDING[BF16], i
        assert rel(ht[i:i + 1], h_ref) < TOL, i
        s += lens[i]


def test_delta_rule_entry(gdn):
    qd, kd, vd, bd, _, h0 = make(1, 190, 3, seed=66, dtype=torch.float16, h0_std=0.1)
    o, ht = gdn.chunk_delta_rule(qd, kd, vd, bd, scale=1.0, initial_state=h0.transpose(-1, -2).contiguous(),
                                 output_final_state=True)
    o_ref, h_ref = oracle(qd, kd, vd, bd, torch.zeros_like(bd), h0)
    assert rel(o, o_ref) < TOL + STORE_ROUNDING[torch.float16]
    assert rel(ht.transpose(-1, -2), h_ref) < TOL


def _fla(module, name):
    try:
        mod = __import__(module, fromlist=[name])
        return getattr(mod, name)
    except Exception as exc:  # not installed, or no Triton backend for this device
        pytest.skip(f"FLA not usable here: {exc}")


@pytest.mark.parametrize("gated", [True, False])
def test_cross_check_with_fla(gdn, gated):
    """The reference checks its kernel against FLA at scale 1.0 (bench_gdn.py:167-179,
    about 7e-4 on o).  FLA keeps 16-bit intermediates (its final state is off
    the fp64 recurrence by a few 1e-3), so each implementation is measured
    against the oracle and their difference is bounded by the sum of the two
    errors; ours must stay within the oracle tolerance."""
    fn = _fla("fla.ops.gated_delta_rule", "chunk_gated_delta_rule") if gated else \
        _fla("fla.ops.delta_rule", "chunk_delta_rule")
    qd, kd, vd, bd, gd, h0 = make(1, 256, 2, seed=67, dtype=BF16, h0_std=0.1)
    if not gated:
        gd = torch.zeros_like(bd)
    h0_kv = h0.transpose(-1, -2).contiguous()
    try:
        if gated:
            o_f, h_f = fn(q=qd, k=kd, v=vd, g=gd, beta=bd, scale=1.0, initial_state=h0_kv, output_final_state=True)
        else:
            o_f, h_f = fn(qd, kd, vd, bd, scale=1.0, initial_state=h0_kv, output_final_state=True)
        torch.cuda.synchronize()
    except Exception as exc:
        pytest.skip(f"FLA kernels did not run here: {exc}")
    if gated:
        o, h = gdn.chunk_gated_delta_rule(qd, kd, vd, gd, bd, scale=1.0, initial_state=h0_kv, output_final_state=True)
    else:
        o, h = gdn.chunk_delta_rule(qd, kd, vd, bd, scale=1.0, initial_state=h0_kv, output_final_state=True)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    h_ref_kv = h_ref.transpose(0, 1, 3, 2)
    err_o, err_h = rel(o, o_ref), rel(h, h_ref_kv)
    fla_o, fla_h = rel(o_f, o_ref), rel(h_f, h_ref_kv)
    print(f"vs fp64 recurrence: ours o {err_o:.2e} h {err_h:.2e} | FLA o {fla_o:.2e} h {fla_h:.2e}")
    assert err_o < TOL + STORE_ROUNDING[BF16]
    assert err_h < TOL
    assert rel(o, o_f.float().cpu().numpy()) < err_o + fla_o + 1e-4
    assert rel(h, h_f.float().cpu().numpy()) < err_h + fla_h + 1e-4


def test_newton_schulz_solver(gdn):
    """The reference's Newton-Schulz solve (gdn_triton_v2.py:58-68): the kernel
    follows the oracle's restatement of it (fp16 operands, fp32 accumulation)
    at every iteration count, and against the exact recurrence its error falls
    with the iterations to the fp16 floor.  Correlated keys make A large
    enough (max|A| ~ 0.56) for the iterations to matter."""
    qd, kd, vd, bd, gd, h0 = make(1, 512, 2, seed=69, dtype=BF16, h0_std=0.1, key_corr=2.0)
    o_ref, h_ref = oracle(qd, kd, vd, bd, gd, h0)
    errs = {}
    for n in (1, 2, 3, 5):
        o, h = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, check=True,
                                 solver="newton_schulz", ns_iters=n)
        o_ns, h_ns = oracle(qd, kd, vd, bd, gd, h0, ns_iters=n)
        print(f"ns_iters={n}: vs NS oracle o {rel(o, o_ns):.2e} h {rel(h, h_ns):.2e}; "
              f"vs exact o {rel(o, o_ref):.2e} (oracle's own {rel(o_ns, o_ref):.2e})")
        assert rel(o, o_ns) < TOL and rel(h, h_ns) < TOL
        errs[n] = rel(o, o_ref)
    o, h = gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, initial_state=h0, output_dtype=torch.float32, check=True)
    assert rel(o, o_ref) < TOL and rel(h, h_ref) < TOL
    assert errs[1] > 10 * errs[2] > 10 * errs[3]
    assert errs[5] < TOL
    with pytest.raises(NotImplementedError):
        gdn.gdn_chunk_fwd(qd, kd, vd, bd, gd, solver="newton_schulz", fused=True)


@pytest.mark.parametrize("solver", ["blocked", "newton_schulz"])
@pytest.mark.parametrize("in_dtype", [BF16, torch.float16])
def test_input_prep_options_combined(gdn, solver, in_dtype):
    """Every input-preparation option of one call at once (q/k L2 norm, beta
    sigmoid, g logsigmoid, a q scale) with either solver: the prep applies them
    in one pass over the chunk, so they are checked together as well as one by
    one.  Five Newton-Schulz rounds are exact for C = 64 (A^64 = 0)."""
    gen = torch.Generator().manual_seed(71)
    B, T, H = 2, 390, 3
    raw_q = (2.0 * torch.randn(B, T, H, 128, generator=gen)).to(in_dtype).cuda()
    raw_k = (0.7 * torch.randn(B, T, H, 128, generator=gen)).to(in_dtype).cuda()
    beta_logit = torch.randn(B, T, H, generator=gen).cuda()
    g_logit = (torch.randn(B, T, H, generator=gen) + 1.0).cuda()
    _, _, vd, _, _, h0 = make(B, T, H, seed=71, dtype=in_dtype, h0_std=0.1)
    o, ht = gdn.gdn_chunk_fwd(raw_q, raw_k, vd, beta_logit, g_logit, initial_state=h0, check=True, scale=0.7,
                              use_qk_l2norm_in_kernel=True, beta_activation="sigmoid", g_activation="logsigmoid",
                              solver=solver, ns_iters=5)
    assert o.dtype == in_dtype
    o_ref, h_ref = oracle(_l2norm(raw_q), _l2norm(raw_k), vd, torch.sigmoid(beta_logit),
                          torch.nn.functional.logsigmoid(g_logit), h0)
    assert rel(o, 0.7 * o_ref) < TOL + STORE_ROUNDING[in_dtype]
    assert rel(ht, h_ref) < TOL


def test_sweep_harness(gdn):
    from gdn_b200 import sweep
    lines = sweep.run(config=1, reps=3, iters=(2,))
    assert [l["solver"] for l in lines] == ["blocked", "newton_schulz"]
    assert all(l["ms_per_forward"] > 0 and l["err_o"] < 1 for l in lines)
