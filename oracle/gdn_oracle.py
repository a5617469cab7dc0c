"""CPU oracle for the chunked Gated DeltaNet forward pass.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import it; the product path
(``gdn_b200``) never does, and it has no fallback to it.

It restates, in numpy, the two definitions of the reference's ``gdn_ref.py``
(123123213weqw/v100-attention-lab):

* ``recurrent``  -- the step-by-step recurrence, ``gdn_ref.py:28-45``::

      h_t = exp(g_t) h_{t-1} + u_t k_t^T
      u_t = beta_t (v_t - exp(g_t) h_{t-1} k_t)
      o_t = h_t q_t

  with the state h stored per head as a V x K matrix (``gdn_ref.py:3-9``).

* ``chunked``    -- the chunked UT-transform form, ``gdn_ref.py:48-99``.
  Inside a chunk of C steps with b = cumsum(g):

      A[t, j] = beta_t exp(b_t - b_j) (k_t . k_j)       (j < t)
      U = (I + A)^-1 (beta v),   W = (I + A)^-1 (beta exp(b) k)
      u = U - W h0^T
      o = tril(Q K^T * exp(b_t - b_j)) u + exp(b) (Q h0^T)      (j <= t)
      h' = exp(b_C) h0 + (exp(b_C - b) u)^T K

  The last line is the algebraic simplification of the reference's
  ``h0 (exp(b_C) I - Wbar^T K) + Ubar^T K`` (``gdn_ref.py:92-98``): the
  ``h0 Wbar^T K`` term folds into ``u``.  The oracle keeps the reference's
  two-GEMM form in ``chunked(..., fold_state=False)`` so both are checked.

* ``chunk_affine`` / ``scan_affine`` -- the same chunk written as an affine
  map of its start state (the regrouping the B200 two-kernel path computes),
  and a scan that composes two chunks per state step; both are pinned to
  ``recurrent`` by the CPU tests.

Layouts follow the reference: q, k [B, T, H, K]; v [B, T, H, V]; beta, g
[B, T, H]; state [B, H, V, K] (K contiguous).  Padding follows
``pad_to_multiple`` (``gdn_ref.py:102-114``): padded steps carry q = k = v = 0,
beta = 0 and g = 0, which leaves the state unchanged and produces o = 0.

The oracle is pinned against golden vectors produced by importing the
reference itself (``tests/golden/make_golden.py``) and against the
reference's own CPU self-check (``gdn_ref.py:117-132``).
"""

from __future__ import annotations

import numpy as np

__all__ = ["l2norm", "recurrent", "chunked", "pad_to_multiple", "chunk_stages", "ns_inverse",
           "chunk_affine", "scan_affine", "make_inputs", "max_rel"]


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Row L2 normalisation along the last axis (``gdn_ref.py:24-25``)."""
    x32 = x.astype(np.float32)
    den = np.sqrt((x32 * x32).sum(-1, keepdims=True) + np.float32(eps))
    return (x32 / den).astype(x.dtype)


def _as(x, dtype):
    return np.asarray(x).astype(dtype)


def recurrent(q, k, v, beta, g, initial_state=None, dtype=np.float64):
    """Step-by-step recurrence (``gdn_ref.py:28-45``).

    Returns (o [B,T,H,V], h_final [B,H,V,K]) in ``dtype``.
    Inputs may be any float dtype; they are widened to ``dtype`` first, exactly
    as the reference widens fp16 inputs to fp32 (``gdn_ref.py:32-33``).
    """
    q = _as(q, dtype); k = _as(k, dtype); v = _as(v, dtype)
    beta = _as(beta, dtype); g = _as(g, dtype)
    B, T, H, K = q.shape
    V = v.shape[-1]
    if initial_state is None:
        h = np.zeros((B, H, V, K), dtype=dtype)
    else:
        h = _as(initial_state, dtype).copy()
    o = np.empty((B, T, H, V), dtype=dtype)
    for t in range(T):
        decay = np.exp(g[:, t])[:, :, None, None]           # [B,H,1,1]
        hd = decay * h                                       # decayed state
        hk = np.einsum("bhvk,bhk->bhv", hd, k[:, t])         # state read along k_t
        u = beta[:, t, :, None] * (v[:, t] - hk)             # delta-rule residual
        h = hd + u[..., None] * k[:, t][:, :, None, :]       # rank-1 write
        o[:, t] = np.einsum("bhvk,bhk->bhv", h, q[:, t])
    return o, h


def _unit_lower_solve(M, R):
    """Solve M X = R for unit lower-triangular M (batched, forward substitution)."""
    C = M.shape[-1]
    X = np.array(R, copy=True)
    for i in range(1, C):
        X[..., i, :] -= np.einsum("...j,...jn->...n", M[..., i, :i], X[..., :i, :])
    return X


def _f16(x):
    return np.asarray(x).astype(np.float16).astype(np.float64)


def ns_inverse(A, iters, final_fp32=True):
    """(I + A)^-1 by the Newton-Schulz iteration of ``gdn_triton_v2.py:58-63``.

    M = I + A and X = I - A are rounded to fp16; each of ``iters`` steps forms
    M X with fp32 accumulation, rounds 2I - M X to fp16 and sets X to
    X (2I - M X), again accumulated in fp32 and rounded to fp16.  The
    reference keeps the last X in fp16 as well; ``final_fp32=True`` keeps the
    last product in fp32, as the B200 kernel does before it splits T into a
    hi + lo pair.  The error falls as A^(2^(iters+1)) (zero once
    2^(iters+1) >= C) until the fp16 roundings bound it.
    """
    A = np.asarray(A, dtype=np.float64)
    eye = np.broadcast_to(np.eye(A.shape[-1]), A.shape)
    m16 = _f16(eye + A)
    x = _f16(eye - A)
    for i in range(iters):
        y = _f16(2.0 * eye - (m16 @ x).astype(np.float32))
        x = (x @ y).astype(np.float32).astype(np.float64)
        if i + 1 < iters or not final_fp32:
            x = _f16(x)
    return x


def chunk_stages(kc, vc, bc, gc, dtype=np.float64, ns_iters=None):
    """Per-chunk, state-independent quantities of ``gdn_ref.py:76-85``.

    kc [..., C, K], vc [..., C, V], bc/gc [..., C].  Returns a dict with
    b (cumsum of g), A (strictly lower), Tinv = (I+A)^-1, U and W.  With
    ``ns_iters`` set, Tinv comes from ``ns_inverse`` (the v2 solver) instead
    of exact forward substitution.
    """
    kc = kc.astype(dtype); vc = vc.astype(dtype)
    bc = bc.astype(dtype); gc = gc.astype(dtype)
    C = kc.shape[-2]
    b = np.cumsum(gc, axis=-1)
    kk = kc @ np.swapaxes(kc, -1, -2)
    dec = np.exp(b[..., :, None] - b[..., None, :])
    A = np.tril(kk * dec * bc[..., :, None], -1)
    eye = np.broadcast_to(np.eye(C, dtype=dtype), A.shape)
    Tinv = _unit_lower_solve(eye + A, eye) if ns_iters is None else ns_inverse(A, ns_iters).astype(dtype)
    U = Tinv @ (vc * bc[..., None])
    W = Tinv @ (kc * (bc * np.exp(b))[..., None])
    return {"b": b, "A": A, "Tinv": Tinv, "U": U, "W": W, "dec": dec}


def chunked(q, k, v, beta, g, C=64, initial_state=None, dtype=np.float64,
            fold_state=True, ns_iters=None):
    """Chunked UT-transform forward (``gdn_ref.py:48-99``).

    T must be a multiple of C (``gdn_ref.py:62``); use ``pad_to_multiple``.
    ``ns_iters`` selects the Newton-Schulz solve (``ns_inverse``).
    Returns (o [B,T,H,V], h_final [B,H,V,K]) in ``dtype``.
    """
    q = _as(q, dtype); k = _as(k, dtype); v = _as(v, dtype)
    beta = _as(beta, dtype); g = _as(g, dtype)
    B, T, H, K = q.shape
    V = v.shape[-1]
    if T % C != 0:
        raise ValueError(f"T={T} is not a multiple of C={C}; pad first")
    h = (np.zeros((B, H, V, K), dtype=dtype) if initial_state is None
         else _as(initial_state, dtype).copy())
    o = np.empty((B, T, H, V), dtype=dtype)
    for c0 in range(0, T, C):
        # [B,T,H,*] -> [B,H,C,*] per chunk, as in gdn_ref.py:71-75
        qc = q[:, c0:c0 + C].transpose(0, 2, 1, 3)
        kc = k[:, c0:c0 + C].transpose(0, 2, 1, 3)
        vc = v[:, c0:c0 + C].transpose(0, 2, 1, 3)
        bc = beta[:, c0:c0 + C].transpose(0, 2, 1)
        gc = g[:, c0:c0 + C].transpose(0, 2, 1)
        st = chunk_stages(kc, vc, bc, gc, dtype, ns_iters)
        b, U, W, dec = st["b"], st["U"], st["W"], st["dec"]
        u = U - np.einsum("bhck,bhvk->bhcv", W, h)
        P = np.tril((qc @ np.swapaxes(kc, -1, -2)) * dec)
        oc = P @ u + np.einsum("bhck,bhvk->bhcv", qc * np.exp(b)[..., None], h)
        o[:, c0:c0 + C] = oc.transpose(0, 2, 1, 3)
        bC = b[..., -1:]
        if fold_state:
            ubar = u * np.exp(bC - b)[..., None]
            h = np.exp(bC)[..., None] * h + np.einsum("bhcv,bhck->bhvk", ubar, kc)
        else:
            Wb = W * np.exp(bC - b)[..., None]
            Ub = U * np.exp(bC - b)[..., None]
            WtK = np.einsum("bhck,bhcl->bhkl", Wb, kc)
            eyeK = np.eye(K, dtype=dtype)
            h = (np.einsum("bhvk,bhkl->bhvl", h, np.exp(bC)[..., None] * eyeK - WtK)
                 + np.einsum("bhcv,bhck->bhvk", Ub, kc))
    return o, h


def chunk_affine(qc, kc, vc, bc, gc, dtype=np.float64):
    """The chunk as an affine map of its start state S = h^T (K x V), the form
    the two-kernel path computes (``gdn_ref.py:86-98`` regrouped):

        S' = gamma S + N S + c          N = -Kbar^T W,  c = Kbar^T U
        o  = Q' S + o_intra             Q' = Qhat - P W,  o_intra = P U

    with Kbar = exp(b_C - b) k, Qhat = exp(b) q, P = tril(Q K^T * exp(b_t - b_j))
    and gamma = exp(b_C).  Inputs per chunk as in ``chunk_stages``.
    """
    qc = qc.astype(dtype)
    st = chunk_stages(kc, vc, bc, gc, dtype)
    b, U, W, dec = st["b"], st["U"], st["W"], st["dec"]
    kc = kc.astype(dtype)
    bC = b[..., -1:]
    kbar_t = np.swapaxes(kc * np.exp(bC - b)[..., None], -1, -2)
    P = np.tril((qc @ np.swapaxes(kc, -1, -2)) * dec)
    return {"gamma": np.exp(bC[..., 0]), "N": -(kbar_t @ W), "c": kbar_t @ U,
            "Qp": qc * np.exp(b)[..., None] - P @ W, "o_intra": P @ U}


def scan_affine(q, k, v, beta, g, C=64, initial_state=None, pairs=False, dtype=np.float64):
    """Forward through ``chunk_affine``: one state step per chunk, or with
    ``pairs`` one step per two chunks composed ahead of the scan:

        N_pair = g2 N1 + g1 N2 + N2 N1     c_pair = g2 c1 + N2 c1 + c2
        Q''_2  = g1 Q'_2 + Q'_2 N1         o''_2  = o_intra_2 + Q'_2 c1
        S_next = g1 g2 S + N_pair S + c_pair,  o_1 = Q'_1 S + o_intra_1,  o_2 = Q''_2 S + o''_2

    (M_i = g_i I + N_i; M2 M1 = g1 g2 I + N_pair).  T must be a multiple of C;
    an odd number of chunks ends with a single step.  Returns (o, h_final).
    """
    q, k, v, beta, g = (_as(x, dtype) for x in (q, k, v, beta, g))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if T % C != 0:
        raise ValueError(f"T={T} is not a multiple of C={C}; pad first")
    nt = T // C
    tr = lambda x: np.moveaxis(x.reshape((B, nt, C) + x.shape[2:]), 3, 1)  # [B,H,nt,C,...]
    aff = chunk_affine(tr(q), tr(k), tr(v), tr(beta), tr(g), dtype)
    S = (np.zeros((B, H, K, V), dtype=dtype) if initial_state is None
         else np.swapaxes(_as(initial_state, dtype), -1, -2).copy())
    o = np.empty((B, H, nt, C, V), dtype=dtype)
    at = lambda name, i: aff[name][:, :, i]
    i = 0
    while i < nt:
        if pairs and i + 1 < nt:
            g1, g2 = at("gamma", i)[..., None, None], at("gamma", i + 1)[..., None, None]
            N1, N2, c1, c2 = at("N", i), at("N", i + 1), at("c", i), at("c", i + 1)
            Qp2 = at("Qp", i + 1)
            o[:, :, i] = at("Qp", i) @ S + at("o_intra", i)
            o[:, :, i + 1] = (g1 * Qp2 + Qp2 @ N1) @ S + at("o_intra", i + 1) + Qp2 @ c1
            S = g1 * g2 * S + (g2 * N1 + g1 * N2 + N2 @ N1) @ S + (g2 * c1 + N2 @ c1 + c2)
            i += 2
        else:
            o[:, :, i] = at("Qp", i) @ S + at("o_intra", i)
            S = at("gamma", i)[..., None, None] * S + at("N", i) @ S + at("c", i)
            i += 1
    o = np.moveaxis(o, 1, 3).reshape(B, T, H, V)
    return o, np.swapaxes(S, -1, -2)


def pad_to_multiple(q, k, v, beta, g, C):
    """Zero-pad T to a multiple of C (``gdn_ref.py:102-114``)."""
    B, T, H, K = q.shape
    Tp = -(-T // C) * C
    if Tp == T:
        return q, k, v, beta, g
    p = Tp - T

    def padt(x):
        w = [(0, 0)] * x.ndim
        w[1] = (0, p)
        return np.pad(x, w)

    return padt(q), padt(k), padt(v), padt(beta), padt(g)


def make_inputs(B, T, H, K, V, seed=0, gate_mean=0.0, h0_std=None, key_corr=0.0):
    """Seeded synthetic float32 inputs with the benchmark workloads' distributions.

    q, k = l2norm(N(0,1)) along K; v = N(0,1); beta = sigmoid(N(0,1));
    g = logsigmoid(N(gate_mean, 1)); h0 = N(0, h0_std) or None.
    ``key_corr`` > 0 adds key_corr times a per-head direction c ~ N(0,1)^K to
    every key before its normalisation, so that keys correlate as in trained
    models and the entries of A grow (0.56 at most for key_corr = 2 instead
    of 0.12); the other inputs keep the same draws.
    """
    rng = np.random.default_rng(seed)
    q = l2norm(rng.standard_normal((B, T, H, K), dtype=np.float32))
    k_raw = rng.standard_normal((B, T, H, K), dtype=np.float32)
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    z = rng.standard_normal((B, T, H), dtype=np.float32)
    beta = (1.0 / (1.0 + np.exp(-z))).astype(np.float32)
    z = rng.standard_normal((B, T, H), dtype=np.float32) + np.float32(gate_mean)
    g = (-np.logaddexp(0.0, -z)).astype(np.float32)              # logsigmoid
    h0 = None
    if h0_std is not None:
        h0 = (rng.standard_normal((B, H, V, K), dtype=np.float32) * np.float32(h0_std))
    if key_corr:
        k_raw = k_raw + np.float32(key_corr) * rng.standard_normal((1, 1, H, K), dtype=np.float32)
    return q, l2norm(k_raw), v, beta, g, h0


def max_rel(x, ref):
    """max|x - ref| / max|ref| -- the reference's error metric (bench_gdn.py:90-93)."""
    x = np.asarray(x, dtype=np.float64); ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(x - ref).max() / (den if den > 0 else 1.0))


if __name__ == "__main__":
    # Same self-check as gdn_ref.py:117-132 (chunked vs recurrent on CPU).
    q, k, v, beta, g, _ = make_inputs(2, 128, 3, 64, 64, seed=0)
    o1, h1 = recurrent(q, k, v, beta, g)
    o2, h2 = chunked(q, k, v, beta, g, C=32)
    print("o err", np.abs(o1 - o2).max(), "h err", np.abs(h1 - h2).max())
