"""The reference's chunked CPU path, restated in PyTorch fp32: the CPU baseline.

TEST AND MEASUREMENT INFRASTRUCTURE ONLY.  ``bench.py`` times this function on
the host cores (its ``cpu_baseline`` leg and its ``--impl reference`` arm) and
``tests/test_oracle.py`` pins it to the golden vectors that the reference
itself produced.  The product path (``gdn_b200``) never imports it.

What it restates: ``gdn_chunk_ref`` of the reference's ``gdn_ref.py``
(``gdn_ref.py:48-99``), the chunked UT-transform forward that the north star
names as the CPU path to time next to the GPU.  The reference is a Python file
that cannot travel to the GPU box, so this is a restatement of the same
sequence of torch operations, chunk after chunk, with the same arithmetic type
(fp32) and the same library calls -- two unit-lower-triangular solves per
chunk (``gdn_ref.py:84-85``) and the two-GEMM state update
(``gdn_ref.py:92-98``) -- so that its time is the reference's time on the same
host.  Nothing in it is optimised beyond the reference: it is a baseline.

Per chunk of C steps, with b the in-chunk cumulative sum of g
(``gdn_ref.py:76``):

    A      = tril(beta_t exp(b_t - b_j) k_t.k_j, -1)               :77-80
    U, W   = (I + A)^-1 [beta v],  (I + A)^-1 [beta exp(b) k]     :81-85
    u      = U - W h^T                                             :86
    o      = tril(exp(b_t - b_j) q_t.k_j) u + exp(b) q h^T          :87-91
    h'     = h (exp(b_C) I - Wbar^T K) + Ubar^T K                  :93-98

Layouts are the reference's: q, k [B, T, H, K]; v [B, T, H, V]; beta, g
[B, T, H]; the state [B, H, V, K].  T must be a multiple of C (the reference
asserts the same, ``gdn_ref.py:62``); callers pad with ``pad_to_multiple``.
"""

from __future__ import annotations

import torch

__all__ = ["chunked_fp32"]


def chunked_fp32(q, k, v, beta, g, C: int = 64, initial_state=None):
    """The chunked forward in fp32 on the tensors' device (the CPU, here).

    Returns (o [B, T, H, V] fp32, h_final [B, H, V, K] fp32).
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    if T % C:
        raise ValueError(f"T = {T} is not a multiple of C = {C}; pad first (gdn_ref.py:62)")
    f32 = torch.float32
    dev = q.device
    # [B, H, T, *] views, so that every chunk below is a batched matrix per (b, h)
    qh, kh, vh = (x.to(f32).transpose(1, 2) for x in (q, k, v))
    bh, gh = (x.to(f32).transpose(1, 2) for x in (beta, g))
    state = (torch.zeros(B, H, V, K, dtype=f32, device=dev) if initial_state is None
             else initial_state.to(f32).clone())
    out = torch.empty(B, H, T, V, dtype=f32, device=dev)
    unit = torch.eye(C, dtype=f32, device=dev)
    ident_k = torch.eye(K, dtype=f32, device=dev)
    strict = torch.ones(C, C, dtype=torch.bool, device=dev).tril(-1)
    causal = torch.ones(C, C, dtype=torch.bool, device=dev).tril(0)
    for t0 in range(0, T, C):
        sl = slice(t0, t0 + C)
        qc, kc, vc = qh[:, :, sl], kh[:, :, sl], vh[:, :, sl]      # [B, H, C, *]
        bc = bh[:, :, sl]                                            # [B, H, C]
        cum = gh[:, :, sl].cumsum(-1)                                # b
        decay = (cum.unsqueeze(-1) - cum.unsqueeze(-2)).exp()        # exp(b_t - b_j)
        gram = kc @ kc.transpose(-1, -2)                             # k_t . k_j
        a_mat = torch.where(strict, gram * decay * bc.unsqueeze(-1), 0.0)
        lower = unit + a_mat                                         # unit lower triangular
        u_rhs = vc * bc.unsqueeze(-1)
        w_rhs = kc * (bc * cum.exp()).unsqueeze(-1)
        u_sol = torch.linalg.solve_triangular(lower, u_rhs, upper=False, unitriangular=True)
        w_sol = torch.linalg.solve_triangular(lower, w_rhs, upper=False, unitriangular=True)
        upd = u_sol - w_sol @ state.transpose(-1, -2)                # u = U - W h^T
        attn = torch.where(causal, (qc @ kc.transpose(-1, -2)) * decay, 0.0)
        out[:, :, sl] = attn @ upd + (qc * cum.exp().unsqueeze(-1)) @ state.transpose(-1, -2)
        tail = cum[:, :, -1:]                                        # b_C
        to_end = (tail - cum).exp().unsqueeze(-1)                    # exp(b_C - b_t)
        w_bar, u_bar = w_sol * to_end, u_sol * to_end
        transition = tail.exp().unsqueeze(-1) * ident_k - w_bar.transpose(-1, -2) @ kc   # [B, H, K, K]
        state = state @ transition + u_bar.transpose(-1, -2) @ kc
    return out.transpose(1, 2), state
