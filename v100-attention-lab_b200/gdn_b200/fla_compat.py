"""FLA-compatible keyword entries backed by the B200 forward.

The reference compares its kernel with flash-linear-attention by calling

    fla.ops.gated_delta_rule.chunk_gated_delta_rule(q=, k=, v=, g=, beta=, scale=1.0, ...)
    fla.ops.delta_rule.chunk_delta_rule(q, k, v, beta, ...)        (the g == 0 case)

(bench_gdn.py:102-108,167-179; bench_zoo.py:107-116).  These functions take
the same arguments, in FLA's order (q, k, v, g, beta) and with its defaults, so
they drop in where those are called:

* ``scale`` defaults to 1/sqrt(K) (FLA); the reference passes 1.0;
* states are ``[N, H, K, V]`` (FLA) unless ``transpose_state_layout=True``,
  which selects ``[N, H, V, K]``, the layout of gdn_ref / gdn_triton;
* ``use_qk_l2norm_in_kernel`` normalises q and k rows inside the kernel;
* ``cu_seqlens`` (variable-length batches, B = 1) runs one batched forward
  per distinct sequence length (equal-length sequences gathered into one
  batch; a length that occurs once runs on views of the packed tensors).

Forward only.  Grouped value heads (v with more heads than q), the in-kernel
gate of newer FLA releases (``use_gate_in_kernel``) and context parallelism
are not provided and raise ``NotImplementedError``.
"""

from __future__ import annotations

import math

import torch

from .ops import gdn_chunk_fwd

__all__ = ["chunk_gated_delta_rule", "chunk_delta_rule"]


def _check_kwargs(kwargs):
    if kwargs.get("head_first", False):
        raise NotImplementedError("head_first layouts are not supported: inputs are [B, T, H, ...]")
    if kwargs.get("use_gate_in_kernel", False):
        raise NotImplementedError("use_gate_in_kernel (A_log / dt_bias gate) is not supported")
    unknown = set(kwargs) - {"head_first", "use_gate_in_kernel", "A_log", "dt_bias"}
    if unknown:
        raise TypeError(f"unexpected keyword arguments {sorted(unknown)}")


def _state_in(initial_state, transpose_state_layout):
    """FLA [N, H, K, V] (or [N, H, V, K] when transposed) -> gdn_ref's [N, H, V, K]."""
    if initial_state is None:
        return None
    return initial_state if transpose_state_layout else initial_state.transpose(-1, -2)


def _state_out(ht, transpose_state_layout):
    if ht is None or transpose_state_layout:
        return ht
    return ht.transpose(-1, -2).contiguous()


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False, cu_seqlens=None, cu_seqlens_cpu=None,
                           cp_context=None, transpose_state_layout=False, **kwargs):
    """Gated DeltaNet forward with FLA's signature; returns (o, final_state or None)."""
    _check_kwargs(kwargs)
    if cp_context is not None:
        raise NotImplementedError("context parallelism is not supported")
    if q.shape[2] != k.shape[2]:
        raise ValueError(f"q and k must have the same number of heads, got {q.shape[2]} and {k.shape[2]}")
    if v.shape[2] != q.shape[2]:
        raise NotImplementedError("grouped value heads (v with more heads than q) are not supported")
    K = q.shape[-1]
    scale = 1.0 / math.sqrt(K) if scale is None else float(scale)
    h0 = _state_in(initial_state, transpose_state_layout)
    common = dict(scale=scale, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)

    if cu_seqlens is None:
        o, ht = gdn_chunk_fwd(q, k, v, beta, g, initial_state=h0, output_final_state=output_final_state,
                              **common)
        return o, _state_out(ht, transpose_state_layout)

    if q.shape[0] != 1:
        raise ValueError(f"the batch size must be 1 with cu_seqlens, got {q.shape[0]}")
    bounds = (cu_seqlens_cpu if cu_seqlens_cpu is not None else cu_seqlens).tolist()
    N = len(bounds) - 1
    if h0 is not None and h0.shape[0] != N:
        raise ValueError(f"initial_state holds {h0.shape[0]} states for {N} sequences")
    H, V = q.shape[2], v.shape[-1]
    o = torch.zeros(q.shape[:3] + (V,), dtype=q.dtype, device=q.device)
    ht = torch.zeros(N, H, V, K, dtype=torch.float32, device=q.device) if output_final_state else None
    # sequences of one length run as one batch (one forward per distinct length);
    # a length that occurs once runs on views of the packed tensors, no copy
    by_len = {}
    for i in range(N):
        s, e = int(bounds[i]), int(bounds[i + 1])
        if e <= s:  # empty sequence: the state passes through
            if ht is not None and h0 is not None:
                ht[i] = h0[i]
            continue
        by_len.setdefault(e - s, []).append(i)
    for L, idx in by_len.items():
        starts = [int(bounds[i]) for i in idx]
        if len(idx) == 1:
            s = starts[0]
            pick = lambda x: None if x is None else x[:, s:s + L]
            h0_g = None if h0 is None else h0[idx[0]:idx[0] + 1]
        else:
            pick = lambda x: None if x is None else torch.cat([x[:, s:s + L] for s in starts], dim=0)
            h0_g = None if h0 is None else h0[idx]
        o_g, ht_g = gdn_chunk_fwd(pick(q), pick(k), pick(v), pick(beta), pick(g), initial_state=h0_g,
                                  output_final_state=output_final_state, **common)
        for j, s in enumerate(starts):
            o[0, s:s + L] = o_g[j]
        if ht is not None:
            ht[idx] = ht_g
    return o, _state_out(ht, transpose_state_layout)


def chunk_delta_rule(q, k, v, beta, scale=None, initial_state=None, output_final_state=False,
                     use_qk_l2norm_in_kernel=False, cu_seqlens=None, cu_seqlens_cpu=None, **kwargs):
    """DeltaNet forward (the gated rule with g == 0) with FLA's signature."""
    return chunk_gated_delta_rule(q, k, v, None, beta, scale=scale, initial_state=initial_state,
                                  output_final_state=output_final_state,
                                  use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, cu_seqlens=cu_seqlens,
                                  cu_seqlens_cpu=cu_seqlens_cpu, **kwargs)
