"""Shared helpers of the GPU parity tests (inputs, oracle runs, tolerances)."""

import numpy as np
import torch

from oracle import gdn_oracle as ora

# Error bar of the north star: max|x - ref| / max|ref| < 1e-3 against the fp32
# step recurrence, for fp16/bf16 inputs with fp32 accumulation.
TOL = 1e-3
# Storing o in a 16-bit format adds its own rounding on top of the kernel's
# error: at most half an ulp, i.e. 2^-9 (bf16) or 2^-12 (fp16) of |o|, which
# relative to max|o| can reach those values.  Tests of 16-bit outputs allow
# TOL plus that storage bound; fp32 outputs must meet TOL itself.
STORE_ROUNDING = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


def make(B, T, H, K=128, V=128, seed=0, dtype=torch.bfloat16, h0_std=None, gate_mean=0.0, dev="cuda", key_corr=0.0):
    q, k, v, beta, g, h0 = ora.make_inputs(B, T, H, K, V, seed=seed, gate_mean=gate_mean, h0_std=h0_std,
                                           key_corr=key_corr)
    t = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).to(dev).to(dt)
    qd, kd, vd = t(q, dtype), t(k, dtype), t(v, dtype)
    h0d = t(h0) if h0 is not None else None
    return qd, kd, vd, t(beta), t(g), h0d


def oracle(qd, kd, vd, bd, gd, h0d, chunked=False, C=64, ns_iters=None):
    """fp64 oracle on exactly the (16-bit-rounded) device inputs (chunked with
    the Newton-Schulz solve when ns_iters is given)."""
    f = lambda x: None if x is None else x.float().cpu().numpy()
    if chunked or ns_iters is not None:
        q, k, v, b, g = ora.pad_to_multiple(f(qd), f(kd), f(vd), f(bd), f(gd), C)
        o, h = ora.chunked(q, k, v, b, g, C=C, initial_state=f(h0d), ns_iters=ns_iters)
        return o[:, : qd.shape[1]], h
    return ora.recurrent(f(qd), f(kd), f(vd), f(bd), f(gd), initial_state=f(h0d))


def rel(x, ref):
    return ora.max_rel(x.float().cpu().numpy() if isinstance(x, torch.Tensor) else x, ref)


def ulp_distance_16(a, b):
    """Largest distance, in units in the last place, between two 16-bit float
    tensors of the same dtype (sign-magnitude bit patterns mapped to ordered
    integers, so -0 and +0 are 0 apart)."""
    assert a.dtype == b.dtype and a.dtype in (torch.float16, torch.bfloat16)

    def ordered(x):
        i = x.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)  # negative: flip magnitude order

    return int((ordered(a) - ordered(b)).abs().max().item())
