"""Solver sweep: the exact blocked inverse vs the Newton-Schulz iteration.

The reference picks its (I + A)^-1 solver and tile shape by sweeping
C / BV / warps / iters on its GPUs (bench_gdn.py:117-137, gdn_triton_v2.py:92;
README.md:199-213: Newton-Schulz was 4.2x faster than forward substitution on
SM89).  This harness makes the same comparison for the sm_100a kernels:

    python -m gdn_b200.sweep [--config 2] [--reps 50] [--iters 1 2 3 4 5 6]

For every solver it prints one JSON line: device time per forward (CUDA events
around --reps back-to-back forwards, median of 5 such runs after warm-up,
inputs rotating over sets larger than L2),
Mtokens/s, and the error max|o - o_ref| / max|o_ref| and the same for the final
state against the float64 step recurrence on a smaller case (B=1, T=1024, H=2)
with the same input distributions: once with independent random keys and once
with correlated keys (each key plus twice a shared per-head direction before
normalisation), where the entries of (I + A) reach 0.5 and the iteration count
shows.  This build fixes C = 64 and BV = 32 (the
tile shapes its tensor-core layouts are written for), so the sweep is over the
solver and its iteration count.
"""

from __future__ import annotations

import argparse
import json
import statistics

import numpy as np
import torch

from .ops import gdn_chunk_fwd

CONFIGS = {
    1: dict(B=2, T=2048, H=8, dtype=torch.float16, h0=False),
    2: dict(B=2, T=4096, H=16, dtype=torch.bfloat16, h0=True),
    4: dict(B=8, T=8192, H=32, dtype=torch.bfloat16, h0=True),
}


def _inputs(B, T, H, dtype, h0, seed, device, key_corr=0.0):
    g = torch.Generator().manual_seed(seed)
    l2 = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    q = l2(torch.randn(B, T, H, 128, generator=g)).to(dtype)
    k = torch.randn(B, T, H, 128, generator=g)
    if key_corr:
        k = k + key_corr * torch.randn(1, 1, H, 128, generator=g)
    k = l2(k).to(dtype)
    v = torch.randn(B, T, H, 128, generator=g).to(dtype)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    gate = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=g))
    s = 0.1 * torch.randn(B, H, 128, 128, generator=g) if h0 else None
    to = lambda x: None if x is None else x.to(device)
    return tuple(to(x) for x in (q, k, v, beta, gate, s))


def _recurrence(q, k, v, beta, g, h0):
    """float64 step recurrence h_t = e^{g_t} h + beta_t (v_t - e^{g_t} h k_t) k_t^T, o_t = h_t q_t."""
    f = lambda x: x.double().cpu()
    q, k, v, beta, g = map(f, (q, k, v, beta, g))
    B, T, H, K = q.shape
    h = torch.zeros(B, H, v.shape[-1], K, dtype=torch.float64) if h0 is None else f(h0)
    o = torch.empty(B, T, H, v.shape[-1], dtype=torch.float64)
    for t in range(T):
        h = torch.exp(g[:, t])[..., None, None] * h
        u = beta[:, t, :, None] * (v[:, t] - torch.einsum("bhvk,bhk->bhv", h, k[:, t]))
        h = h + u[..., None] * k[:, t][:, :, None, :]
        o[:, t] = torch.einsum("bhvk,bhk->bhv", h, q[:, t])
    return o, h


def _rel(x, ref):
    x = x.double().cpu()
    return float((x - ref).abs().max() / ref.abs().max())


def run(config=2, reps=50, iters=(1, 2, 3, 4, 5, 6), device="cuda"):
    dev = torch.device(device)
    cfg = CONFIGS[config]
    B, T, H = cfg["B"], cfg["T"], cfg["H"]
    nsets = max(2, -(-2 * 126 * 2 ** 20 // (B * T * H * 3 * 128 * 2)))
    sets = [_inputs(B, T, H, cfg["dtype"], cfg["h0"], s, dev) for s in range(nsets)]
    checks = []
    for corr in (0.0, 2.0):
        small = _inputs(1, 1024, 2, cfg["dtype"], True, 99, dev, key_corr=corr)
        checks.append((small, _recurrence(*small)))
    solvers = [("blocked", None)] + [("newton_schulz", n) for n in iters]
    out = []
    for solver, n in solvers:
        kw = dict(solver=solver, ns_iters=n if n else 3)
        errs = []
        for small, (o_ref, h_ref) in checks:
            o, h = gdn_chunk_fwd(*small[:5], initial_state=small[5], output_dtype=torch.float32, check=True, **kw)
            errs += [_rel(o, o_ref), _rel(h, h_ref)]
        for i in range(3):
            gdn_chunk_fwd(*sets[i % nsets][:5], initial_state=sets[i % nsets][5], **kw)
        times = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                s = sets[i % nsets]
                gdn_chunk_fwd(*s[:5], initial_state=s[5], **kw)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / reps)
        ms = statistics.median(times)
        line = {"solver": solver, "iters": n, "config": config, "C": 64, "BV": 32, "ms_per_forward": ms,
                "mtokens_per_s": B * T / (ms / 1e3) / 1e6, "err_o": errs[0], "err_h": errs[1],
                "err_o_corr_keys": errs[2], "err_h_corr_keys": errs[3]}
        print(json.dumps(line), flush=True)
        out.append(line)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--iters", type=int, nargs="+", default=[1, 2, 3, 4, 5, 6])
    args = ap.parse_args()
    np.set_printoptions(precision=3)
    run(args.config, args.reps, tuple(args.iters))


if __name__ == "__main__":
    main()
