"""Generate the golden fixtures in this folder by running the reference itself.

The reference's oracle (``gdn_ref.py`` of 123123213weqw/v100-attention-lab) is
pure PyTorch, so it is imported from a checkout of the reference and run on
CPU.  The resulting inputs/outputs are stored as small compressed ``.npz``
files; the tests read only those files, never the reference.

Usage:  python tests/golden/make_golden.py <path-to-reference-checkout>

Fixtures
--------
selfcheck.npz   the reference's own CPU self-check case (gdn_ref.py:117-132):
                torch seed 0, B2 T128 H3 K=V=64, beta~U(0.4,0.9), g~-U(0,0.1);
                outputs of gdn_recurrent_ref and gdn_chunk_ref(C=32).
cfg0.npz        config 0, the reference's CPU-runnable case: B1 T256 H2 K=V=64
                fp32, h0 = 0, C=32, with the benchmark distributions
                (l2norm q/k, sigmoid beta, logsigmoid g).
h0_f16.npz      B1 T128 H2 K=V=128, fp16 q/k/v, random h0 (std 0.1); recurrent
                (fp64) and chunked (C=64) outputs.
bf16_ragged.npz B1 T100 H2 K=V=128, bf16 q/k/v, h0 = 0, T padded to 128 with
                pad_to_multiple (gdn_ref.py:102-114); recurrent outputs of the
                unpadded and chunked outputs of the padded sequence.
stages.npz      per-chunk U and W captured from inside gdn_chunk_ref (its two
                solve_triangular calls, gdn_ref.py:84-85) on B1 T128 H2 K=V=128
                fp16, C=64.
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(x):
    return x.detach().to(torch.float32).cpu().numpy()


def _np64(x):
    return x.detach().to(torch.float64).cpu().numpy()


def main(ref_dir):
    sys.path.insert(0, ref_dir)
    import gdn_ref  # noqa: E402  (the reference's own module)

    torch.set_num_threads(8)
    out = {}

    # 1. the reference's own self-check inputs (gdn_ref.py:119-125)
    torch.manual_seed(0)
    B, T, H, K, V, C = 2, 128, 3, 64, 64, 32
    q = gdn_ref._l2norm(torch.randn(B, T, H, K))
    k = gdn_ref._l2norm(torch.randn(B, T, H, K))
    v = torch.randn(B, T, H, V)
    beta = torch.rand(B, T, H) * 0.5 + 0.4
    g = -torch.rand(B, T, H) * 0.1
    o1, h1 = gdn_ref.gdn_recurrent_ref(q, k, v, beta, g)
    o2, h2 = gdn_ref.gdn_chunk_ref(q, k, v, beta, g, C=C)
    out["selfcheck"] = dict(q=_np(q), k=_np(k), v=_np(v), beta=_np(beta), g=_np(g),
                            o_rec=_np(o1), h_rec=_np(h1), o_chunk=_np(o2), h_chunk=_np(h2),
                            C=np.int32(C))

    # inputs with the benchmark distributions, made with a seeded torch generator
    def make(B, T, H, K, V, seed, dt, h0_std=None):
        gen = torch.Generator().manual_seed(seed)
        q = gdn_ref._l2norm(torch.randn(B, T, H, K, generator=gen)).to(dt)
        k = gdn_ref._l2norm(torch.randn(B, T, H, K, generator=gen)).to(dt)
        v = torch.randn(B, T, H, V, generator=gen).to(dt)
        beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
        g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen))
        h0 = None if h0_std is None else torch.randn(B, H, V, K, generator=gen) * h0_std
        return q, k, v, beta, g, h0

    # 2. config 0
    q, k, v, beta, g, _ = make(1, 256, 2, 64, 64, seed=100, dt=torch.float32)
    o1, h1 = gdn_ref.gdn_recurrent_ref(q, k, v, beta, g)
    o2, h2 = gdn_ref.gdn_chunk_ref(q, k, v, beta, g, C=32)
    out["cfg0"] = dict(q=_np(q), k=_np(k), v=_np(v), beta=_np(beta), g=_np(g),
                       o_rec=_np(o1), h_rec=_np(h1), o_chunk=_np(o2), h_chunk=_np(h2),
                       C=np.int32(32))

    # 3. fp16 inputs with a random initial state
    q, k, v, beta, g, h0 = make(1, 128, 2, 128, 128, seed=101, dt=torch.float16, h0_std=0.1)
    o1, h1 = gdn_ref.gdn_recurrent_ref(q, k, v, beta, g, initial_state=h0, dtype=torch.float64)
    o2, h2 = gdn_ref.gdn_chunk_ref(q, k, v, beta, g, C=64, initial_state=h0)
    out["h0_f16"] = dict(q=_np(q), k=_np(k), v=_np(v), beta=_np(beta), g=_np(g), h0=_np(h0),
                         o_rec=_np64(o1), h_rec=_np64(h1), o_chunk=_np(o2), h_chunk=_np(h2),
                         C=np.int32(64), in_dtype=np.array("float16"))

    # 4. bf16 inputs, ragged T, padded with the reference's own helper
    q, k, v, beta, g, _ = make(1, 100, 2, 128, 128, seed=102, dt=torch.bfloat16)
    o1, h1 = gdn_ref.gdn_recurrent_ref(q, k, v, beta, g, dtype=torch.float64)
    qp, kp, vp, bp, gp = gdn_ref.pad_to_multiple(q, k, v, beta, g, 64)
    o2, h2 = gdn_ref.gdn_chunk_ref(qp, kp, vp, bp, gp, C=64)
    out["bf16_ragged"] = dict(q=_np(q), k=_np(k), v=_np(v), beta=_np(beta), g=_np(g),
                              o_rec=_np64(o1), h_rec=_np64(h1),
                              o_chunk_padded=_np(o2), h_chunk=_np(h2),
                              C=np.int32(64), in_dtype=np.array("bfloat16"))

    # 5. U and W captured from the reference's solve_triangular calls
    q, k, v, beta, g, _ = make(1, 128, 2, 128, 128, seed=103, dt=torch.float16)
    captured = []
    orig = torch.linalg.solve_triangular

    def spy(*a, **kw):
        r = orig(*a, **kw)
        captured.append(r.detach().clone())
        return r

    torch.linalg.solve_triangular = spy
    try:
        o2, h2 = gdn_ref.gdn_chunk_ref(q, k, v, beta, g, C=64)
    finally:
        torch.linalg.solve_triangular = orig
    # calls alternate U, W per chunk (gdn_ref.py:84-85); each is [B,H,C,*]
    U = torch.stack(captured[0::2], 0)     # [NT,B,H,C,V]
    W = torch.stack(captured[1::2], 0)     # [NT,B,H,C,K]
    out["stages"] = dict(q=_np(q), k=_np(k), v=_np(v), beta=_np(beta), g=_np(g),
                         U=_np(U), W=_np(W), o_chunk=_np(o2), h_chunk=_np(h2),
                         C=np.int32(64), in_dtype=np.array("float16"))

    for name, d in out.items():
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **d)
        print(f"wrote {path} ({os.path.getsize(path) / 1e3:.0f} kB)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GDN_REFERENCE_DIR", ""))
