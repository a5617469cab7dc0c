"""Phase timing of the two kernels from in-kernel clock64 stamps.

    python -m gdn_b200.trace [--config 2] [--base 1024]

Builds a copy of the library with ``-DGDN_TRACE`` (``libgdn_b200_trace.so``
next to the product library; the product build carries no trace code), runs
a few forwards of a bench config, and prints

* the prep kernel's phases for 64 CTAs starting at CTA ``--base`` (a
  mid-kernel wave by default, so the L2 prefetch of the inputs is in steady
  state), median SM cycles per phase;
* the scan kernel's per-chunk hand-offs for its first CTA (one (b, h, V
  slice)), median over the middle chunks.

The stamps are clock64 of one thread per role, written to a device buffer the
host hands over through ``gdn_set_trace_buffer[_wy]``.  A traced build is
slightly slower; its timings explain, they are not bench numbers.
"""

from __future__ import annotations

import argparse
import ctypes
import os
import subprocess
import sys

from . import _build

TRACE_LIB = os.path.join(_build.PKG_DIR, "libgdn_b200_trace.so")

PREP_PHASES = [  # (slot, name): the order the phases complete in
    (0, "start"), (1, "k/q landed"), (2, "S = [K;Q]K^T"), (3, "A, P"), (4, "inverse"), (5, "T split"),
    (6, "[W|U] product"), (7, "epilogue A"), (10, "PW, PU"), (11, "epilogue C"), (8, "N, c"),
    (9, "epilogue B"), (12, "exit"),
]


def build_trace_lib(base: int) -> str:
    stamp = TRACE_LIB + ".base"
    if (not _build.is_stale(TRACE_LIB) and os.path.exists(stamp)
            and open(stamp).read().strip() == str(base)):
        return TRACE_LIB
    cmd = [_build.nvcc_path(), *_build.NVCC_FLAGS, "-DGDN_TRACE", f"-DGDN_TRACE_BASE={base}",
           "-I", _build.INCLUDE_DIR, "-o", TRACE_LIB,
           *[os.path.join(_build.SRC_DIR, s) for s in _build.SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    with open(stamp, "w") as f:
        f.write(str(base))
    return TRACE_LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--base", type=int, default=1024, help="first traced prep CTA")
    args = ap.parse_args()
    build_trace_lib(args.base)
    os.environ["GDN_B200_LIB"] = TRACE_LIB  # before the first load of the library
    import numpy as np
    import torch

    from . import _lib, ops
    sys.path.insert(0, os.path.dirname(_build.PKG_DIR))
    sys.path.insert(0, os.path.dirname(os.path.dirname(_build.PKG_DIR)))
    import bench  # the repository's bench: same configs and input distributions

    lib = _lib.load()
    lib.gdn_set_trace_buffer.argtypes = [ctypes.c_void_p]
    lib.gdn_set_trace_buffer_wy.argtypes = [ctypes.c_void_p]
    cfg = bench.CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    q, k, v, beta, g, h0 = bench.make_inputs(cfg, cfg["B"], 0, dev)
    nt = -(-cfg["T"] // 64)
    tr_wy = torch.zeros(64, 24, dtype=torch.int64, device=dev)
    tr_sc = torch.zeros(nt, 24, dtype=torch.int64, device=dev)
    lib.gdn_set_trace_buffer_wy(ctypes.c_void_p(tr_wy.data_ptr()))
    lib.gdn_set_trace_buffer(ctypes.c_void_p(tr_sc.data_ptr()))
    for _ in range(5):
        ops.gdn_chunk_fwd(q, k, v, beta, g, initial_state=h0, check=True)
    torch.cuda.synchronize()
    lib.gdn_set_trace_buffer_wy(ctypes.c_void_p(0))
    lib.gdn_set_trace_buffer(ctypes.c_void_p(0))

    t = tr_wy.cpu().numpy().astype(np.int64)
    t = t[t[:, 0] > 0]
    slots = [s for s, _ in PREP_PHASES]
    d = t[:, slots] - t[:, [0]]
    steps = np.median(np.diff(d, axis=1), axis=0)
    print(f"prep kernel, config {args.config}, CTAs {args.base}..{args.base + len(t) - 1}: "
          f"median SM cycles per phase")
    for (_, name), c in zip(PREP_PHASES[1:], steps):
        print(f"  {name:16s} {c:8.0f}")
    print(f"  {'total':16s} {np.median(d[:, -1]):8.0f}")

    s = tr_sc.cpu().numpy().astype(np.int64)[4:-4]
    s_next = tr_sc.cpu().numpy().astype(np.int64)[5:-3]
    print(f"scan kernel, config {args.config}, CTA 0: median SM cycles per chunk")
    print(f"  period (N S complete to N S complete)      {np.median(np.diff(s[:, 2])):8.0f}")
    print(f"  S' ready seen by the issuer -> N S issued   {np.median(s[:, 6] - s[:, 1]):8.0f}")
    print(f"  N S issued -> seen complete by chain warp 0 {np.median(s[:, 2] - s[:, 6]):8.0f}")
    print(f"  state epilogue (-> S' of the next chunk)     {np.median(s[:, 3] - s[:, 2]):8.0f}")
    print(f"  S' written -> seen by the issuer             {np.median(s_next[:, 1] - s[:, 3]):8.0f}")
    print(f"  output products issued after N S             {np.median(s[:, 7] - s[:, 6]):8.0f}")


if __name__ == "__main__":
    main()
