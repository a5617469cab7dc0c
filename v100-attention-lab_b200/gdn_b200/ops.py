"""Python entry points of the B200 chunked Gated DeltaNet forward.

``gdn_chunk_fwd`` is the drop-in for the reference's
``gdn_triton.gdn_chunk_fwd(q, k, v, beta, g)`` (gdn_triton.py:113-140):
same positional order (q, k, v, beta, g), same shapes, same outputs
(o in q's dtype, the final state in fp32 with K contiguous).  It also takes
the initial state and chunk size that ``gdn_ref.gdn_chunk_ref`` accepts
(gdn_ref.py:48) and that the reference kernels ignore (gdn_triton.py:52).

Everything runs in the sm_100a library through its C ABI; if the library is
missing, or the device is not a B200, the call raises instead of falling back.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

__all__ = ["gdn_chunk_fwd", "gdn_chunk_fwd_v2", "gdn_wy_prep", "GdnError", "check_status"]


class GdnError(RuntimeError):
    """Error reported by the native library."""

    def __init__(self, code: int, where: str):
        self.code = int(code)
        super().__init__(f"{where}: {_lib.status_string(code)} (status {code})")


_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}
_status_words: dict[int, torch.Tensor] = {}
# scratch of the two-kernel path, one per (device index, stream handle)
_workspaces: dict[tuple[int, int], torch.Tensor] = {}

# Upper bound of the scratch of the two-kernel path per (device, stream);
# longer inputs run in several segments of chunks, so memory does not grow
# with T.
WORKSPACE_CAP_BYTES = int(os.environ.get("GDN_B200_WORKSPACE_MB", "4096")) << 20


def _workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
    """Cached uint8 scratch for launches on ``stream``; grows (never shrinks).

    The packets of one forward live in this buffer from its prep kernel to its
    scan kernel, so two forwards that may run at the same time must not share
    it: each stream gets its own, and launches on one stream are ordered.  The
    buffer is allocated while ``stream`` is current, so the caching allocator
    ties it to that stream; a buffer that is replaced because it is too small
    is freed in stream order behind the launches already queued on it.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, int(stream.cuda_stream))
    w = _workspaces.get(key)
    if w is None or w.numel() < nbytes:
        with torch.cuda.stream(stream):
            w = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[key] = w
    return w


def release_workspaces() -> None:
    """Drop the cached scratch buffers (all devices and streams).

    Forwards already queued keep their buffers alive until they complete (the
    caching allocator frees each in its stream's order)."""
    _workspaces.clear()


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def check_status(device=None) -> None:
    """Synchronise ``device`` and raise if any kernel launched there aborted.

    Kernels never hang: a device-side wait that expires aborts the CTA and
    records GDN_ERR_TIMEOUT in a per-device status word, read here.
    """
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = _status_word(dev)
    val = int(w.item())
    if val:
        w.zero_()
        code = max(c for c in range(1, 8) if val & (1 << c))
        raise GdnError(code, "gdn_b200 kernel")


def _check_inputs(q, k, v, beta, g):
    tensors = {"q": q, "k": k, "v": v, "beta": beta}
    if g is not None:
        tensors["g"] = g
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [B, T, H, K] / [B, T, H, V]")
    B, T, H, K = q.shape
    if tuple(k.shape) != (B, T, H, K):
        raise ValueError(f"k shape {tuple(k.shape)} != q shape {tuple(q.shape)}")
    if tuple(v.shape[:3]) != (B, T, H):
        raise ValueError(f"v shape {tuple(v.shape)} does not match q's [B, T, H]")
    if tuple(beta.shape) != (B, T, H) or (g is not None and tuple(g.shape) != (B, T, H)):
        raise ValueError(f"beta and g must be [B, T, H] = {(B, T, H)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"q, k, v must share a dtype (got {q.dtype}, {k.dtype}, {v.dtype})")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError(f"gdn_b200 takes fp16 or bf16 q/k/v (got {q.dtype})")
    for name in ("q", "k", "v"):
        if tensors[name].stride(-1) != 1:
            raise ValueError(f"{name} must have a contiguous last dimension")
    dev = q.device
    for name, t in tensors.items():
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (got device {t.device})")
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, q is on {dev}")
    return B, T, H, K, v.shape[-1]


def _fill_args(q, k, v, beta, g, h0, o, ht, chunk_size, block_v, status, scale=1.0, flags=0) -> _lib.GdnFwdArgs:
    B, T, H, K = q.shape
    a = _lib.GdnFwdArgs()
    a.abi_version = _lib.ABI_VERSION
    a.B, a.T, a.H, a.K, a.V = B, T, H, K, v.shape[-1]
    a.chunk_size = int(chunk_size)
    a.in_dtype = _DTYPES[q.dtype]
    a.out_dtype = _DTYPES[o.dtype] if o is not None else _lib.DTYPE_F32
    a.block_v = int(block_v)
    for name, t in (("q", q), ("k", k), ("v", v), ("beta", beta), ("g", g)):
        if t is None:  # g: no gate (g == 0)
            continue
        setattr(a, name, t.data_ptr())
        st = getattr(a, name + "_stride")
        st[0], st[1], st[2] = t.stride(0), t.stride(1), t.stride(2)
    a.h0 = h0.data_ptr() if h0 is not None else None
    if o is not None:
        a.o = o.data_ptr()
        a.o_stride[0], a.o_stride[1], a.o_stride[2] = o.stride(0), o.stride(1), o.stride(2)
    a.ht = ht.data_ptr() if ht is not None else None
    a.status = status.data_ptr() if status is not None else None
    a.scale = float(scale)
    a.flags = int(flags)
    return a


def _prep_flags(use_qk_l2norm_in_kernel, beta_activation, g_activation, solver="blocked", ns_iters=3):
    flags = 0
    if solver == "newton_schulz":
        if not 1 <= int(ns_iters) <= 15:
            raise ValueError(f"ns_iters must be in 1..15 (got {ns_iters})")
        flags |= _lib.FLAG_SOLVER_NS | (int(ns_iters) << _lib.NS_ITERS_SHIFT)
    elif solver != "blocked":
        raise ValueError(f"solver must be 'blocked' or 'newton_schulz' (got {solver!r})")
    if use_qk_l2norm_in_kernel:
        flags |= _lib.FLAG_QK_L2NORM
    if beta_activation is not None:
        if beta_activation != "sigmoid":
            raise ValueError(f"beta_activation must be None or 'sigmoid' (got {beta_activation!r})")
        flags |= _lib.FLAG_BETA_SIGMOID
    if g_activation is not None:
        if g_activation != "logsigmoid":
            raise ValueError(f"g_activation must be None or 'logsigmoid' (got {g_activation!r})")
        flags |= _lib.FLAG_G_LOGSIGMOID
    return flags


def gdn_chunk_fwd(q, k, v, beta, g, initial_state=None, chunk_size=64, *, output_dtype=None,
                  output_final_state=True, block_v=0, check=False, fused=False, scale=None,
                  use_qk_l2norm_in_kernel=False, beta_activation=None, g_activation=None, solver="blocked",
                  ns_iters=3):
    """Chunked Gated DeltaNet forward on a B200.

    Args:
        q, k: [B, T, H, K] fp16/bf16 (last dim contiguous)
        v:    [B, T, H, V] same dtype
        beta: [B, T, H] (cast to fp32 if needed)
        g:    [B, T, H] log decay (<= 0), cast to fp32 if needed; None means
              g == 0 (no decay: the DeltaNet recurrence)
        initial_state: optional [B, H, V, K] state h0 (fp32 is used)
        chunk_size: C, 32 or 64 (the reference's two values).  C only sets
            how the sequence is tiled: the forward is the step recurrence
            for any C (gdn_ref.py:117-132 checks exactly that), so this build
            computes with its 64-token chunks either way.
        output_dtype: dtype of o (default q.dtype, as gdn_triton.py:126)
        output_final_state: return the final state (else None)
        block_v: V columns per CTA (0 = choose)
        check: synchronise and raise if the kernel reported an error
        fused: run the single fused kernel instead of the two-kernel path
            (chunk-parallel WY/UT preparation + state scan); both meet the
            same tolerance, the fused one needs no scratch memory
        scale: q is scaled by this factor (the FLA convention); None = 1,
            the reference's behaviour
        use_qk_l2norm_in_kernel: q and k are raw; their rows are
            L2-normalised inside the kernel (gdn_ref.py:24-25), fp32 math
        beta_activation: 'sigmoid' if beta holds logits
        g_activation: 'logsigmoid' if g holds logits
        solver: 'blocked' (exact fp32 inverse of I + A, the default) or
            'newton_schulz' (the approximate fp16 iteration of
            gdn_triton_v2.py:58-68, ``ns_iters`` steps; two-kernel path only)
    Returns:
        (o [B, T, H, V], h_final [B, H, V, K] fp32 or None)

    T need not be a multiple of chunk_size: the tail is padded on the device
    with the rule of gdn_ref.py:102-114, without the host-side copies of
    gdn_triton.py:122-125.

    Launches on the current stream of q's device (as the reference's Triton
    launch does) and returns without synchronising.  The scratch of the
    two-kernel path is cached per (device, stream), so forwards issued on
    different streams may run at the same time.
    """
    B, T, H, K, V = _check_inputs(q, k, v, beta, g)
    if chunk_size not in (32, 64):
        raise NotImplementedError(f"chunk_size must be 32 or 64 (got {chunk_size})")
    chunk_size = 64
    flags = _prep_flags(use_qk_l2norm_in_kernel, beta_activation, g_activation, solver, ns_iters)
    if g is None and g_activation is not None:
        raise ValueError("g_activation needs a g tensor")
    scale = 1.0 if scale is None else float(scale)
    lib = _lib.load()
    dev = q.device
    beta = beta if beta.dtype == torch.float32 else beta.float()
    g = g if (g is None or g.dtype == torch.float32) else g.float()
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (B, H, V, K):
            raise ValueError(f"initial_state must be [B, H, V, K] = {(B, H, V, K)}")
        if initial_state.device != dev:
            raise ValueError("initial_state must be on q's device")
        h0 = initial_state.to(torch.float32).contiguous()
    out_dtype = q.dtype if output_dtype is None else output_dtype
    if out_dtype not in _DTYPES:
        raise ValueError(f"unsupported output_dtype {out_dtype}")
    o = torch.empty(B, T, H, V, dtype=out_dtype, device=dev)
    ht = torch.empty(B, H, V, K, dtype=torch.float32, device=dev) if output_final_state else None
    status = _status_word(dev)
    args = _fill_args(q, k, v, beta, g, h0, o, ht, chunk_size, block_v, status, scale, flags)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        if not fused:
            need = int(lib.gdn_fwd_workspace_bytes(ctypes.byref(args)))
            per_head = _lib.WORKSPACE_HEADER_BYTES + B * H * (_lib.PACKET_BYTES_PER_CHUNK + V * K * 4)
            nbytes = max(min(need, WORKSPACE_CAP_BYTES), per_head)
            ws = _workspace(dev, stream, nbytes)
            args.workspace = ws.data_ptr()
            args.workspace_bytes = ws.numel()
        rc = lib.gdn_fwd_sm100(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
    if rc != _lib.OK:
        _raise(rc, "gdn_fwd_sm100")
    if check:
        with torch.cuda.device(dev):
            check_status(dev)
    return o, ht


def gdn_chunk_fwd_v2(q, k, v, beta, g, C=32, BV=32, num_warps=4, num_stages=1, iters=3, solver="blocked", **kw):
    """Keyword-compatible stand-in for ``gdn_chunk_fwd_v2`` (gdn_triton_v2.py:92),
    with the reference's defaults.

    C maps to ``chunk_size`` (32 or 64; computed with 64-token chunks) and BV
    to ``block_v``; num_warps and num_stages tune the reference's Triton
    kernel and have no counterpart.  The default
    solver inverts (I + A) exactly; ``solver="newton_schulz"`` runs the
    reference's iteration with ``iters`` steps instead (approximate).
    """
    del num_warps, num_stages
    return gdn_chunk_fwd(q, k, v, beta, g, chunk_size=C, block_v=BV, solver=solver, ns_iters=iters, **kw)


def gdn_chunk_fwd_fixed(q, k, v, beta, g, C=32, BV=32, num_warps=4, num_stages=1, **kw):
    """Stand-in for ``gdn_chunk_fwd_fixed`` (bench_gdn.py:43-59): the forward
    launched with a fixed configuration instead of the reference's autotuner.

    Same arguments and outputs ``(o, hf)``; C and BV as in
    ``gdn_chunk_fwd_v2``, num_warps / num_stages have no counterpart.  The
    reference's fixed launch needs T to be a multiple of C; here any T works.
    """
    del num_warps, num_stages
    return gdn_chunk_fwd(q, k, v, beta, g, chunk_size=C, block_v=BV, **kw)


def gdn_wy_prep(q, k, v, beta, g, chunk_size=64, check=True):
    """The chunk-parallel WY/UT stage alone (gdn_ref.py:76-85).

    Returns (W [B, H, NT, C, K], U [B, H, NT, C, V]) in fp32 for every chunk,
    computed by the same device code as the fused forward.
    """
    B, T, H, K, V = _check_inputs(q, k, v, beta, g)
    lib = _lib.load()
    dev = q.device
    beta = beta if beta.dtype == torch.float32 else beta.float()
    g = g if g.dtype == torch.float32 else g.float()
    NT = -(-T // chunk_size)
    W = torch.empty(B, H, NT, chunk_size, K, dtype=torch.float32, device=dev)
    U = torch.empty(B, H, NT, chunk_size, V, dtype=torch.float32, device=dev)
    status = _status_word(dev)
    args = _fill_args(q, k, v, beta, g, None, None, None, chunk_size, 0, status)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.gdn_wy_prep_sm100(ctypes.byref(args), ctypes.c_void_p(W.data_ptr()),
                                   ctypes.c_void_p(U.data_ptr()), ctypes.c_void_p(stream))
    if rc != _lib.OK:
        _raise(rc, "gdn_wy_prep_sm100")
    if check:
        with torch.cuda.device(dev):
            check_status(dev)
    return W, U


def _raise(rc: int, where: str):
    if rc in (_lib.ERR_INVALID_ARGUMENT, _lib.ERR_ALIGNMENT):
        raise ValueError(f"{where}: {_lib.status_string(rc)}")
    if rc == _lib.ERR_UNSUPPORTED:
        raise NotImplementedError(f"{where}: {_lib.status_string(rc)}")
    raise GdnError(rc, where)
