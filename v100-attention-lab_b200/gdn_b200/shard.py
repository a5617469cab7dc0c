"""Multi-GPU partitioning of the chunked GDN forward by (batch, head) pairs.

Every (b, h) pair is an independent recurrence (gdn_ref.py:39-44; the
reference's program map gdn_triton.py:42-45), so N GPUs split the B*H pairs
into N disjoint blocks and run with no collective on the hot path.  One
process per GPU (torchrun); an optional all-gather of the outputs over NCCL
is a separate, explicitly requested step.

Blocks are taken as whole batches when N divides B, else as whole head
ranges when N divides H, so a rank's inputs are strided views of the
caller's tensors (no copies); otherwise the pairs are split in contiguous
b-major order and the slices are copied.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["ShardPlan", "plan", "local_inputs", "run_local", "gather_outputs"]


@dataclass(frozen=True)
class ShardPlan:
    B: int
    H: int
    world: int
    rank: int
    mode: str          # "batch", "head" or "pairs"
    start: int         # first owned index (batch, head or flattened pair)
    stop: int          # one past the last

    @property
    def pairs(self) -> int:
        if self.mode == "batch":
            return (self.stop - self.start) * self.H
        if self.mode == "head":
            return self.B * (self.stop - self.start)
        return self.stop - self.start


def _split(n, world, rank):
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def plan(B: int, H: int, world: int, rank: int) -> ShardPlan:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad world/rank {world}/{rank}")
    if B % world == 0:
        s, e = _split(B, world, rank)
        return ShardPlan(B, H, world, rank, "batch", s, e)
    if H % world == 0:
        s, e = _split(H, world, rank)
        return ShardPlan(B, H, world, rank, "head", s, e)
    s, e = _split(B * H, world, rank)
    return ShardPlan(B, H, world, rank, "pairs", s, e)


def _take(x, p: ShardPlan, state=False):
    """Slice x ([B,T,H,*] / [B,T,H] / state [B,H,V,K]) to the rank's pairs."""
    if x is None:
        return None
    if p.mode == "batch":
        return x[p.start:p.stop]
    if p.mode == "head":
        return x[:, p.start:p.stop] if state else x[:, :, p.start:p.stop]
    # flattened pairs: [B,T,H,...] -> [1, T, P, ...] (copy)
    if state:
        flat = x.reshape(p.B * p.H, *x.shape[2:])
        return flat[p.start:p.stop].unsqueeze(0).contiguous()
    xt = x.transpose(1, 2).reshape(p.B * p.H, x.shape[1], *x.shape[3:])
    return xt[p.start:p.stop].transpose(0, 1).unsqueeze(0).contiguous()


def local_inputs(p: ShardPlan, q, k, v, beta, g, initial_state=None):
    """The rank's views (or copies, in "pairs" mode) of the global inputs."""
    return (_take(q, p), _take(k, p), _take(v, p), _take(beta, p), _take(g, p),
            _take(initial_state, p, state=True))


def run_local(p: ShardPlan, q, k, v, beta, g, initial_state=None, fwd=None, **kw):
    """Run this rank's shard.  ``fwd`` defaults to gdn_b200.gdn_chunk_fwd."""
    if fwd is None:
        from .ops import gdn_chunk_fwd as fwd
    lq, lk, lv, lb, lg, lh = local_inputs(p, q, k, v, beta, g, initial_state)
    return fwd(lq, lk, lv, lb, lg, initial_state=lh, **kw)


def gather_outputs(p: ShardPlan, o_local, h_local, group=None):
    """All-gather the shards into full [B,T,H,V] / [B,H,V,K] tensors on every rank.

    Off the hot path: one collective per tensor over the process group.
    """
    import torch.distributed as dist
    world = p.world
    if p.mode == "pairs":
        raise NotImplementedError("gather for uneven pair splits")
    sizes = [plan(p.B, p.H, world, r) for r in range(world)]
    outs, hs = [], []
    for sp in sizes:
        n = sp.stop - sp.start
        if p.mode == "batch":
            outs.append(torch.empty((n,) + tuple(o_local.shape[1:]), dtype=o_local.dtype, device=o_local.device))
            hs.append(torch.empty((n,) + tuple(h_local.shape[1:]), dtype=h_local.dtype, device=h_local.device))
        else:
            so = list(o_local.shape); so[2] = n
            sh = list(h_local.shape); sh[1] = n
            outs.append(torch.empty(so, dtype=o_local.dtype, device=o_local.device))
            hs.append(torch.empty(sh, dtype=h_local.dtype, device=h_local.device))
    dist.all_gather(outs, o_local.contiguous(), group=group)
    dist.all_gather(hs, h_local.contiguous(), group=group)
    if p.mode == "batch":
        return torch.cat(outs, 0), torch.cat(hs, 0)
    return torch.cat(outs, 2), torch.cat(hs, 1)
