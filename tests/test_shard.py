"""(batch, head) sharding across ranks, checked with gloo on CPU.

Each of two ranks runs its own block of (b, h) pairs -- here through the CPU
oracle standing in for the GPU kernel, which is what the N-GPU bench and
runner do with gdn_b200.gdn_chunk_fwd -- then the shards are all-gathered
and compared with the oracle on the whole batch.  No collective is needed on
the compute path itself.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn_b200 import shard


def test_plan_covers_every_pair_once():
    for B, H in [(8, 32), (2, 16), (3, 5), (1, 7), (4, 6)]:
        for world in (1, 2, 3, 4, 8):
            seen = np.zeros((B, H), dtype=int)
            for r in range(world):
                p = shard.plan(B, H, world, r)
                if p.mode == "batch":
                    seen[p.start:p.stop] += 1
                elif p.mode == "head":
                    seen[:, p.start:p.stop] += 1
                else:
                    for f in range(p.start, p.stop):
                        seen[f // H, f % H] += 1
            assert (seen == 1).all(), (B, H, world)


def test_plan_prefers_views():
    assert shard.plan(8, 32, 8, 0).mode == "batch"   # config 4 on 8 GPUs: one batch per GPU
    assert shard.plan(2, 16, 4, 0).mode == "head"
    assert shard.plan(3, 5, 2, 0).mode == "pairs"


def _oracle_fwd(q, k, v, beta, g, initial_state=None, **kw):
    from oracle import gdn_oracle as ora
    f = lambda x: None if x is None else x.numpy()
    o, h = ora.chunked(f(q), f(k), f(v), f(beta), f(g), C=16, initial_state=f(initial_state), dtype=np.float64)
    return torch.from_numpy(o), torch.from_numpy(h)


def _worker(rank, world, port, B, H, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import gdn_oracle as ora
        q, k, v, b, g, h0 = ora.make_inputs(B, 32, H, 16, 16, seed=5, h0_std=0.1)
        t = torch.from_numpy
        p = shard.plan(B, H, world, rank)
        o_l, h_l = shard.run_local(p, t(q), t(k), t(v), t(b), t(g), t(h0), fwd=_oracle_fwd)
        o, h = shard.gather_outputs(p, o_l, h_l)
        o_ref, h_ref = _oracle_fwd(t(q), t(k), t(v), t(b), t(g), t(h0))
        ok = torch.allclose(o, o_ref, atol=1e-10) and torch.allclose(h, h_ref, atol=1e-10)
        result_q.put((rank, bool(ok), p.mode))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("B,H", [(2, 3), (1, 4)])
def test_two_rank_gloo_shards_match_full_batch(B, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, H, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = [q.get(timeout=5) for _ in range(2)]
    assert all(ok for _, ok, _ in results), results
    assert all(p.exitcode == 0 for p in procs)


def _dropout_worker(rank, world, port, result_q):
    """Rank 1 leaves before the gather; rank 0's collective must end with an
    error within the process-group timeout instead of waiting forever."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        result_q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001
        result_q.put((rank, "error:" + type(e).__name__))


def test_rank_dropout_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    res = q.get(timeout=5)
    assert res[0] == 0 and res[1].startswith("error"), res
    for p in procs:
        if p.is_alive():
            p.kill()
