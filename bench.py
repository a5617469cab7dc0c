"""Benchmark of the chunked Gated DeltaNet forward (replaces the reference's bench_gdn.py).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|2|3|4]

One JSON line on stdout (rank 0).  Metric: GDN fwd Mtokens/s (tokens = B*T).
The default workload is the headline shape, config 2: B=2, T=4096, H=16,
K=V=128, bf16 inputs, C=64, h0 ~ N(0, 0.1), fp32 state.

* ``value``     device-resident throughput: inputs already in HBM, K forwards
                replayed from a CUDA graph, CUDA events around exactly K steps
                on the launching stream, max over ranks.
* ``eager``     the same K forwards as plain calls of ``gdn_chunk_fwd`` (no
                graph): device time per step and the host time per call
                (argument checks, ctypes, tensor maps, launches).
* ``e2e``       the same metric through the public Python API with pinned host
                buffers: every step copies its inputs host->device and reads o
                and the final state back (copies of neighbouring steps overlap
                on separate streams, as a streaming caller would run them).
* ``roofline``  one forward (the prep kernel and the scan kernel it feeds):
                its algorithmic bytes / its average device time, against the
                measured HBM copy bandwidth; ``traffic`` is the DRAM bytes of
                both kernels per forward from the committed ncu summary.
* ``cpu_baseline`` the reference's chunked CPU path (gdn_ref.gdn_chunk_ref,
                restated in torch fp32 in oracle/gdn_chunk_torch.py) on the
                host cores, full B*H, rank 0 at N=1 only.

Multi-GPU (torchrun, one process per GPU): the (batch, head) pairs of one
global input set are split by ``gdn_b200.shard.plan`` and each rank runs its
shard through ``shard.local_inputs`` (views of the global tensors); the hot
path has no collective.  Configs 1-3 scale weakly (the global batch is B*N,
each rank owns the config's shape); config 4 (B8 T8192 H32) scales strongly
(one global problem split N ways).  ``--impl reference`` times the
reference's CPU path on the same config and prints the same line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "v100-attention-lab_b200"), ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "GDN fwd Mtokens/s (B2 H16 K=V=128 T4096 bf16) + % of roofline"
UNIT = "Mtokens/s"

CONFIGS = {
    1: dict(name="config1: B2 T2048 H8 K=V=128 fp16 C64 h0=0", B=2, T=2048, H=8, dtype="fp16", h0=False,
            gate_mean=0.0, scaling="weak"),
    2: dict(name="config2: B2 T4096 H16 K=V=128 bf16 C64 h0~N(0,0.1)", B=2, T=4096, H=16, dtype="bf16", h0=True,
            gate_mean=0.0, scaling="weak"),
    3: dict(name="config3: B2 T65536 H16 K=V=128 bf16 C64 g=logsigmoid(N(2,1))", B=2, T=65536, H=16, dtype="bf16",
            h0=False, gate_mean=2.0, scaling="weak"),
    4: dict(name="config4: B8 T8192 H32 K=V=128 bf16 C64 h0~N(0,0.1), (b,h) sharded", B=8, T=8192, H=32,
            dtype="bf16", h0=True, gate_mean=0.0, scaling="strong"),
}
K_DIM = V_DIM = 128
CHUNK = 64


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def measured_traffic(config):
    """DRAM bytes per forward from the committed ncu summary, if one covers this config."""
    path = os.path.join(ROOT, "profiles", f"gdn_fwd_config{config}_traffic.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1])
    except OSError:
        pass
    return None


def algo_bytes(B, T, H, s_in=2, s_out=2, h0=True):
    """Algorithmic HBM bytes of one forward: q,k,v read, o written, beta/g read,
    h0 read (if given) and the final state written."""
    per_tok_head = (2 * K_DIM + V_DIM) * s_in + V_DIM * s_out + 8
    state = K_DIM * V_DIM * 4 * (2 if h0 else 1)
    return B * T * H * per_tok_head + B * H * state


def algo_flops(B, T, H, C=CHUNK):
    """6KV + 4CK + 2CV + C(K+V) flops per token per head."""
    K, V = K_DIM, V_DIM
    return B * T * H * (6 * K * V + 4 * C * K + 2 * C * V + C * (K + V))


# ----------------------------------------------------------------------------- inputs
def make_inputs(cfg, B, seed, device):
    """Seeded synthetic inputs with the workload's distributions: q, k
    L2-normalised N(0,1) rows, v ~ N(0,1), beta = sigmoid(N(0,1)),
    g = logsigmoid(N(gate_mean, 1)), h0 ~ N(0, 0.1) where the config has one.
    Generated on ``device``; the same seed gives the same tensors on every GPU."""
    dt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    T, H = cfg["T"], cfg["H"]
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def l2n(x):
        return x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)

    q = l2n(torch.randn(B, T, H, K_DIM, device=device, generator=g)).to(dt)
    k = l2n(torch.randn(B, T, H, K_DIM, device=device, generator=g)).to(dt)
    v = torch.randn(B, T, H, V_DIM, device=device, generator=g).to(dt)
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=g))
    gg = torch.nn.functional.logsigmoid(torch.randn(B, T, H, device=device, generator=g) + cfg["gate_mean"])
    h0 = torch.randn(B, H, V_DIM, K_DIM, device=device, generator=g) * 0.1 if cfg["h0"] else None
    return q, k, v, beta, gg, h0


def global_batch(cfg, world):
    """Batch of the global problem: the config's own B for strong scaling,
    B per rank for weak scaling."""
    return cfg["B"] if cfg["scaling"] == "strong" else cfg["B"] * world


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        try:
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.gpu = str(device.index or 0)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), pw=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [r for r in rows if r["pw"] > 200.0] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": rows[0]["smax"],
                "reasons": sorted(reasons), "samples": len(loaded),
                "power_w_median": statistics.median(r["pw"] for r in loaded)}


# ----------------------------------------------------------------------------- CPU baseline
def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_inputs(cfg, B, H, seed=3):
    """CPU tensors of the workload's shape and distributions (bf16/fp16 q, k, v)."""
    return make_inputs(dict(cfg, H=H), B, seed, torch.device("cpu"))


def cpu_forward(cfg, B, H):
    """One call of the reference's chunked path (torch fp32 restatement) on B x H pairs."""
    from oracle.gdn_chunk_torch import chunked_fp32
    q, k, v, beta, g, h0 = cpu_inputs(cfg, B, H)
    T = cfg["T"]
    assert T % CHUNK == 0

    def run():
        return chunked_fp32(q, k, v, beta, g, C=CHUNK, initial_state=h0)
    return run


def cpu_baseline(cfg, budget_s=15.0):
    """Time the reference's chunked CPU path on the host cores: the full
    workload (all B*H pairs) repeated until ~budget_s of CPU time, at least once."""
    torch.set_num_threads(os.cpu_count() or 1)
    B, T, H = cfg["B"], cfg["T"], cfg["H"]
    run = cpu_forward(cfg, B, H)
    run()  # first call: thread pool and allocator warm-up, not timed
    times = []
    while not times or (sum(times) < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": B * T / t / 1e6, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "host_cpus": os.cpu_count(), "cpu_model": _cpu_model(),
            "sample": f"gdn_chunk_ref (gdn_ref.py:48-99) restated in torch fp32, full workload B={B} T={T} H={H}, "
                      f"median of {len(times)} runs ({sum(times):.1f} s), torch threads {torch.get_num_threads()}"}


# ----------------------------------------------------------------------------- distributed
def dist_setup(n):
    if n <= 1 or "RANK" not in os.environ:
        return 0, 1, 0
    import datetime
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size(), local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------- arms
def run_reference(args, cfg, rank, world, budget_s=120.0):
    """The reference's CPU path on rank 0 (other ranks exit without work).

    Each step is one forward of the workload on the host cores; when K full
    forwards would not fit in ~budget_s, each step is a bounded sample (the
    first pairs of the workload), and tokens are counted for the pairs run."""
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    B, T, H = cfg["B"], cfg["T"], cfg["H"]
    steps = max(1, args.steps)
    one = cpu_forward(cfg, 1, 1)
    one()
    t0 = time.perf_counter()
    one()
    t_pair = time.perf_counter() - t0
    pairs = max(1, min(B * H, int(budget_s / steps / max(t_pair, 1e-6))))
    sb, sh = (pairs // H, H) if pairs >= H else (1, pairs)
    run = cpu_forward(cfg, sb, sh)
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    val = sb * sh * T * steps / total / H / 1e6  # tokens of the full B*H workload per pair-set
    sample = (f"gdn_chunk_ref (gdn_ref.py:48-99) restated in torch fp32; each step {sb}x{sh} of {B}x{H} "
              f"(batch, head) pairs at T={T}, {steps} steps ({total:.1f} s), torch threads {torch.get_num_threads()}")
    cb = {"value": val, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
          "host_cpus": os.cpu_count(), "cpu_model": _cpu_model(), "sample": sample}
    return {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": total / steps * 1e3, "higher_is_better": True,
        "scaling": cfg["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; the workload's distributions)",
        "config": {"workload": cfg["name"], "B": B, "T": T, "H": H, "K": K_DIM, "V": V_DIM,
                   "chunk": CHUNK, "parallelism": "host cores"},
        "cpu_baseline": cb,
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def launches_per_forward(B, T, H):
    """Kernel launches of one gdn_chunk_fwd call: a prep and a scan launch per
    segment of chunks that fits the (capped) workspace."""
    from gdn_b200 import _lib, ops
    nt = -(-T // CHUNK)
    state = B * H * K_DIM * V_DIM * 4 + _lib.WORKSPACE_HEADER_BYTES
    per_chunk = B * H * _lib.PACKET_BYTES_PER_CHUNK
    need = nt * per_chunk + state
    ws = max(min(need, ops.WORKSPACE_CAP_BYTES), per_chunk + state)
    ns_max = (ws - state) // per_chunk
    return 2 * -(-nt // ns_max)


def run_ours(args, cfg, rank, world, local):
    import gdn_b200
    from gdn_b200 import _lib, shard
    _lib.load()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T, H = cfg["T"], cfg["H"]
    B_glob = global_batch(cfg, world)
    plan = shard.plan(B_glob, H, world, rank)
    # every rank builds the same global input sets from the global seeds and
    # runs its own (batch, head) block of them: the product's sharding path
    in_bytes_one = plan.pairs * T * (2 * K_DIM + V_DIM) * 2
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 * 2 ** 20)
    nsets = max(1, min(4, -(-2 * l2 // in_bytes_one)))  # rotate enough sets to exceed 2x L2
    sets = []
    for s in range(nsets):
        glob = make_inputs(cfg, B_glob, seed=1000 + s, device=dev)
        sets.append(shard.local_inputs(plan, *glob))
        del glob
    torch.cuda.empty_cache()
    B_rank = sets[0][0].shape[0]
    H_rank = sets[0][0].shape[2]
    out_dtype = sets[0][0].dtype

    def step(s):
        q, k, v, beta, g, h0 = sets[s % nsets]
        return gdn_b200.gdn_chunk_fwd(q, k, v, beta, g, initial_state=h0, chunk_size=CHUNK)

    # one launch checked for kernel errors before anything is timed
    step(0)
    gdn_b200.check_status(dev)

    # CUDA graph holding one forward per input set, replayed K / nsets times
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for s in range(nsets):
            step(s)
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for s in range(nsets):
            step(s)
    # exactly K timed steps: K // nsets replays of the full rotation, then the
    # first K % nsets input sets once more from a second graph
    steps = max(1, args.steps)
    reps, rem = divmod(steps, nsets)
    graph_rem = None
    if rem:
        graph_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_rem, stream=stream):
            for s in range(rem):
                step(s)
    for _ in range(max(3, -(-args.warmup // nsets))):
        graph.replay()
    if graph_rem is not None:
        graph_rem.replay()
    torch.cuda.synchronize(dev)

    # clocks: sampled over a ~1.5 s soak of the same replays and the timed region
    # right after it, so that the samples see the GPU under this load
    clocks = ClockSampler(dev)
    if rank == 0:
        clocks.start()
    soak_end = time.perf_counter() + (1.5 if rank == 0 or world > 1 else 0.0)
    while time.perf_counter() < soak_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    launch_stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(launch_stream)
    for _ in range(reps):
        graph.replay()
    if graph_rem is not None:
        graph_rem.replay()
    e1.record(launch_stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    if rank == 0:
        clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    gdn_b200.check_status(dev)
    tokens_all = B_glob * T * steps
    value = tokens_all / (ms / 1e3) / 1e6
    ms_per_step = ms / steps

    # eager: the same K forwards as plain calls on the current stream
    with torch.cuda.stream(stream):
        for s in range(3):
            step(s)
    torch.cuda.synchronize(dev)
    barrier(world)
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        g0.record(stream)
        h0t = time.perf_counter()
        for s in range(steps):
            step(s)
        host_s = time.perf_counter() - h0t
        g1.record(stream)
    torch.cuda.synchronize(dev)
    eager_ms = max_over_ranks(g0.elapsed_time(g1), world)
    host_us = max_over_ranks(host_s / steps * 1e6, world)
    gdn_b200.check_status(dev)

    # e2e: public API with pinned host buffers, H2D of inputs and D2H of o + h_final every step
    host = []
    for s in range(min(nsets, 2)):
        host.append([None if x is None else x.cpu().pin_memory() for x in sets[s]])
    e2e_steps = max(3, min(steps, 20))
    h2d = sum(x.numel() * x.element_size() for x in host[0] if x is not None)
    o_host = torch.empty(B_rank, T, H_rank, V_DIM, dtype=out_dtype).pin_memory()
    ht_host = torch.empty(B_rank, H_rank, V_DIM, K_DIM, dtype=torch.float32).pin_memory()
    d2h = o_host.numel() * o_host.element_size() + ht_host.numel() * 4

    # Three streams so that PCIe works both ways at once: the inputs of step j+1
    # travel host->device while step j computes and step j-1's outputs travel
    # back; every step still copies its own inputs in and its results out.
    h2d_s, cmp_s, d2h_s = (torch.cuda.Stream(device=dev) for _ in range(3))
    dbuf = [[None if x is None else torch.empty(x.shape, dtype=x.dtype, device=dev) for x in host[0]]
            for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n):
        for j in range(n):
            b = j % 2
            with torch.cuda.stream(h2d_s):
                if j >= 2:
                    h2d_s.wait_event(ev_cmp[b])  # step j-2 finished reading this buffer
                for d, h in zip(dbuf[b], host[j % len(host)]):
                    if d is not None:
                        d.copy_(h, non_blocking=True)
                ev_in[b].record(h2d_s)
            with torch.cuda.stream(cmp_s):
                cmp_s.wait_event(ev_in[b])
                o, ht = gdn_b200.gdn_chunk_fwd(*dbuf[b][:5], initial_state=dbuf[b][5], chunk_size=CHUNK)
                ev_cmp[b].record(cmp_s)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ev_cmp[b])
                o_host.copy_(o, non_blocking=True)
                ht_host.copy_(ht, non_blocking=True)
                o.record_stream(d2h_s)
                ht.record_stream(d2h_s)

    e2e_run(2)
    torch.cuda.synchronize(dev)
    barrier(world)
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(h2d_s)
    e2e_run(e2e_steps)
    f1.record(d2h_s)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    e2e_value = B_glob * T * e2e_steps / (e2e_ms / 1e3) / 1e6

    if rank != 0:
        return None
    hbm, tf, peak_src = load_peaks()
    # roofline of one rank's forward (its shard), timed as the slowest rank's
    abytes = algo_bytes(B_rank, T, H_rank, h0=cfg["h0"])
    kern_s = ms_per_step / 1e3
    achieved = abytes / kern_s / 1e9
    flops = algo_flops(B_rank, T, H_rank)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded; the workload's distributions)",
        "config": {"workload": cfg["name"], "global_B": B_glob, "T": T, "H": H, "K": K_DIM, "V": V_DIM,
                   "chunk": CHUNK, "per_gpu": f"B={B_rank} H={H_rank} ({plan.mode} shard of the global batch)",
                   "l2": f"inputs rotate over {nsets} resident sets ({nsets * in_bytes_one / 1e6:.0f} MB > 2x L2)",
                   "parallelism": f"{world} GPU(s), disjoint (batch, head) shards (gdn_b200.shard), "
                                  f"no collective on the hot path"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": measured_traffic(args.config) if world == 1 else None,
                     "peak_source": peak_src, "algorithmic_bytes_per_launch": abytes,
                     "launch": "one forward = prep kernel + scan kernel",
                     "tensor_frac": flops / kern_s / 1e12 / tf},
        "eager": {"ms_per_step": eager_ms / steps, "value": tokens_all / (eager_ms / 1e3) / 1e6,
                  "host_us_per_call": host_us},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
        "gpu_launches": steps * launches_per_forward(B_rank, T, H_rank),
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", 0))
        line = run_reference(args, cfg, rank, args.gpus)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        line = run_ours(args, cfg, rank, world, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
