"""Benchmark of the higher-order SDPA path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl theria|reference]
                    [--workload fwdbwd|fwdbwd_causal|jvp|hvp|maml] [--no-extra]

Headline (one JSON line on rank 0): bf16 SDPA forward+backward TFLOP/s at
B=4, H=16, N=4096, D=128, non-causal (configs[1] of the benchmark plan), as
the whole-job aggregate over N GPUs.  Each rank runs that full workload on
its own shard of batch*head units (weak scaling, no collective on the data
path).  A step is one forward (O, LSE) plus one backward (dQ, dK, dV).

Algorithmic FLOPs (non-causal; causal x (N+1)/(2N)):
  fwd 4 BHN^2D, fwd+bwd 14 BHN^2D, bwd 10 BHN^2D, JVP 12 BHN^2D,
  HVP 32 BHN^2D.

Keys beyond the base contract: ``e2e`` (same metric through the public
autograd API with pinned host inputs copied in and gradients copied out
inside the timed region), ``roofline`` (the backward launch against the
measured dense-bf16 peak), ``cpu_baseline`` (the CPU oracle, a restatement
of the reference's CPU math, on a bounded sample), ``clocks``,
``gpu_launches`` and ``extra`` (JVP / HVP at configs[2] and the full-MAML
meta-step at configs[3]).

``--impl reference`` times the reference's CPU implementation of the path
(the oracle port, since the reference is pure Python/PyTorch and does not
travel to the GPU box) with all host threads on a bounded sample of the
same workload; under torchrun only rank 0 runs.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CFG2 = dict(B=4, H=16, N=4096, D=128)
CFG3 = dict(B=2, H=8, N=2048, D=64)

# DRAM bytes per launch of the backward's main kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum), keyed by workload; None
# until a capture exists for the kernel that runs.  The capture of
# bwd_kernel at B=1 H=16 N=4096 D=128 read 101.3 MB and wrote 22.7 MB;
# traffic grows with the (b, h) units, so x4 for B=4.
NCU_TRAFFIC_BYTES: dict[str, float | None] = {"cfg2": 4 * (101.3e6 + 22.7e6)}


def flops(kind, B, H, N, D, causal=False):
    per = {"fwd": 4, "bwd": 10, "fwdbwd": 14, "jvp": 12, "hvp": 32}[kind]
    f = per * B * H * N * N * D
    return f * (N + 1) / (2 * N) if causal else f


def load_peaks():
    if os.path.exists(PEAKS_FILE):
        with open(PEAKS_FILE) as fh:
            return json.load(fh), "measured"
    return FALLBACK_PEAKS, "fallback"


# ------------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ host placement
def bind_to_gpu_numa(dev):
    """Pin this process to the CPUs of the GPU's own NUMA node (read from
    sysfs), so pinned host buffers allocated afterwards live next to the
    GPU's PCIe root and host<->device copies do not cross sockets.  Returns
    the CPU list used, or None when the topology is not available."""
    try:
        pr = torch.cuda.get_device_properties(dev)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        path = f"/sys/bus/pci/devices/{bus}/local_cpulist"
        if not os.path.exists(path):
            return None
        cpus = set()
        for part in open(path).read().strip().split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.update(range(int(a), int(b) + 1))
            elif part:
                cpus.add(int(part))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return sorted(cpus)
    except (OSError, ValueError, AttributeError):
        return None
    return None


# ------------------------------------------------------------------ helpers
def randn(shape, gen, dtype, device):
    return torch.randn(*shape, generator=gen, dtype=torch.float32).to(dtype).to(device)


def launch_count():
    from theria_b200 import _lib
    return int(_lib.load().theria_launch_count())


def timed(fn, steps, warmup, world):
    """Run fn warmup times, then time exactly `steps` calls with CUDA events.

    Barrier + synchronize on both sides; returns (max-over-ranks ms/step,
    kernel launches of this library inside the timed region)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    n0 = launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    n1 = launch_count()
    barrier(world)
    ms = e0.elapsed_time(e1) / steps
    return max_over_ranks(ms, world), n1 - n0


def cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_fwdbwd_sample(budget_s=12.0, min_units=1, max_units=4096, dtype=torch.bfloat16):
    """The CPU oracle's fwd+bwd (autograd through the restated forward, as the
    reference's CPU path computes it) on whole (b, h) units of configs[1],
    repeated until `budget_s` of CPU work.  Returns (TFLOP/s, units, seconds)."""
    from oracle import sdpa_oracle as orc
    N, D = CFG2["N"], CFG2["D"]
    gen = torch.Generator("cpu").manual_seed(0)
    units, t_total = 0, 0.0
    while units < max_units and (units < min_units or t_total < budget_s):
        q, k, v, do = (torch.randn(1, 1, N, D, generator=gen).to(dtype).requires_grad_(i < 3)
                       for i in range(4))
        t0 = time.perf_counter()
        o = orc.attention(q, k, v)
        torch.autograd.grad(o, (q, k, v), do)
        t_total += time.perf_counter() - t0
        units += 1
    return flops("fwdbwd", 1, units, N, D) / t_total / 1e12, units, t_total


# ------------------------------------------------------------------ workloads
def run_fwdbwd(args, world, rank, dev, causal=False, with_e2e=True, dt=torch.bfloat16):
    from theria_b200.attention import ops
    B, H, N, D = CFG2["B"], CFG2["H"], CFG2["N"], CFG2["D"]
    gen = torch.Generator("cpu").manual_seed(rank)  # rank r owns shard r of the job
    q, k, v, do = (randn((B, H, N, D), gen, dt, dev) for _ in range(4))

    def step():
        o, lse = ops.forward(q, k, v, causal=causal)
        ops.backward(q, k, v, do, lse, o=o, causal=causal)

    with ClockSampler(dev.index) as clk:
        ms, launches = timed(step, args.steps, args.warmup, world)
    f = flops("fwdbwd", B, H, N, D, causal) * world
    out = {"ms_per_step": ms, "value": f / (ms * 1e-3) / 1e12,
           "gpu_launches": launches, "clocks": clk.summary()}

    # per-launch split of the step (same stream, CUDA events) for the roofline;
    # a step queued ahead keeps the device busy, so no interval includes the
    # host's launch latency
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(5)]
    step()
    for e in evs:
        e[0].record()
        o, lse = ops.forward(q, k, v, causal=causal)
        e[1].record()
        ops.backward(q, k, v, do, lse, o=o, causal=causal)
        e[2].record()
    torch.cuda.synchronize()
    t_f = [e[0].elapsed_time(e[1]) for e in evs]
    t_b = [e[1].elapsed_time(e[2]) for e in evs]
    out["t_fwd_ms"] = statistics.median(t_f)
    out["t_bwd_ms"] = statistics.median(t_b)
    out["fwd_tflops"] = flops("fwd", B, H, N, D, causal) / (out["t_fwd_ms"] * 1e-3) / 1e12
    out["bwd_tflops"] = flops("bwd", B, H, N, D, causal) / (out["t_bwd_ms"] * 1e-3) / 1e12

    if with_e2e:
        out["e2e"] = run_e2e(args, world, rank, dev, causal)
    del q, k, v, do
    torch.cuda.empty_cache()
    return out


def run_e2e(args, world, rank, dev, causal):
    """Same metric through the public API: pinned host inputs -> device,
    sdpa_custom forward + autograd backward, gradients -> pinned host.

    Every step's host->device copy of its four inputs and device->host copy
    of its three gradients are inside the timed region; they run on two copy
    streams so that step i+1's inputs arrive and step i-1's gradients leave
    while step i computes (double-buffered device inputs, event ordering).
    """
    from theria_b200.attention.custom import sdpa_custom
    B, H, N, D = CFG2["B"], CFG2["H"], CFG2["N"], CFG2["D"]
    dt = torch.bfloat16
    gen = torch.Generator("cpu").manual_seed(rank)
    host = [torch.randn(B, H, N, D, generator=gen).to(dt).pin_memory() for _ in range(4)]
    outs = [torch.empty(B, H, N, D, dtype=dt).pin_memory() for _ in range(3)]
    bufs = [[torch.empty(B, H, N, D, dtype=dt, device=dev) for _ in range(4)] for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev(), ev()]
    computed = [ev(), ev()]
    out_done = [ev(), ev()]

    def h2d(b):
        with torch.cuda.stream(s_in):
            for d_, h_ in zip(bufs[b], host):
                d_.copy_(h_, non_blocking=True)
            in_ready[b].record(s_in)

    def run(steps):
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        h2d(0)
        for i in range(steps):
            b = i & 1
            comp.wait_event(in_ready[b])
            if i + 1 < steps:
                if i >= 1:
                    s_in.wait_event(computed[1 - b])  # step i-1 is done with buffer 1-b
                h2d(1 - b)
            q, k, v = (t.detach().requires_grad_(True) for t in bufs[b][:3])
            o = sdpa_custom(q, k, v, causal=causal)
            grads = torch.autograd.grad(o, (q, k, v), bufs[b][3])
            computed[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[b])
                for dst, g in zip(outs, grads):
                    dst.copy_(g, non_blocking=True)
                    g.record_stream(s_out)
                out_done[b].record(s_out)
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    for _ in range(args.warmup):
        run(2)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(args.steps)
    e1.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    f = flops("fwdbwd", B, H, N, D, causal) * world
    nbytes = B * H * N * D * 2
    return {"value": f / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 3 * nbytes,
            "overlap": "H2D of step i+1 and D2H of step i-1 overlap step i's compute"}


def run_jvp_hvp(args, world, rank, dev):
    from theria_b200.attention import ops
    B, H, N, D = CFG3["B"], CFG3["H"], CFG3["N"], CFG3["D"]
    dt = torch.bfloat16
    gen = torch.Generator("cpu").manual_seed(rank)
    q, k, v, tq, tk, tv, w = (randn((B, H, N, D), gen, dt, dev) for _ in range(7))
    steps = max(3, args.steps)
    _, lse = ops.forward(q, k, v)

    def fb():
        o, l2 = ops.forward(q, k, v)
        ops.backward(q, k, v, w, l2, o=o)

    ms_fb, _ = timed(fb, steps, 3, world)
    ms_j, _ = timed(lambda: ops.jvp(q, k, v, tq, tk, tv, lse), steps, 3, world)
    ms_h, _ = timed(lambda: ops.hvp(q, k, v, w, lse, tq, tk, tv), steps, 3, world)
    f = lambda kind, ms: flops(kind, B, H, N, D) * world / (ms * 1e-3) / 1e12  # noqa: E731
    return {"config": "configs[2] bf16 B2 H8 N2048 D64",
            "fwdbwd_ms": ms_fb, "fwdbwd_tflops": f("fwdbwd", ms_fb),
            "jvp_ms": ms_j, "jvp_tflops": f("jvp", ms_j), "jvp_over_fwdbwd": ms_j / ms_fb,
            "hvp_ms": ms_h, "hvp_tflops": f("hvp", ms_h), "hvp_over_fwdbwd": ms_h / ms_fb}


def run_strong_split(args, world, rank, dev, peak):
    """The fixed configs split over the ranks (strong scaling): configs[1]'s
    B*H = 64 (b, h) units and configs[2]'s 16 units are divided evenly, each
    rank running its units as one [1, units, N, D] call; aggregate TFLOP/s =
    the whole config's flops / the max rank time."""
    from theria_b200.attention import ops
    res = {}
    for name, cfg, kinds in (("cfg2_fwdbwd", CFG2, ("fwdbwd",)),
                             ("cfg3_jvp_hvp", CFG3, ("fwdbwd", "jvp", "hvp"))):
        B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
        units = B * H
        per = units // world
        gen = torch.Generator("cpu").manual_seed(100 + rank)
        q, k, v, w, tq, tk, tv = (randn((1, per, N, D), gen, torch.bfloat16, dev)
                                  for _ in range(7))
        _, lse = ops.forward(q, k, v)
        steps = max(5, args.steps)

        def fb():
            o, l2 = ops.forward(q, k, v)
            ops.backward(q, k, v, w, l2, o=o)

        fns = {"fwdbwd": fb, "jvp": lambda: ops.jvp(q, k, v, tq, tk, tv, lse),
               "hvp": lambda: ops.hvp(q, k, v, w, lse, tq, tk, tv)}
        out = {"units_total": units, "units_per_rank": per}
        for kind in kinds:
            ms, _ = timed(fns[kind], steps, 3, world)
            tf = flops(kind, B, H, N, D) / (ms * 1e-3) / 1e12
            out[kind + "_ms"] = ms
            out[kind + "_tflops"] = tf
            out[kind + "_frac"] = tf / (peak * world)  # per GPU, of one GPU's peak
        res[name] = out
        del q, k, v, w, tq, tk, tv, lse
    torch.cuda.empty_cache()
    return res


def run_maml(args, world, rank, dev, steps=None):
    """meta-batch 32 tasks sharded over the ranks, 5 inner SGD
    steps (lr 0.4, create_graph=True), Adam 1e-3, one gradient all-reduce."""
    from theria_b200.maml.distributed import MetaStep, broadcast_params, shard_range
    from theria_b200.maml.model import MAMLClassifier, ModelConfig
    from theria_b200.maml.tasks import sample_tasks, stack_tasks
    torch.manual_seed(0)
    model = MAMLClassifier(ModelConfig()).to(dev)
    broadcast_params(model)
    meta_batch = 32
    start, per = shard_range(meta_batch, rank, world)
    from theria_b200.maml.distributed import GraphedMetaStep
    ms_step = MetaStep(model, meta_batch=meta_batch, inner_lr=0.4, inner_steps=5, fo=False,
                       outer_lr=1e-3, world=world, capturable=True)
    pool = [stack_tasks(sample_tasks(1000 + i, per, start=start), pin=True) for i in range(4)]
    n0 = launch_count()
    graphed = GraphedMetaStep(ms_step, pool[0])  # 3 eager warm-up steps + the capture
    captured = (launch_count() - n0) // 4  # this library's kernels in one step
    it = [0]

    def step():
        # host tasks -> device buffers of the captured step, then replay
        graphed.step(pool[it[0] % len(pool)])
        it[0] += 1

    steps = steps or max(3, args.steps)
    ms, _ = timed(step, steps, 3, world)
    return {"config": "configs[3] full MAML, meta-batch 32, k=5, meta-step captured in a CUDA graph",
            "ms_per_meta_step": ms,
            "meta_steps_per_s": 1000.0 / ms, "tasks_per_rank": per,
            "theria_kernels_per_step": captured,
            "note": "replays launch the captured kernels without calling the library, "
                    "so its launch counter sees them only at capture"}


def run_sweep(args, world, rank, dev, peak, points=None):
    """causal bf16, B=1, H=32, D in {64,128}, N in 512..16384;
    heads sharded over the ranks (H/world each, strong split: the total is
    fixed); fwd, fwd+bwd, JVP, HVP as aggregate TFLOP/s (all 32 heads' flops
    over the max rank time) and as a fraction of the dense-bf16 peak."""
    from theria_b200.attention import ops
    H = 32 // world
    out = []
    if points is None:
        points = [(D, N) for D in (64, 128) for N in (512, 1024, 2048, 4096, 8192, 16384)]
    for D, N in points:
        if True:
            gen = torch.Generator("cpu").manual_seed(rank)
            q, k, v, w, tq, tk, tv = (randn((1, H, N, D), gen, torch.bfloat16, dev)
                                      for _ in range(7))
            o, lse = ops.forward(q, k, v, causal=True)
            steps = 3 if N >= 8192 else 10
            t_f, _ = timed(lambda: ops.forward(q, k, v, causal=True), steps, 3, world)
            t_b, _ = timed(lambda: ops.backward(q, k, v, w, lse, o=o, causal=True), steps, 3,
                           world)
            t_j, _ = timed(lambda: ops.jvp(q, k, v, tq, tk, tv, lse, causal=True), steps, 3,
                           world)
            t_h, _ = timed(lambda: ops.hvp(q, k, v, w, lse, tq, tk, tv, causal=True), steps, 3,
                           world)
            f = lambda kind, ms: flops(kind, 1, 32, N, D, True) / (ms * 1e-3) / 1e12  # noqa: E731
            pt = {"D": D, "N": N, "fwd_tflops": f("fwd", t_f),
                  "fwdbwd_tflops": f("fwdbwd", t_f + t_b), "jvp_tflops": f("jvp", t_j),
                  "hvp_tflops": f("hvp", t_h), "fwd_ms": t_f, "bwd_ms": t_b,
                  "jvp_ms": t_j, "hvp_ms": t_h}
            for kind in ("fwd", "fwdbwd", "jvp", "hvp"):
                pt[kind + "_frac"] = pt[kind + "_tflops"] / (peak * world)  # per GPU
            out.append(pt)
            del q, k, v, w, tq, tk, tv, o, lse
    torch.cuda.empty_cache()
    return {"config": f"configs[4] causal bf16 B=1 H=32, {H} heads per rank (strong split), "
                      "fwd+bwd = fwd + bwd launch times",
            "peak_tflops": peak, "points": out}


# ------------------------------------------------------------------ arms
METRIC = "SDPA fwd+bwd TFLOP/s (bf16, N=4096)"
CONFIG = {"workload": "configs[1]: SDPA fwd+bwd, bf16, B=4 H=16 N=4096 D=128, non-causal, "
                      "scale 1/sqrt(D), each rank its own B*H shard",
          "global_batch": None, "seq_len": 4096, "head_dim": 128, "heads": 16,
          "batch_per_rank": 4, "parallelism": None,
          "l2": "inputs larger than L2 (4 x 64 MiB per rank), no flush"}


def reference_arm(args, world, rank):
    if rank != 0:
        return
    cores = cpu_threads()
    vals = []
    for i in range(args.warmup + args.steps):
        tf, units, secs = cpu_fwdbwd_sample(budget_s=0.0, min_units=1, max_units=1)
        if i >= args.warmup:
            vals.append(tf)
    v = statistics.median(vals)
    sample = ("CPU oracle fwd+bwd (reference_attention restated + autograd, bf16) on one "
              "(b,h) unit [1,1,4096,128] of configs[1] per step")
    cfg = dict(CONFIG, global_batch=4 * world, parallelism=f"dp{world}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops("fwdbwd", 1, 1, 4096, 128) / (v * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1), seeded", "config": cfg,
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def theria_arm(args, world, rank, local):
    import theria_b200  # noqa: F401  (fails loudly if the library is missing)
    from theria_b200 import _lib
    _lib.load()
    dev = torch.device("cuda", local)
    all_cpus = os.sched_getaffinity(0)
    numa_cpus = bind_to_gpu_numa(dev)
    peaks, peak_src = load_peaks()
    # every timed launch here is short (milliseconds, at most a few seconds of
    # steps), so the burst dense-bf16 figure is the denominator
    peak = peaks["bf16_tflops"]
    causal = args.workload == "fwdbwd_causal"
    res = run_fwdbwd(args, world, rank, dev, causal=causal)
    _lib.check_device_error(local)
    extra = {}
    if not args.no_extra:
        extra["jvp_hvp"] = run_jvp_hvp(args, world, rank, dev)
        extra["maml"] = run_maml(args, world, rank, dev)
        if not causal:
            c = run_fwdbwd(args, world, rank, dev, causal=True, with_e2e=False)
            extra["fwdbwd_causal"] = {"tflops": c["value"], "ms_per_step": c["ms_per_step"],
                                      "frac": c["value"] / world / peak}
        f16 = run_fwdbwd(args, world, rank, dev, causal=causal, with_e2e=False,
                         dt=torch.float16)
        extra["fwdbwd_fp16"] = {"config": "configs[1] in fp16", "tflops": f16["value"],
                                "ms_per_step": f16["ms_per_step"],
                                "frac": f16["value"] / world / peak,
                                "fwd_tflops": f16["fwd_tflops"], "bwd_tflops": f16["bwd_tflops"]}
        extra["strong_split"] = run_strong_split(args, world, rank, dev, peak)
        extra["long_seq_sweep"] = run_sweep(
            args, world, rank, dev, peak,
            points=None if args.sweep else [(64, 4096), (64, 16384), (128, 4096), (128, 16384)])
        _lib.check_device_error(local)
    if rank != 0:
        return
    achieved = res["bwd_tflops"]
    key = "cfg2_causal" if causal else "cfg2"
    traffic = NCU_TRAFFIC_BYTES.get(key)
    roofline = {"kernel": "theria_sdpa_bwd (z prepass + dQ/dK/dV kernels of one call)",
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "peak_source": f"{peak_src} (bf16_tflops, burst: each launch is timed alone)",
                "algorithmic_flops_per_launch": flops("bwd", 4, 16, 4096, 128, causal),
                "launch_ms": res["t_bwd_ms"],
                "fwd": {"achieved": res["fwd_tflops"], "frac": res["fwd_tflops"] / peak,
                        "launch_ms": res["t_fwd_ms"]}}
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
    cores = cpu_threads()
    tf, units, secs = cpu_fwdbwd_sample(budget_s=args.cpu_budget)
    cfg = dict(CONFIG, global_batch=4 * world, parallelism=f"dp{world}")
    if causal:
        cfg["workload"] = cfg["workload"].replace("non-causal", "causal")
    line = {
        "metric": METRIC + (" causal" if causal else ""), "value": res["value"],
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded per rank",
        "config": cfg, "e2e": dict(res["e2e"], host_cpus=(
            f"{len(numa_cpus)} CPUs of the GPU's NUMA node" if numa_cpus else "unbound")),
        "gpu_launches": res["gpu_launches"],
        "clocks": res["clocks"], "roofline": roofline,
        "cpu_baseline": {"value": tf, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"CPU oracle fwd+bwd, bf16, {units} (b,h) units "
                                   f"[1,1,4096,128] of configs[1], {secs:.1f} s"},
        "extra": extra,
    }
    print(json.dumps(line), flush=True)


def profile_maml_step(tasks=4, top=25):
    """Kernel list of one eager full-MAML meta-step at the 8-GPU share (4
    tasks), from the torch profiler (CUPTI): per kernel name its launches,
    device time and share."""
    import collections
    from torch.profiler import ProfilerActivity, profile
    from theria_b200.maml.distributed import MetaStep
    from theria_b200.maml.model import MAMLClassifier, ModelConfig
    from theria_b200.maml.tasks import sample_tasks, stack_tasks
    torch.cuda.set_device(0)
    torch.manual_seed(0)
    model = MAMLClassifier(ModelConfig()).cuda()
    ms = MetaStep(model, meta_batch=32, inner_lr=0.4, inner_steps=5, fo=False, world=1,
                  capturable=True)
    tb = stack_tasks(sample_tasks(1000, tasks)).to("cuda")
    for _ in range(3):
        ms.step(tb)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        ms.step(tb)
        torch.cuda.synchronize()
    cnt, tim = collections.Counter(), collections.Counter()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            cnt[ev.name] += 1
            tim[ev.name] += ev.device_time
    total = sum(tim.values())
    print(f"kernels {sum(cnt.values())}  device time {total / 1000:.2f} ms  (tasks {tasks})")
    for name, t in tim.most_common(top):
        print(f"{cnt[name]:5d}  {t:9.1f} us  {100 * t / total:5.1f} %  {name[:110]}")


def profile_case(case):
    """A few launches of one operator at a size ncu can capture in minutes
    (inputs still larger than L2): --profile-case fwdbwd|fwd64|bwd64|jvp|hvp, or
    maml_heads: forward + HVP of 3,200 fp32 MAML heads [800, 4, 64, 16]
    (the whole-head kernels); maml_step: kernel list of one meta-step."""
    from theria_b200.attention import ops
    torch.cuda.set_device(0)
    if case == "maml_step":
        return profile_maml_step()
    if case == "maml_heads":
        shape = (800, 4, 64, 16)
    elif case == "fwd64":
        shape = (1, 32, 8192, 64)
    elif case == "bwd64":
        shape = (1, 32, 4096, 64)
    elif case == "fwdbwd":
        shape = (1, 16, 4096, 128)
    else:
        shape = (CFG3["B"], CFG3["H"], CFG3["N"], CFG3["D"])
    gen = torch.Generator("cpu").manual_seed(0)
    dt = torch.float32 if case == "maml_heads" else torch.bfloat16
    q, k, v, w, tq, tk, tv = (randn(shape, gen, dt, "cuda") for _ in range(7))
    for _ in range(3):
        o, lse = ops.forward(q, k, v)
        if case in ("fwdbwd", "bwd64"):
            ops.backward(q, k, v, w, lse, o=o)
        elif case == "jvp":
            ops.jvp(q, k, v, tq, tk, tv, lse)
        elif case != "fwd64":
            ops.hvp(q, k, v, w, lse, tq, tk, tv)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "shape": list(shape), "ok": True}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["theria", "reference"], default="theria")
    ap.add_argument("--workload", choices=["fwdbwd", "fwdbwd_causal"], default="fwdbwd")
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="run every configs[4] sweep point (default: D 64/128 x N 4096/16384)")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--profile-case",
                    choices=["fwdbwd", "fwd64", "bwd64", "jvp", "hvp", "maml_heads", "maml_step"],
                    default=None,
                    help="run a few launches of one operator for ncu, print no bench line")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case)
        return
    if args.warmup < 3:
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")),
                          int(os.environ.get("RANK", "0")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return
    world, rank, local = dist_setup()
    theria_arm(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
