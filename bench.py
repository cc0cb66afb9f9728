#!/usr/bin/env python
"""GDN-2 operator benchmark on B200: fwd + bwd tokens/s at B=4, H=6, L=2048, D=128.

One step = the reference's timed objective (README.md:22-23, benchmarks/honest_gdn2.py:74-78):
grad of sum(o^2) + sum(h_final^2) w.r.t. q, k, v, w, b, g, forward included, h0 fixed, through
the public operator make_blr_trainable(cfg, scale) with the reference's benchmark config
(bt=128, bs2=64, dot_mode highest, solve/B3 bf16x3, wy_eps=0; benchmarks/README.md:24).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--dtype fp32|bf16]

N > 1 runs under torchrun, one process per GPU.  The operator shards over batch x heads with no
communication (every head is an independent recurrence): the B*H = 24 heads of the one B4 H6 L2048
problem are split over the ranks ("1 GPU then B x H sharded over 2/4/8"), each
rank copies in only its heads' inputs and copies out only their results (strong scaling); time is
the max over ranks of the device time of the timed region; value = the problem's B*L tokens / that
time.  The line also carries the weak-scaling figure (every rank running a whole B4 H6 L2048
problem of its own) as the extra field `weak`.  Rank 0 prints one JSON line.  `--impl reference`
times the CPU oracle (a restatement of the reference's pure-JAX path; JAX is not available) on
the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "atomic-ops_b200"))

import torch  # noqa: E402

B, H, L, D = 4, 6, 2048, 128
T = 128
METRIC = "GDN-2 fwd+bwd tokens/s (B4 H6 L2048 D128)"
# Published reference number for this metric: 2.888 ms per fwd+bwd on TPU v5e-1 (README.md:30).
PUBLISHED_TOKS = B * L / 2.888e-3
CFG_KW = dict(bt=128, bc=64, score_bs=128, bs2=64, mb=8, wy_eps=0.0,
              dot_mode="highest", solve_dot_mode="bf16x3", b3_dot_mode="bf16x3")


def op_launches(nbh, nl, cfg, sms):
    """This library's kernel launches in one fwd+bwd operator call over nbh heads: per batch group
    (one launch sequence per side stream; one group when the chunk-heads fit in one wave of the
    `sms` multiprocessors) and segment group, fwd_intra (wide chunks included), the forward scan,
    fwd_out, bwd_pre, the backward scan, bwd_intra and its wide-channel launch."""
    from atomic_gdn2 import _lib
    seg = min(nl // T, cfg.max_chunks_per_call)
    groups = 1 if nbh * seg <= sms else min(_lib.batch_groups(), nbh)
    return 7 * groups * math.ceil((nl // T) / cfg.max_chunks_per_call)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--dtype", default="fp32", choices=["fp32", "bf16"])
    ap.add_argument("--workload", default="op", choices=["op", "lm"],
                    help="op: the operator's fwd+bwd tokens/s (headline); lm: the 8-layer LM training step")
    ap.add_argument("--torch-profile", action="store_true",
                    help="lm workload: also print torch.profiler's per-kernel CUDA time table for 2 steps")
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the headline line, print one line per sweep shape (BASELINE configs 3 and 4)")
    return ap.parse_args()


# --------------------------------------------------------------------------------------
# inputs (BASELINE config 2 distributions, generated on the device)
# --------------------------------------------------------------------------------------
def make_inputs(seed, device, dtype, shape=(B, H, L)):
    gen = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s: torch.randn(*s, generator=gen, device=device, dtype=torch.float32)
    l2 = lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)
    nb, nh, nl = shape
    sh = (nb, nh, nl, D)
    q, k, w = l2(n(*sh)), l2(n(*sh)), l2(n(*sh))
    v = n(*sh)
    b = torch.sigmoid(n(*sh))
    g = torch.nn.functional.logsigmoid(n(*sh) + 3.0)
    h0 = n(nb, nh, D, D) * 0.01
    return [t.to(dtype).contiguous() for t in (q, k, v, w, b, g)], h0.contiguous()


# --------------------------------------------------------------------------------------
# roofline bookkeeping: per chunk-head algorithmic FLOPs / compulsory HBM bytes per kernel
# (the split of the reference algorithm's GEMM list and compulsory traffic over the kernels)
# --------------------------------------------------------------------------------------
# Tensor-core cost of one algorithmic FLOP in a precision mode, in bf16-MMA equivalents: "highest"
# is three tf32 passes (tf32 MMAs run at half the bf16 rate), "bf16x3" three bf16 passes.
MODE_COST = {"highest": 6.0, "bf16x3": 3.0, "default": 1.0, "tf32": 2.0}


def mode_cost(tf32_ratio):
    """MODE_COST with the tf32 modes charged at a measured bf16 / tf32 throughput ratio."""
    return {"highest": 3.0 * tf32_ratio, "bf16x3": 3.0, "default": 1.0, "tf32": tf32_ratio}


def measured_tf32_tflops(dev):
    """Dense TF32 tensor-core throughput of this GPU, measured like MEASURED_PEAKS.json's bf16
    figure: a library fp32 GEMM with TF32 allowed, 8192^3 (2 N^3 FLOPs), best of 10 after warm-up,
    CUDA events.  Returns TFLOP/s."""
    n = 8192
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = torch.empty(n, n, device=dev)
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        return 2.0 * n ** 3 / (best / 1e3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def kernel_work(s_in, nc, modes, cost=MODE_COST):
    """Per chunk-head: (algorithmic FLOPs, bf16-equivalent MMA FLOPs in the configured modes,
    compulsory HBM bytes) of each kernel.  The FLOPs are the reference algorithm's dense GEMM count
    split over the kernels that perform its parts; B4 (four T^2 D products of bwd_intra) is
    fixed at "highest" (mega.py:13)."""
    t2d = T * T * D
    td2 = T * D * D
    t3 = T ** 3
    td = T * D
    dot, sol, b3 = (cost[modes[k]] for k in ("dot_mode", "solve_dot_mode", "b3_dot_mode"))
    hi = cost["highest"]
    f_fi, f_bi = 2 * 4 * t2d + (2 / 3) * t3, 2 * (10 * t2d + 3 * td2 + 2 * t3)
    return {
        "fwd_intra": (f_fi, 2 * 4 * t2d * dot + (2 / 3) * t3 * sol, 6 * s_in * td),
        "fwd_scan": (2 * 2 * td2, 2 * 2 * td2 * dot, 8 * D * D / nc),
        "fwd_out": (2 * (t2d + td2), 2 * (t2d + td2) * dot, 4 * td),
        "bwd_pre": (2 * (t2d + td2), 2 * (t2d + td2) * b3, 0),
        "bwd_scan": (2 * 2 * td2, 2 * 2 * td2 * b3, 8 * D * D / nc),
        "bwd_intra": (f_bi, 2 * 4 * t2d * hi + (f_bi - 2 * 4 * t2d) * b3, td * (12 * s_in + 4)),
    }


def peaks():
    """(HBM GB/s, bf16 dense TFLOP/s burst, bf16 dense TFLOP/s sustained, source).  The per-kernel
    times bench.py reports come from a few isolated steps, so the burst figure is their peak."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        burst = float(j["bf16_tflops"])
        return float(j["hbm_gbs"]), burst, float(j.get("bf16_tflops_sustained", burst)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes per kernel from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "ncu_traffic.txt"
    out = {}
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


# --------------------------------------------------------------------------------------
# host CPUs local to the GPU (placement of the end-to-end pinned buffers)
# --------------------------------------------------------------------------------------
def gpu_local_cpus(dev):
    """The host CPUs NVML reports as closest to this GPU (its NUMA node), or None.  Pinned host
    buffers first touched from these CPUs live in the GPU's local memory node, so host-to-device
    copies do not cross the inter-socket link."""
    try:
        import pynvml
        pr = torch.cuda.get_device_properties(dev)
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(
                f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0")
            words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        return cpus or None
    except Exception:
        return None


# --------------------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = [r.split(", ") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for nm, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------
# CPU baseline (oracle restatement of the reference's pure-JAX path, all host threads)
# --------------------------------------------------------------------------------------
def cpu_head_seconds(reps, warmup, budget_s=None):
    """Median seconds of one fwd+bwd of ONE head (B1 H1 L2048 D128, fp32) of the benchmark problem
    through the CPU oracle with every host thread.  Heads are independent recurrences, so the
    B4 H6 problem's CPU time is B*H = 24 times this.  With budget_s, reps grow (up to 30) to fill
    about that many seconds.  Returns (seconds, reps, threads)."""
    from oracle import gdn2_oracle as O  # test infrastructure: used here only as the CPU baseline
    torch.set_num_threads(os.cpu_count() or 1)
    (q, k, v, w, b, g), h0 = O.bench_inputs(1, 1, L, D, 0, dtype=torch.float32)
    ocfg = O.OracleCfg(bt=128, score_bs=128, mb=8, wy_eps=0.0)
    run = lambda: O.loss_and_grads(q, k, v, w, b, g, D ** -0.5, h0, ocfg)
    for _ in range(warmup):
        run()
    ts = []
    while len(ts) < reps or (budget_s and sum(ts) < budget_s and len(ts) < 30):
        t0 = time.perf_counter()
        run()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), len(ts), torch.get_num_threads()


CPU_SAMPLE = ("one head (B1 H1 L2048 D128) of the B4 H6 problem per timed call, fp32, fwd+bwd of "
              "sum(o^2)+sum(h_final^2); the problem's time is 24 x the median (heads are independent)")


def run_reference(args):
    """The reference arm: the reference's CPU path (its pure-JAX chunked-WY forward + autograd
    gradients, restated in PyTorch because JAX is absent) on every host core.  Each timed step is
    one head of the B4 H6 L2048 problem; `value` is the whole problem's tokens per second
    (B*L tokens / (24 x the per-head time)); ms_per_step is the time of the timed step itself."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    reps = max(1, args.steps)
    t_head, n, cores = cpu_head_seconds(reps, max(1, min(args.warmup, 2)))
    nbh = B * H
    val = B * L / (nbh * t_head)
    line = {
        "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": args.gpus, "steps": n,
        "warmup": args.warmup, "ms_per_step": t_head * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": val / PUBLISHED_TOKS, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "B4 H6 L2048 D128 fwd+bwd, timed one head per step", "global_batch": B,
                   "seq_len": L, "heads": H, "head_dim": D, "parallelism": "cpu"},
        "sample_scale": nbh, "problem_ms": nbh * t_head * 1e3,
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": CPU_SAMPLE},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is JAX/Pallas (TPU); JAX is not installed here, so the reference's pure-JAX "
                "chunked-WY path is timed as its PyTorch-CPU restatement (oracle/gdn2_oracle.py)",
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------------------
def status_gate(step, inputs, dist, max_over_ranks):
    """One step, then every rank's device status word read and reduced over the ranks: all ranks
    stop together when any word has a bit set, so that no rank is left alone in a collective."""
    import atomic_gdn2
    from atomic_gdn2.pipeline import _status_message
    atomic_gdn2.set_checks(False)
    step(inputs)
    torch.cuda.synchronize()
    code = int(max_over_ranks(float(atomic_gdn2.last_status())))
    if code:
        if dist is not None:
            dist.destroy_process_group()
        raise RuntimeError(_status_message(code, "first step (any rank)"))


def _time_graph(step, xs_base, dev, warmup, steps, flush=None):
    """Capture step(leaf inputs) once into a CUDA graph on a side stream (leaf tensors and warm-up
    live on the capture stream, so autograd's per-stream bookkeeping stays inside the capture).
    Returns (graph, captured leaf inputs) or (None, None) when capture is unavailable."""
    try:
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            xs_g = [t.detach().clone().requires_grad_(True) for t in xs_base]
            for _ in range(2):
                step(xs_g)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step(xs_g)
        torch.cuda.current_stream(dev).wait_stream(side)
        for _ in range(warmup):
            graph.replay()
        return graph, xs_g
    except Exception as exc:  # pragma: no cover - reported; the eager measurement stands
        print(f"bench: CUDA graph capture unavailable ({exc}); reporting the eager timing", file=sys.stderr)
        return None, None


def run_ours(args):
    import atomic_gdn2
    from atomic_gdn2 import _lib, make_blr_trainable, make_cfg
    from atomic_gdn2.sharding import bh_range, shard_heads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    dtype = torch.float32 if args.dtype == "fp32" else torch.bfloat16
    s_in = 4 if dtype == torch.float32 else 2
    cfg = make_cfg(**CFG_KW)
    if args.dtype == "bf16":
        cfg = cfg.with_(dot_mode="default", solve_dot_mode="default", b3_dot_mode="default")
    fn = make_blr_trainable(cfg, D ** -0.5)
    # the one B4 H6 L2048 problem (same seed on every rank); this rank's heads as (1, n_local, L, D)
    xs_all, h0_all = make_inputs(1234, dev, dtype)
    if world > 1:
        xs_base = [shard_heads(t, rank, world).contiguous() for t in xs_all]
        h0 = shard_heads(h0_all, rank, world).contiguous()
    else:
        xs_base, h0 = xs_all, h0_all
    hs, he = bh_range(B, H, rank, world)
    nbh_local = he - hs
    del xs_all, h0_all
    xs = [t.requires_grad_(True) for t in xs_base]

    def step(inputs):
        o, hf = fn(*inputs, h0)
        loss = (o * o).sum() + (hf * hf).sum()
        grads = torch.autograd.grad(loss, inputs)
        return loss, grads

    # correctness gate on every device before timing (device status words must stay clean)
    status_gate(step, xs, dist, max_over_ranks)

    for _ in range(args.warmup):
        step(xs)
    # eager timing (every launch issued by the host each step; device status checks at their
    # default, asynchronous setting, as a drop-in caller gets them -- on one rank only: with
    # several ranks an error raised on one of them would leave the others alone in a collective,
    # so there the words are read after the loops and reduced over the ranks)
    # The un-graphed step is bound by the host's issue rate (about 1 ms of Python, autograd and C
    # calls per step against 1 ms of device work), so it is timed in five rounds and the median
    # round is reported, with every round and the host's issue time per step beside it.
    atomic_gdn2.set_checks("async" if dist is None else False)
    barrier()
    eager_rounds, eager_host = [], []
    for _ in range(5):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(args.steps):
            loss, grads = step(xs)
        e1.record()
        eager_host.append((time.perf_counter() - t0) * 1e3 / args.steps)
        torch.cuda.synchronize()
        eager_rounds.append(e0.elapsed_time(e1) / args.steps)
    atomic_gdn2.set_checks(False)
    eager_ms = max_over_ranks(statistics.median(eager_rounds))
    # headline: the same step captured once into a CUDA graph and replayed (the analogue of the
    # reference's jitted XLA program: no per-launch host work inside the timed region)
    graph, xs_g = _time_graph(step, xs_base, dev, args.warmup, args.steps)
    clocks = Clocks(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    if graph is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms_local = e0.elapsed_time(e1) / args.steps
    else:  # the eager measurement above stands (a failed capture leaves no trustworthy stream state)
        ms_local = eager_ms
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ms_local)
    value = B * L / (ms / 1e3)

    # the reference's benchmark protocol (benchmarks/honest_gdn2.py:99-111): 3 seeds x 3 rounds x
    # (2 warm-up + 4 timed calls), median per round, median per seed, mean +- SD over seeds; each
    # timed call is one graph replay of the step on that seed's inputs, max over ranks
    protocol = None
    if graph is not None:
        per_seed = []
        for seed in (0, 1, 2):
            xa, _ = make_inputs(seed, dev, dtype)
            with torch.no_grad():
                for dst, src in zip(xs_g, xa):
                    dst.copy_(shard_heads(src, rank, world)[0].reshape(dst.shape) if world > 1 else src)
            del xa
            rounds = []
            for _ in range(3):
                for _ in range(2):
                    graph.replay()
                ts = []
                for _ in range(4):
                    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    barrier()
                    a.record()
                    graph.replay()
                    b_.record()
                    torch.cuda.synchronize()
                    ts.append(max_over_ranks(a.elapsed_time(b_)))
                rounds.append(statistics.median(ts))
            per_seed.append(statistics.median(rounds))
        mean = statistics.mean(per_seed)
        protocol = {"seeds": 3, "rounds": 3, "warmup_calls": 2, "timed_calls": 4,
                    "ms_per_seed": [round(x, 4) for x in per_seed], "ms_mean": mean,
                    "ms_sd": statistics.stdev(per_seed), "tokens_per_s": B * L / (mean / 1e3)}

    # weak-scaling figure (extra field): every rank runs a whole B4 H6 L2048 problem of its own
    weak = None
    if world > 1:
        xw, _ = make_inputs(4321 + rank, dev, dtype)
        with torch.no_grad():
            h0w = torch.randn(B, H, D, D, device=dev) * 0.01

        def step_w(inputs):
            o, hf = fn(*inputs, h0w)
            return torch.autograd.grad((o * o).sum() + (hf * hf).sum(), inputs)

        gw, _ = _time_graph(step_w, xw, dev, args.warmup, args.steps)
        if gw is not None:
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                gw.replay()
            e1.record()
            torch.cuda.synchronize()
            ms_w = max_over_ranks(e0.elapsed_time(e1) / args.steps)
            weak = {"value": world * B * L / (ms_w / 1e3), "unit": "tokens/s", "ms_per_step": ms_w,
                    "workload": "B4 H6 L2048 D128 per GPU (every rank its own problem)"}
            del gw
        del xw

    # per-kernel device time (CUDA events on the launching stream, inside the library) with this
    # rank's heads as one launch sequence (one batch group), so that every launch covers all of the
    # rank's chunk-heads, the units the roofline's algorithmic work counts
    groups = _lib.set_batch_groups(1)
    _lib.profile_enable(True)
    nprof = 3
    for _ in range(nprof):
        step(xs)
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    _lib.profile_enable(False)
    _lib.set_batch_groups(groups)

    # end to end through the public API with host buffers: every step copies this rank's inputs
    # from pinned host memory, and copies its results (o, h_final and the six gradients) and its
    # loss back to pinned host memory, where the host reads the loss.  The copies of the next two
    # steps' inputs run on a copy stream while step i computes (three device input buffers, events
    # order reuse); step i's results and loss go out on a third stream while step i+1 computes; the
    # host reads step i's loss once step i+2 has been issued (an event on the result stream), so
    # that no host wait sits in front of the copy engines' queues.  Measured against two buffers
    # and a synchronous read of step i-1's loss: 4.24 against 4.64 ms per step at B4 H6 L2048 fp32
    # (the copies alone take 3.83 ms).  The pinned buffers are allocated and filled from the CPUs
    # local to the GPU (NVML's affinity mask), as an input pipeline placed on the GPU's NUMA node
    # would; the process's affinity is restored afterwards (the CPU baseline below uses every core).
    saved_affinity = os.sched_getaffinity(0)
    local_cpus = gpu_local_cpus(dev)
    if local_cpus:
        os.sched_setaffinity(0, local_cpus)
    host = [t.detach().cpu().pin_memory() for t in xs_base]
    h2d = sum(t.numel() * t.element_size() for t in host)
    out_shapes = [((1 if world > 1 else B), (nbh_local if world > 1 else H), L, D, torch.float32),
                  ((1 if world > 1 else B), (nbh_local if world > 1 else H), D, D, torch.float32)]
    out_shapes += [tuple(t.shape) + (t.dtype,) for t in xs_base]
    NBUF, LAG = 3, 2
    host_out = [[torch.empty(sh[:-1], dtype=sh[-1]).pin_memory() for sh in out_shapes] for _ in range(NBUF)]
    e2e_steps = max(3, min(args.steps, 30))
    host_loss = torch.zeros(e2e_steps, dtype=torch.float32).pin_memory()
    d2h = sum(t.numel() * t.element_size() for t in host_out[0]) + host_loss.element_size()
    cs = torch.cuda.Stream(device=dev)
    os_ = torch.cuda.Stream(device=dev)
    bufs = [[torch.empty_like(t).requires_grad_(True) for t in xs_base] for _ in range(NBUF)]
    ready = [torch.cuda.Event() for _ in range(NBUF)]
    free = [torch.cuda.Event() for _ in range(NBUF)]
    loss_ev = [torch.cuda.Event() for _ in range(e2e_steps)]
    cur = torch.cuda.current_stream(dev)

    def step_out(inputs):
        o, hf = fn(*inputs, h0)
        loss = (o * o).sum() + (hf * hf).sum()
        grads = torch.autograd.grad(loss, inputs)
        return loss, [o.detach(), hf.detach(), *grads]

    def issue_copy(i, after=None):
        bi = i % NBUF
        with torch.cuda.stream(cs):
            if after is not None:
                cs.wait_event(after)
            if i >= NBUF:
                cs.wait_event(free[bi])
            for d_, h_ in zip(bufs[bi], host):
                d_.detach().copy_(h_, non_blocking=True)
            ready[bi].record(cs)

    def read_loss(i):
        loss_ev[i].synchronize()
        return float(host_loss[i])

    def run_e2e(n, start_event=None):
        for k in range(min(NBUF - 1, n)):
            issue_copy(k, start_event if k == 0 else None)
        lv = None
        for i in range(n):
            if i + NBUF - 1 < n:
                issue_copy(i + NBUF - 1)
            bi = i % NBUF
            cur.wait_event(ready[bi])
            loss, outs = step_out(bufs[bi])
            free[bi].record(cur)
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(os_):
                os_.wait_event(done)
                for dst, src in zip(host_out[bi], outs):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(os_)
                host_loss[i].copy_(loss.detach(), non_blocking=True)
                loss.record_stream(os_)
                loss_ev[i].record(os_)
            if i >= LAG:
                lv = read_loss(i - LAG)
        for j in range(max(0, n - LAG), n):
            lv = read_loss(j)
        cur.wait_stream(os_)
        return lv

    run_e2e(2)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(cur)
    run_e2e(e2e_steps, f0)
    f1.record(cur)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / e2e_steps)
    e2e_val = B * L / (e2e_ms / 1e3)
    os.sched_setaffinity(0, saved_affinity)
    status = atomic_gdn2.last_status()
    status = int(max_over_ranks(float(status)))

    if rank == 0:
        hbm, tf_burst, tf_sust, peak_kind = peaks()
        modes = {k: cfg.__dict__[k] for k in ("dot_mode", "solve_dot_mode", "b3_dot_mode")}
        tf32 = measured_tf32_tflops(dev)
        work = kernel_work(s_in, L // T, modes, mode_cost(tf_burst / tf32))
        nch = nbh_local * (L // T)
        traffic = ncu_traffic() if (dtype == torch.float32 and world == 1) else {}
        kern = {}
        for name, (tot_ms, cnt) in prof.items():
            if cnt == 0:
                continue
            per = tot_ms / cnt
            f, f_eff, by = work[name]
            t_f = f * nch / (tf_burst * 1e12)          # algorithmic FLOPs at the measured bf16 peak
            t_b = by * nch / (hbm * 1e9)               # compulsory bytes at the measured HBM copy rate
            t_mode = f_eff * nch / (tf_burst * 1e12)   # estimate: FLOPs at the modes' MMA cost
            kern[name] = {"ms_per_launch": per, "share": tot_ms, "flops": f * nch, "bytes": by * nch,
                          "t_roof_ms": max(t_f, t_b) * 1e3, "t_mode_ms": max(t_mode, t_b) * 1e3,
                          "bound": "tensor" if t_f >= t_b else "hbm"}
        tot = sum(k["share"] for k in kern.values()) or 1.0
        for k in kern.values():
            k["share"] = k["share"] / tot
        dom = max(kern, key=lambda n: kern[n]["share"])
        kd = kern[dom]
        sec = kd["ms_per_launch"] / 1e3
        tensor = {"achieved": kd["flops"] / sec / 1e12, "peak": tf_burst, "unit": "TFLOP/s"}
        tensor["frac"] = tensor["achieved"] / tensor["peak"]
        mem = {"achieved": kd["bytes"] / sec / 1e9, "peak": hbm, "unit": "GB/s"}
        mem["frac"] = mem["achieved"] / mem["peak"]
        main_ = tensor if kd["bound"] == "tensor" else mem
        t_step_roof = sum(k["t_roof_ms"] for k in kern.values())
        t_step_mode = sum(k["t_mode_ms"] for k in kern.values())
        cpu = None
        if world == 1:
            t_head, n_cpu, cores = cpu_head_seconds(3, 1, budget_s=10.0)
            cpu = {"value": B * L / (B * H * t_head), "unit": "tokens/s", "cores": cores, "kind": "port",
                   "sample": CPU_SAMPLE + f" ({n_cpu} timed calls)"}
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": value / PUBLISHED_TOKS,
            "timing": "CUDA-graph replay of the whole step" if graph is not None else "eager launches",
            "eager_ms_per_step": eager_ms,
            "eager": {"rounds_ms": [round(x, 4) for x in eager_rounds],
                      "host_issue_ms_per_step": round(statistics.median(eager_host), 4),
                      "note": "median of five rounds of the un-graphed step (rank 0's rounds shown)"},
            "dtype": "f32" if dtype == torch.float32 else "bf16", "data": "synthetic",
            "config": {"workload": "B4 H6 L2048 D128 fwd+bwd of sum(o^2)+sum(h_final^2) w.r.t. q,k,v,w,b,g"
                                   + (f", its 24 heads sharded over {world} GPUs" if world > 1 else ""),
                       "global_batch": B, "seq_len": L, "heads": H, "head_dim": D,
                       "parallelism": f"bh-shard x{world}" if world > 1 else "1 GPU",
                       "heads_per_gpu": nbh_local, "batch_groups": _lib.batch_groups(),
                       "modes": modes,
                       "l2": "inputs (6 x 25 MB), residuals (127 MB) and workspaces exceed the 126 MB L2"},
            "roofline": {"kernel": dom, "bound": kd["bound"], "achieved": main_["achieved"], "peak": main_["peak"],
                         "unit": main_["unit"], "frac": main_["frac"], "traffic": traffic.get(dom),
                         "algorithmic_bytes": kd["bytes"], "algorithmic_flops": kd["flops"],
                         "peak_source": f"{peak_kind} (bf16 dense burst; HBM copy)",
                         "tensor": tensor, "hbm": mem,
                         "bound_note": "bound = the larger of algorithmic FLOPs at the measured bf16 dense peak and "
                                       "compulsory bytes at the measured HBM rate",
                         "step_frac": t_step_roof / ms,
                         "mode_adjusted_estimate": {
                             "note": "each FLOP charged its precision mode's MMA cost in bf16-MMA equivalents: "
                                     "3 x bf16 = 3, bf16 = 1, tf32 = the measured bf16 / tf32 GEMM throughput "
                                     "ratio, 3 x tf32 = 3 x that ratio",
                             "tf32_tflops_measured": tf32, "bf16_over_tf32": tf_burst / tf32,
                             "kernel_frac": kd["t_mode_ms"] / kd["ms_per_launch"],
                             "step_frac": t_step_mode / ms}},
            "kernels": {n: {"ms": round(v["ms_per_launch"], 4), "share": round(v["share"], 3),
                            "bound": v["bound"], "roof_ms": round(v["t_roof_ms"], 4),
                            "frac": round(v["t_roof_ms"] / v["ms_per_launch"], 4),
                            "ncu_dram_bytes": traffic.get(n)} for n, v in kern.items()},
            "protocol": protocol,
            "weak": weak,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms,
                    "copies": "inputs q,k,v,w,b,g H2D; o, h_final, dq..dg D2H; loss read per step",
                    "pipeline": "the next two steps' H2D (three input buffers) and the previous step's D2H "
                                "overlapped with this step's compute; each step's loss read on the host two "
                                "steps later, inside the timed region",
                    "host_buffers": ("pinned, on the GPU's local CPUs (NVML affinity, %d CPUs)" % len(local_cpus))
                    if local_cpus else "pinned"},
            "gpu_launches": op_launches(nbh_local, L, cfg, torch.cuda.get_device_properties(dev).multi_processor_count)
            * args.steps,
            "clocks": clk,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    del graph
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------------------
# sweep (B4, H in {2,4,6}, L in {2048,4096}, fwd-only and fwd+bwd;
# config 4: B1 H6 L65536 as 16 segments of 4096 chunks with h carried, fwd+bwd)
# --------------------------------------------------------------------------------------
SWEEP = [(4, 2, 2048), (4, 4, 2048), (4, 6, 2048), (4, 2, 4096), (4, 4, 4096), (4, 6, 4096), (1, 6, 65536)]
# Published fwd+bwd latencies of the reference on TPU v5e-1 (README.md:26-31).
PUBLISHED_FWDBWD_MS = {(4, 2, 2048): 1.701, (4, 2, 4096): 2.943, (4, 4, 2048): 2.702, (4, 4, 4096): 10.493,
                       (4, 6, 2048): 2.888, (4, 6, 4096): 13.818}


def run_sweep(args):
    """One JSON line per (shape, pass).  Each timed step is bracketed by its own CUDA events and
    preceded by an L2 flush (a 256 MB write outside the events), so shapes whose inputs fit in the
    126 MB L2 are still timed from HBM."""
    import atomic_gdn2
    from atomic_gdn2 import make_blr_trainable, make_cfg

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dtype = torch.float32 if args.dtype == "fp32" else torch.bfloat16
    cfg = make_cfg(**CFG_KW)
    if args.dtype == "bf16":
        cfg = cfg.with_(dot_mode="default", solve_dot_mode="default", b3_dot_mode="default")
    fn = make_blr_trainable(cfg, D ** -0.5)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    steps, warmup = max(1, min(args.steps, 20)), max(3, args.warmup)
    for shape in SWEEP:
        nb, nh, nl = shape
        xs_base, h0 = make_inputs(7, dev, dtype, shape)
        for mode in ("fwd", "fwd+bwd"):
            if mode == "fwd":
                xs = xs_base

                def step():
                    o, hf = fn(*xs, h0)
                    return o
            else:
                xs = [t.detach().requires_grad_(True) for t in xs_base]

                def step():
                    o, hf = fn(*xs, h0)
                    return torch.autograd.grad((o * o).sum() + (hf * hf).sum(), xs)
            atomic_gdn2.set_checks(True)
            step()
            atomic_gdn2.set_checks(False)
            for _ in range(warmup):
                step()
            # the step as one CUDA graph, as the headline line times it (eager launches if capture
            # fails): the device time of the program, not the Python launch rate of small shapes
            run, timing = step, "eager launches"
            try:
                side = torch.cuda.Stream(device=dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    for _ in range(2):
                        step()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=side):
                        step()
                torch.cuda.current_stream(dev).wait_stream(side)
                for _ in range(warmup):
                    graph.replay()
                run, timing = graph.replay, "CUDA-graph replay of the whole step"
            except Exception as exc:  # pragma: no cover - reported; eager timing stands
                print(f"bench: CUDA graph capture unavailable for {shape} {mode} ({exc})", file=sys.stderr)
            times = []
            for _ in range(steps):
                flush.fill_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                run()
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            ms = statistics.median(times)
            run = graph = None
            pub = PUBLISHED_FWDBWD_MS.get(shape) if mode == "fwd+bwd" else None
            nchunk = nl // T
            segs = math.ceil(nchunk / cfg.max_chunks_per_call)
            line = {"sweep": True, "metric": f"GDN-2 {mode} tokens/s", "value": nb * nl / (ms / 1e3),
                    "unit": "tokens/s", "ms_per_step": ms, "ms_min": min(times), "steps": steps, "warmup": warmup,
                    "dtype": "f32" if dtype == torch.float32 else "bf16", "data": "synthetic",
                    "config": {"workload": f"B{nb} H{nh} L{nl} D{D}", "segments": segs,
                               "chunks_per_segment": min(nchunk, cfg.max_chunks_per_call),
                               "l2": "flushed before every timed step"},
                    "status": atomic_gdn2.last_status(), "timing": timing,
                    "tpu_v5e_published_ms": pub, "speedup_vs_published": (pub / ms) if pub else None}
            print(json.dumps(line), flush=True)
            del xs
        del xs_base, h0
        torch.cuda.empty_cache()


# --------------------------------------------------------------------------------------
# LM step: 8-layer GDN-2 LM, B8 L2048 per GPU, data parallel over NCCL
# --------------------------------------------------------------------------------------
LM_B, LM_L = 8, 2048
# The reference's published LM step (204.659 ms, TPU v5e-1, README.md:43) is for its notebook's
# 34,873,952-parameter model, not this layer.py model (39,121,152 parameters): no vs_baseline.
LM_PUBLISHED_MS_OTHER_MODEL = 204.659


def run_lm(args):
    import datetime
    import atomic_gdn2
    from atomic_gdn2 import _lib, make_cfg
    from atomic_gdn2.training import GDN2LM, TrainStep, lm_config, make_optimizer
    from atomic_gdn2.training.model import n_params

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # dense layers in TF32 on the tensor cores (fp32 storage and accumulation)
    torch.backends.cuda.matmul.allow_tf32 = True
    cfg = make_cfg()
    mc = lm_config()
    model = GDN2LM(cfg, **mc, seed=0).to(dev)
    net = model
    if dist is not None:
        from torch.nn.parallel import DistributedDataParallel as DDP
        net = DDP(model, device_ids=[local], gradient_as_bucket_view=True, bucket_cap_mb=32)
    opt = make_optimizer(model, 3e-4)
    step = TrainStep(net, opt, lr=3e-4, warmup=200, total=2000)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)

    def tokens():
        return torch.randint(0, mc["vocab"], (LM_B, LM_L), generator=gen, device=dev)

    status_gate(step, tokens(), dist, max_over_ranks)
    # the default a drop-in caller gets (no host synchronisation) on one rank; with several ranks
    # the words are read after the loops and reduced, so that no rank leaves a collective alone
    atomic_gdn2.set_checks("async" if dist is None else False)
    steps, warmup = max(1, min(args.steps, 20)), max(3, args.warmup)
    batches = [tokens() for _ in range(steps)]
    for _ in range(warmup):
        step(batches[0])
    clocks = Clocks(local)
    clocks.start()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        loss, gn, ok = step(batches[i])
    e1.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    ms = max_over_ranks(ms)
    # operator kernels inside one step, with each operator call's batch as one launch sequence so
    # that launches do not overlap and their durations add up (the timed steps overlap the batch
    # groups on their streams)
    groups = _lib.set_batch_groups(1)
    _lib.profile_enable(True)
    step(batches[0])
    torch.cuda.synchronize()
    prof = _lib.profile_collect()
    _lib.profile_enable(False)
    _lib.set_batch_groups(groups)
    # end to end: tokens from pinned host memory every step, loss read back every step
    host = [b.cpu().pin_memory() for b in batches]
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(steps):
        loss, gn, ok = step(host[i].to(dev, non_blocking=True))
        lv = loss.item()
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / steps)
    final_loss = float(loss)
    # the data-parallel gradient all-reduce on its own: one all-reduce of a buffer the size of all
    # gradients (the DDP buckets' total), timed on the device, max over ranks; set beside the
    # 1-GPU step time it tells how much of it the backward pass hides
    allreduce_ms = None
    if dist is not None:
        nbytes = sum(p_.numel() for p_ in model.parameters())
        buf = torch.ones(nbytes, device=dev)
        for _ in range(3):
            dist.all_reduce(buf)
        torch.cuda.synchronize()
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(10):
            dist.all_reduce(buf)
        a1.record()
        torch.cuda.synchronize()
        allreduce_ms = max_over_ranks(a0.elapsed_time(a1) / 10)
        del buf
    # every call since the gate: timed steps, profiled step and end-to-end steps, any rank
    status = int(max_over_ranks(float(atomic_gdn2.last_status())))
    if args.torch_profile:      # every rank steps (the DDP all-reduce is collective); rank 0 prints
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as tp:
            for i in range(2):
                step(batches[i])
            torch.cuda.synchronize()
        if rank == 0:
            print(tp.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=70),
                  file=sys.stderr, flush=True)
    if rank == 0:
        tok = world * LM_B * LM_L
        op_ms = {n: round(t, 3) for n, (t, c) in prof.items() if c}
        line = {
            "metric": "GDN-2 LM step ms (8 layers, 39.1M params, B8 L2048 per GPU)", "value": ms, "unit": "ms",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "tokens_per_s": tok / (ms / 1e3), "dtype": "f32", "data":
            "synthetic (uniform random byte tokens), random-init weights",
            "config": {"workload": "LM training step: fwd, bwd, DP all-reduce, clip 1.0, AdamW lr 3e-4",
                       "model": "atomic_gdn2 layer.py LM", "params": n_params(model), **mc,
                       "global_batch": LM_B * world, "seq_len": LM_L, "parallelism": f"dp{world} (NCCL DDP)",
                       "matmul": "tf32 tensor cores, fp32 storage", "operator_modes":
                       {k: cfg.__dict__[k] for k in ("dot_mode", "solve_dot_mode", "b3_dot_mode")},
                       "l2": "activations (~10 GB per step) exceed the 126 MB L2"},
            "operator_kernels_ms_per_step": op_ms,
            "operator_share": sum(op_ms.values()) / ms,  # of the timed (overlapped) step: an upper bound
            "e2e": {"value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": LM_B * LM_L * 8, "d2h_bytes_per_step": 4},
            "gpu_launches": (op_launches(LM_B * mc["n_heads"], LM_L, cfg,
                                         torch.cuda.get_device_properties(dev).multi_processor_count) + 2)
            * len(model.layers) * steps,
            "final_loss": final_loss,
            "published_other_model_ms": LM_PUBLISHED_MS_OTHER_MODEL,
            "grad_allreduce_alone_ms": allreduce_ms,
            "clocks": clk, "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    # Multi-rank runs keep NCCL off NVLink multicast (NVLS): a rank that dies while its memory is
    # bound to a multicast object raises NVLink faults on the other ranks' GPUs.  The operator's
    # only collectives are the timing barrier and scalar reductions; the LM's gradient all-reduce
    # runs over plain peer copies.
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    if args.workload == "lm":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference LM step needs JAX/optax "
                                  "(not installed); its CPU restatement is not timed at this size"}))
            return
        run_lm(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
