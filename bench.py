"""Benchmark of the routed-expert NVFP4 MoE layer on B200.

Headline workload (config 1: decode-shaped full layer): E=170 routed
experts, hidden d=4096, expert intermediate I=1280, top-8, T=64 tokens, NVFP4
weights (bf16 N(0, 0.02) quantised with per-tensor global amax/(448*6)),
bf16 N(0, 1) activations, uniform-random top-8 routing with softmax-
renormalised weights. Synthetic seeded data; the weights are random-init.

A "step" is one routed-expert layer forward over one batch of T tokens. Four
independent layers (4 x 1.5 GB) rotate across steps so consecutive steps
never find their weights in the 126 MB L2. The device-resident number replays
one captured CUDA graph per (layer, batch), as a serving engine replays its
decode step; the eager time of the same calls is reported beside it, and the
end-to-end number goes through the public op with host buffers.

Timing: every K-step loop is bracketed by synchronize + barrier +
synchronize, and starts with one untimed step whose cross-GPU waits (expert
parallel) line the ranks up on the device, so the first event records after
every rank has arrived; the loop is repeated enough times to cover about a
second of device time with nvidia-smi clock samples (the sampler is started
before the first barrier), the per-rank median is taken, then the maximum
over ranks.

With one GPU the default run also measures, in the same process, the other
single-GPU workloads of the benchmark configurations (T = 1, 8, 32 decode;
T = 8192 prefill; T = 4096 Zipf routing, W4A16 and W4A4), each under
"workloads" with its own roofline. With N > 1 GPUs it runs expert
parallelism (170 experts sharded, the T tokens split over the ranks, strong
scaling) and checks the step's output against this library's single-GPU
path on the full layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T]
    python bench.py --impl reference ...   # the reference's CPU expert tier

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

E, D, I, TOP_K = 170, 4096, 1280, 8
EXPERT_BYTES = 2 * I * D // 2 + 2 * I * D // 16 + D * I // 2 + D * I // 16 + 8
W13_EXPERT_BYTES = 2 * I * D // 2 + 2 * I * D // 16 + 4
W2_EXPERT_BYTES = D * I // 2 + D * I // 16 + 4
METRIC = "routed-expert tokens/s"
W4A16_DTYPE = ("nvfp4 W4A16: e2m1 weights x e2m1 activation terms (4 interleaved terms at decode "
               "sizes, 3 term planes along K at prefill sizes), mxf4nvf4 MMA, fp32 accumulate")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--eager", action="store_true",
                    help="time eager calls instead of CUDA-graph replay")
    ap.add_argument("--routing", default=None, choices=["uniform", "biased", "zipf"],
                    help="routing (default: uniform for decode sizes, biased from 1024 tokens)")
    ap.add_argument("--w4a4", action="store_true",
                    help="quantise activations once (W4A4, dynamic per-row globals)")
    ap.add_argument("--stack", type=int, default=0,
                    help="run a stack of this many layers per step (config 3: 46 layers)")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1, run N independent single-GPU replicas instead of "
                         "expert parallelism")
    ap.add_argument("--layers", type=int, default=4,
                    help="independent layers rotated across steps (>= 2 keeps weights out of L2)")
    ap.add_argument("--no-stack-extras", dest="stack_extras", action="store_false",
                    help="skip the config-3 46-layer stack in the default one-GPU run")
    ap.add_argument("--no-extras", action="store_true",
                    help="single GPU: measure the headline workload only")
    ap.add_argument("--min-timed-s", type=float, default=1.0,
                    help="device seconds the repeated K-step loops of the headline cover")
    return ap.parse_args()


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------

def dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_over_ranks(v: float, world: int, op: str = "max") -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def max_over_ranks(v: float, world: int) -> float:
    return reduce_over_ranks(v, world, "max")


# --------------------------------------------------------------------------
# synthetic inputs
# --------------------------------------------------------------------------

def quantize_plane_torch(w, G):
    """NVFP4 quantisation of a [rows, cols] plane with plain torch ops (vLLM
    ref_nvfp4_quant semantics); G is a scalar or a [rows, 1] column of
    per-row quantisation globals. Data generation shared by both bench arms,
    so they see identical bytes; the library's own quantiser is not used."""
    import torch
    rows, cols = w.shape
    x = w.float().reshape(rows, cols // 16, 16)
    if isinstance(G, torch.Tensor) and G.dim() == 2:
        G = G[:, :, None]
    vmax = x.abs().amax(dim=-1, keepdim=True)
    scale = (G * (vmax * (1.0 / 6.0))).clamp(-448.0, 448.0)
    sf = scale.to(torch.float8_e4m3fn)
    sq = sf.float()
    inv_g = 1.0 / (G + (G == 0).float() * 1e8)
    t = sq * inv_g
    out_scale = 1.0 / (t + (t == 0).float() * 1e8)
    y = (x * out_scale).clamp(-6.0, 6.0)
    a = y.abs()
    mag = torch.zeros_like(a, dtype=torch.uint8)
    for code, lo, lo_incl, hi, hi_incl in ((1, 0.25, False, 0.75, False), (2, 0.75, True, 1.25, True),
                                           (3, 1.25, False, 1.75, False), (4, 1.75, True, 2.5, True),
                                           (5, 2.5, False, 3.5, False), (6, 3.5, True, 5.0, True)):
        m = ((a >= lo) if lo_incl else (a > lo)) & ((a <= hi) if hi_incl else (a < hi))
        mag = torch.where(m, torch.full_like(mag, code), mag)
    mag = torch.where(a > 5.0, torch.full_like(mag, 7), mag)
    code = mag | (((y < 0) & (mag != 0)).to(torch.uint8) << 3)
    code = code.reshape(rows, cols)
    q = code[:, 0::2] | (code[:, 1::2] << 4)
    return q.contiguous(), sf.view(torch.uint8).reshape(rows, cols // 16).contiguous()


def make_layers(device, n_layers, seed=0):
    """n_layers independent 170-expert NVFP4 layers: bf16 N(0, 0.02) planes,
    per-plane quantisation global G = 448*6/amax, stored global amax/(448*6)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        w13 = torch.empty((E, 2 * I, D // 2), dtype=torch.uint8, device=device)
        s13 = torch.empty((E, 2 * I, D // 16), dtype=torch.uint8, device=device)
        w2 = torch.empty((E, D, I // 2), dtype=torch.uint8, device=device)
        s2 = torch.empty((E, D, I // 16), dtype=torch.uint8, device=device)
        g13 = torch.empty(E, dtype=torch.float32, device=device)
        g2 = torch.empty(E, dtype=torch.float32, device=device)
        chunk = 16  # experts generated and quantised per batch of torch ops
        for e0 in range(0, E, chunk):
            e1 = min(E, e0 + chunk)
            for (q, sf, g, shape) in ((w13, s13, g13, (2 * I, D)), (w2, s2, g2, (D, I))):
                w = (torch.randn((e1 - e0,) + shape, generator=gen, device=device) * 0.02).to(
                    torch.bfloat16)
                amax = w.float().abs().amax(dim=(1, 2))
                G = torch.tensor(2688.0, device=device) / amax
                g[e0:e1] = amax / 2688.0
                qe, se = quantize_plane_torch(w.reshape(-1, shape[1]),
                                              G.repeat_interleave(shape[0])[:, None])
                q[e0:e1].copy_(qe.reshape(e1 - e0, shape[0], -1))
                sf[e0:e1].copy_(se.reshape(e1 - e0, shape[0], -1))
                del w
        layers.append((w13, s13, g13, w2, s2, g2))
    return layers


def layer_to_host(tensors):
    from oracle import nvfp4 as O
    w13, s13, g13, w2, s2, g2 = (t.cpu().numpy() for t in tensors)
    return O.Layer(E, D, I, w13, s13, g13, w2, s2, g2)


def make_batch(device, T, seed, routing="uniform"):
    """bf16 N(0,1) hidden [T, d] and top-8 routing with softmax-renormalised
    weights: "uniform" (top-8 of N(0,1) logits, config 1), "biased" (logits
    N(0,1) plus a per-expert bias N(0,0.5): mildly uneven loads, config 2) or
    "zipf" (8 distinct experts drawn with probability rank^-1.2 over a seeded
    permutation, weights a softmax of N(0,1) logits: config 4)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    hidden = torch.randn((T, D), generator=gen, device=device).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=device)
    if routing == "biased":
        bgen = torch.Generator(device=device)
        bgen.manual_seed(7)  # one bias vector per layer stack
        logits = logits + torch.randn(E, generator=bgen, device=device) * 0.5
    if routing == "zipf":
        pgen = torch.Generator(device=device)
        pgen.manual_seed(11)
        perm = torch.randperm(E, generator=pgen, device=device)
        p = 1.0 / torch.arange(1, E + 1, device=device, dtype=torch.float64) ** 1.2
        pick = torch.multinomial((p / p.sum()).float().expand(T, E), TOP_K, replacement=False,
                                 generator=gen)
        ids = perm[pick]
        w = torch.softmax(torch.randn((T, TOP_K), generator=gen, device=device), dim=1)
        return hidden, ids.to(torch.int32).contiguous(), w.float().contiguous()
    vals, ids = torch.topk(logits, TOP_K, dim=1)
    w = torch.softmax(vals, dim=1)
    return hidden, ids.to(torch.int32).contiguous(), w.float().contiguous()


def algorithmic_bytes(ids_cpu, T):
    """Algorithmic bytes of one layer forward: every distinct routed expert's
    packed weights, scales and globals once, bf16 activations in, ids and
    weights, bf16-sized output."""
    import numpy as np
    distinct = len(np.unique(ids_cpu[ids_cpu >= 0]))
    return distinct * EXPERT_BYTES + T * D * 2 + T * TOP_K * 8 + T * D * 2, distinct


def default_routing(T):
    return "uniform" if T < 1024 else "biased"


def workload_name(T, routing, w4a4):
    """The config name both arms print for a single-layer workload."""
    if T >= 4096 and routing == "zipf":
        kind = "config4-skewed-w4a4" if w4a4 else "config4-skewed-w4a16"
    elif T <= 64:
        kind = "config1-decode"
    elif T >= 8192:
        kind = "config2-prefill"
    else:
        kind = "layer"
    if w4a4 and not kind.endswith("w4a4"):
        kind += "-w4a4"
    return f"{kind} E={E} d={D} I={I} top{TOP_K} T={T} routing={routing}"


def single_config(T, routing, w4a4):
    """`config` of a single-GPU line; the reference arm prints the same dict."""
    return {"workload": workload_name(T, routing, w4a4), "global_batch": T,
            "parallelism": "single", "l2": "inputs larger than L2 (rotating 1.5 GB layers)"}


def load_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


# --------------------------------------------------------------------------
# clocks
# --------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        """Start nvidia-smi and block until it has printed its first line, so
        the samples that follow cover what runs next."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        import select
        r, _, _ = select.select([self.proc.stdout], [], [], 3.0)
        if r:
            self.proc.stdout.readline()
        return self

    def stop(self):
        if self.proc is not None:
            # a region shorter than the 50 ms period may have no sample yet:
            # take the one that follows it rather than none
            import select
            select.select([self.proc.stdout], [], [], 0.5)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
            self.proc = None

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------
# timing
# --------------------------------------------------------------------------

class StepTimer:
    """Device time per step of K-step loops on one stream.

    Each loop: synchronize, barrier, synchronize; one untimed step (in the
    expert-parallel step its cross-GPU waits hold every rank until all have
    arrived, so the ranks start the timed steps together on the device);
    event; K steps; event. Loops are repeated, the per-rank median kept and
    the maximum over ranks reported. Every rank runs the same number of
    loops (the count is agreed over the ranks first)."""

    def __init__(self, stream, world):
        self.stream = stream
        self.world = world

    def loop_ms(self, run_one, steps, finish=None):
        import torch
        torch.cuda.synchronize()
        barrier(self.world)
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        run_one(0)
        ev0.record(self.stream)
        for i in range(steps):
            run_one(i + 1)
        if finish is not None:  # work on other streams the steps left in flight
            finish()
        ev1.record(self.stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / steps

    def repeats_for(self, est_ms, steps, seconds, lo=3, hi=200):
        n = math.ceil(seconds * 1e3 / max(est_ms * steps, 1e-3)) if seconds > 0 else lo
        return int(max_over_ranks(float(min(hi, max(lo, n))), self.world))

    def run(self, run_one, steps, repeats, finish=None):
        per = [self.loop_ms(run_one, steps, finish) for _ in range(repeats)]
        med = statistics.median(per)
        return max_over_ranks(med, self.world), {"repeats": repeats, "min_ms": min(per),
                                                 "max_ms": max(per)}


class CopyPipeline:
    """End-to-end steps as a serving loop runs them: step i's inputs go up
    from pinned host memory on one copy stream while step i-1's kernels run,
    and its result comes back to pinned host memory on a second copy stream
    while step i+1's kernels run. Device inputs are double-buffered (a buffer
    is refilled once the step that read it has finished). Every step's bytes
    still cross PCIe; `finish` makes the compute stream wait for the last
    read-back, so a timed region closed after it contains it.

    host_in: list of tuples of pinned tensors (one tuple per step, cycled);
    compute(i, device_inputs) -> the step's device result (bf16, out_shape)."""

    DESCRIPTION = ("per step: inputs copied up from pinned host memory on one copy stream while "
                   "the previous step's kernels run, result copied back to pinned host memory on "
                   "a second copy stream while the next step's run (double-buffered device "
                   "inputs); the timed region ends after the last read-back")

    def __init__(self, device, host_in, out_shape, compute):
        import torch
        self.comp = torch.cuda.current_stream(device)
        self.cs_in = torch.cuda.Stream(device)
        self.cs_out = torch.cuda.Stream(device)
        self.host_in = host_in
        self.dev = [tuple(torch.empty(x.shape, dtype=x.dtype, device=device) for x in host_in[0])
                    for _ in range(2)]
        self.ready = [torch.cuda.Event() for _ in range(2)]
        self.free = [None, None]
        self.host_out = torch.empty(out_shape, dtype=torch.bfloat16).pin_memory()
        self.compute = compute
        self.last = None

    def step(self, i):
        import torch
        b = i % 2
        dev = self.dev[b]
        with torch.cuda.stream(self.cs_in):
            if self.free[b] is not None:
                self.cs_in.wait_event(self.free[b])
            for d, h in zip(dev, self.host_in[i % len(self.host_in)]):
                d.copy_(h, non_blocking=True)
            self.ready[b].record(self.cs_in)
        self.comp.wait_event(self.ready[b])
        o = self.compute(i, dev)
        done = torch.cuda.Event()
        done.record(self.comp)
        self.free[b] = done
        with torch.cuda.stream(self.cs_out):
            self.cs_out.wait_event(done)
            self.host_out.copy_(o, non_blocking=True)
            o.record_stream(self.cs_out)
            back = torch.cuda.Event()
            back.record(self.cs_out)
        self.last = back

    def finish(self):
        if self.last is not None:
            self.comp.wait_event(self.last)

    def bytes_per_step(self):
        up = sum(x.numel() * x.element_size() for x in self.host_in[0])
        return up, self.host_out.numel() * self.host_out.element_size()


# --------------------------------------------------------------------------
# CPU baselines (reference CPU expert tier, compiled from its source)
# --------------------------------------------------------------------------

def cpu_reference_run(layer_host, hidden_bits, ids, w, seconds, max_calls=500, warmup=1):
    """Time the reference's CPU expert tier (sb_cpu_moe_forward, compiled from
    its source) on one 170-expert layer of the headline workload with all host
    threads: `warmup` untimed calls, then whole-batch calls until `seconds`
    have passed or `max_calls` were timed (at least one). Returns (tokens/s,
    sample description, threads, seconds/call, calls timed)."""
    from oracle import nvfp4 as O
    threads = os.cpu_count() or 1
    T = hidden_bits.shape[0]
    tier = O.ReferenceCpuTier(layer_host, threads=threads)
    for _ in range(max(1, warmup)):  # the first call also touches the arena
        tier.forward(hidden_bits, ids, w)
    times = []
    t_end = time.perf_counter() + seconds
    while (time.perf_counter() < t_end or not times) and len(times) < max(1, max_calls):
        t0 = time.perf_counter()
        tier.forward(hidden_bits, ids, w)
        times.append(time.perf_counter() - t0)
    tier.close()
    per_call = sum(times) / len(times)
    return T / per_call, (f"mean of {len(times)} timed sb_cpu_moe_forward calls (whole T={T} "
                          f"batch each) on one 170-expert layer"), threads, per_call, len(times)


def cpu_isa():
    try:
        from oracle import nvfp4 as O
        return O.reference_isa()
    except Exception:
        return None


def profiled_traffic(T):
    """dram__bytes_read.sum + dram__bytes_write.sum of one gate/up launch,
    from the committed ncu summary of this workload, or None."""
    import re
    f = ROOT / "profiles" / f"moe_gemm_bs_gateup_decode_T{T}.md"
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", f.read_text())
    except OSError:
        return None
    return int(m.group(1)) if m else None


def host_batch(batch):
    """(bf16 bits, ids, weights) numpy copies of a device batch."""
    import torch
    h, ids, w = batch
    return (h.view(torch.int16).cpu().numpy().view("uint16"), ids.cpu().numpy(),
            w.cpu().numpy())


# --------------------------------------------------------------------------
# reference arm
# --------------------------------------------------------------------------

def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from oracle import nvfp4 as O
    if not O.reference_available():
        try:
            O.build(ref=True)
        except Exception:
            pass
    if not O.reference_available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference CPU expert tier library not built (oracle/_ref absent)"}))
        return
    T = args.tokens
    device = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    # the same seeded layer 0 and batch 0 as the B200 arm
    layer_host = layer_to_host(make_layers(device, 1, seed=1000)[0])
    routing = args.routing or default_routing(T)
    hb, ids, w = host_batch(make_batch(device, T, seed=2000, routing=routing))
    # K timed whole-batch calls after W warm-up calls, bounded to a few
    # minutes of host time (the step count actually timed is reported).
    tps, sample, threads, per_call, n = cpu_reference_run(
        layer_host, hb, ids, w, seconds=150.0, max_calls=args.steps, warmup=args.warmup)
    world = args.gpus
    config = (single_config(T, routing, args.w4a4) if world == 1 or args.replicas else
              ep_config(T, routing, args.w4a4, world))
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": per_call * 1e3, "higher_is_better": True,
        "scaling": "weak" if world == 1 or args.replicas else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads,
                         "kind": "reference", "sample": sample, "isa": cpu_isa()},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if world > 1:
        line["note"] = ("the reference CPU expert tier on this host's cores runs the whole "
                        "global batch through all 170 experts")
    if args.w4a4:
        line["note"] = ("the reference CPU expert tier keeps activations in f32 (it has no "
                        "activation quantisation); it is timed on the same layer and routes")
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# expert parallel
# --------------------------------------------------------------------------

def ep_config(T, routing, w4a4, world):
    return {"workload": workload_name(T, routing, w4a4) + f", experts sharded over {world} GPUs",
            "global_batch": T, "parallelism": f"ep{world}",
            "l2": "inputs larger than L2 (rotating 1.5 GB layers, sharded)"}


def run_expert_parallel(args, sbb, rank, world, local):
    """Expert parallelism over NVLink, strong scaling: the global batch of T
    tokens (config 1) is split evenly over the ranks, the 170 experts are
    sharded contiguously, and every step runs one sbb200_ep_forward per rank.
    `value` = T / (max over ranks of the per-step time). The output of one
    step is checked against this library's single-GPU forward of the full
    layer on the same tokens (itself checked against the CPU oracle by the
    GPU tests)."""
    import importlib

    import torch
    ep_mod = importlib.import_module(sbb.__name__ + ".ep")
    device = torch.device("cuda", local)
    T = args.tokens
    if T % world:
        raise SystemExit(f"--tokens {T} must divide evenly over {world} ranks")
    Tr = T // world
    N_LAYERS = args.layers
    ep = ep_mod.ExpertParallel(rank=rank, world=world, device=local, max_tokens=Tr, top_k=TOP_K,
                               E=E, K=D, I=I, w4a4=args.w4a4)
    routing = args.routing or default_routing(T)
    layers, full0 = [], None
    for li, lw in enumerate(make_layers(device, N_LAYERS, seed=1000)):
        layers.append(tuple(ep.local_experts(t).contiguous() for t in lw))
        if li == 0:
            full0 = lw  # kept for the single-GPU parity check
        del lw
    torch.cuda.empty_cache()
    gbatches = [make_batch(device, T, seed=2000 + 17 * i, routing=routing)
                for i in range(N_LAYERS)]
    batches = [tuple(x[rank * Tr:(rank + 1) * Tr].contiguous() for x in b) for b in gbatches]
    out = torch.empty((Tr, D), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    timer = StepTimer(stream, world)

    def step(i):
        h, ids, w = batches[i % N_LAYERS]
        ep.forward(h, ids, w, *layers[i % N_LAYERS], out=out)

    for i in range(max(args.warmup, 3)):
        step(i)
    est = timer.loop_ms(step, max(args.warmup, 3))
    graphs = []
    clk = ClockSampler(local)
    if not args.eager:
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        torch.cuda.synchronize()
        for i in range(N_LAYERS):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap):
                step(i)
            graphs.append(gr)
        torch.cuda.synchronize()
        barrier(world)
        for i in range(max(args.warmup, 3)):
            graphs[i % N_LAYERS].replay()
        replay = lambda i: graphs[i % N_LAYERS].replay()  # noqa: E731
        repeats = timer.repeats_for(est, args.steps, args.min_timed_s)
        clk.start()
        ms, spread = timer.run(replay, args.steps, repeats)
        clk.stop()
        eager_ms, _ = timer.run(step, args.steps, 3)
    else:
        repeats = timer.repeats_for(est, args.steps, args.min_timed_s)
        clk.start()
        ms, spread = timer.run(step, args.steps, repeats)
        clk.stop()
        eager_ms = ms
    clocks = clk.summary()

    # end to end: this rank's tokens from pinned host memory, result back
    host_in = [(h.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory())
               for (h, ids, w) in batches]
    pipe = CopyPipeline(device, host_in, (Tr, D),
                        lambda i, x: ep.forward(*x, *layers[i % N_LAYERS],
                                                out_dtype=torch.bfloat16))
    for i in range(max(args.warmup, 3)):
        pipe.step(i)
    e2e_ms, _ = timer.run(pipe.step, args.steps, 3, finish=pipe.finish)
    errors = ep.device_errors() | sbb.device_errors(device)

    # parity: one eager step (layer 0, batch 0) against the single-GPU path
    # on the full layer and this rank's tokens; every rank takes part
    h0, ids0, w0 = batches[0]
    got = ep.forward(h0, ids0, w0, *layers[0], out_dtype=torch.float32)
    if args.w4a4:
        want = sbb.nvfp4_moe_w4a4(h0, ids0, w0, *full0, out_dtype=torch.float32)
    else:
        want = sbb._nvfp4_moe_impl(h0, ids0, w0, *full0, True, torch.float32)
    torch.cuda.synchronize()
    errors |= ep.device_errors() | sbb.device_errors(device)
    diff = float((got.double() - want.double()).abs().max())
    scale = float(want.double().abs().max())
    cos = float(torch.nn.functional.cosine_similarity(got.double().flatten(),
                                                      want.double().flatten(), dim=0))
    max_rel = reduce_over_ranks(diff / max(scale, 1e-30), world, "max")
    min_cos = reduce_over_ranks(cos, world, "min")
    all_errors = int(reduce_over_ranks(float(errors), world, "max"))
    del full0

    ids_all = [b[1].cpu().numpy() for b in gbatches]
    byts = [algorithmic_bytes(x, T) for x in ids_all]
    avg_bytes = sum(b for b, _ in byts) / len(byts)
    avg_distinct = sum(d for _, d in byts) / len(byts)
    peaks = load_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    per_gpu = avg_bytes / world / (ms * 1e-3) / 1e9
    # routes each rank's shard serves per step (load imbalance across ranks)
    shard_routes = []
    for r in range(world):
        b, c = ep_mod.expert_shard(E, world, r)
        shard_routes.append(sum(int(((x >= b) & (x < b + c)).sum()) for x in ids_all) / len(ids_all))
    mean_routes = sum(shard_routes) / world
    launches = ep.kernels_per_step()
    del graphs
    valid = all_errors == 0 and max_rel <= 1e-2 and min_cos >= 0.9999
    # the other multi-GPU workloads of the configurations, once the headline
    # step is known good on every rank
    workloads = None
    if valid and not args.no_extras and not args.w4a4 and T == 64:
        layers.clear()
        torch.cuda.empty_cache()
        try:  # the headline line is printed whatever happens to the extras
            workloads = ep_extras(args, sbb, ep_mod, rank, world, local)
        except Exception as exc:
            workloads = {"error": f"{type(exc).__name__}: {str(exc)[:160]}"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": T / (ms * 1e-3) if valid else None, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("nvfp4 W4A4: e2m1 weights x e2m1 activations (dynamic per-row globals), "
                      "mxf4nvf4 MMA, fp32 accumulate") if args.w4a4 else
                     W4A16_DTYPE,
            "data": "synthetic",
            "config": ep_config(T, routing, args.w4a4, world),
            "tokens_per_gpu": Tr,
            "exchange": "NVLink peer loads/stores (CUDA IPC), no NCCL on the data path",
            "distinct_experts_avg": avg_distinct, "algorithmic_bytes_per_step": avg_bytes,
            "timing": ("CUDA graph replay" if not args.eager else "eager calls")
                      + f"; median of {spread['repeats']} loops of {args.steps} steps, each after "
                        "one untimed step that lines the ranks up on the device; max over ranks",
            "loop_spread_ms": spread,
            "eager_ms_per_step": eager_ms,
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": hbm_peak, "unit": "GB/s",
                         "frac": per_gpu / hbm_peak, "traffic": None,
                         "kernel": "whole expert-parallel step per GPU (weight stream of the "
                                   "shard + exchange)",
                         "peak_source": f"{peak_src} hbm_gbs"},
            "cpu_baseline": None,
            "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": Tr * D * 2 + Tr * TOP_K * 8,
                    "d2h_bytes_per_step": Tr * D * 2, "ms_per_step": e2e_ms,
                    "copies": CopyPipeline.DESCRIPTION},
            "gpu_launches": launches * args.steps,
            "load_imbalance": {"routes_per_rank": shard_routes,
                               "max_over_mean": max(shard_routes) / mean_routes if mean_routes else None},
            "parity": {"vs": "this library's single-GPU forward of the full layer on the same "
                             "tokens (fp32 out), layer 0 batch 0, every rank",
                       "max_rel": max_rel, "cos": min_cos, "bar": "max_rel <= 1e-2, cos >= 0.9999"},
            "device_errors": all_errors,
            "clocks": clocks,
            "workloads": workloads,
        }
        if not valid:
            line["invalid"] = "device error bits set or parity outside the bar; no value reported"
        print(json.dumps(line), flush=True)
    ep.close()
    import torch.distributed as dist
    dist.barrier()
    dist.destroy_process_group()


def ep_extras(args, sbb, ep_mod, rank, world, local):
    """The expert-parallel runs of configurations 4 and 3 at this world size:
    the Zipf-routed 4,096-token layer (W4A16 and W4A4) with its per-rank
    load-imbalance tail, then the 46-layer stack at decode T=64 and prefill
    T=32,768. Each is a fixed sequence of collective steps on every rank;
    the first one that fails on any rank (agreed over the ranks) ends the
    list. Returns {workload: result} (rank 0; None elsewhere)."""
    import torch
    device = torch.device("cuda", local)
    stream = torch.cuda.current_stream(device)
    timer = StepTimer(stream, world)
    peaks = load_peaks()
    tf_peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    out = {}

    def agreed(ok: bool) -> bool:
        return reduce_over_ranks(1.0 if ok else 0.0, world, "min") > 0.5

    # config 4: Zipf(1.2) routing, 4,096 tokens split over the ranks
    try:
        Tz = 4096
        Tzr = Tz // world
        zl = []
        for lw in make_layers(device, 2, seed=1000):
            zl.append(lw)
        ok = True
        for w4 in (False, True):
            epz = ep_mod.ExpertParallel(rank=rank, world=world, device=local, max_tokens=Tzr,
                                        top_k=TOP_K, E=E, K=D, I=I, w4a4=w4)
            lay = [tuple(epz.local_experts(t).contiguous() for t in lw) for lw in zl]
            gb = [make_batch(device, Tz, seed=3000 + Tz + 17 * i, routing="zipf")
                  for i in range(len(lay))]
            bat = [tuple(x[rank * Tzr:(rank + 1) * Tzr].contiguous() for x in b) for b in gb]
            o = torch.empty((Tzr, D), dtype=torch.bfloat16, device=device)

            def zstep(i):
                h, ids, w = bat[i % len(bat)]
                epz.forward(h, ids, w, *lay[i % len(lay)], out=o)

            for i in range(3):
                zstep(i)
            ms, spread = timer.run(zstep, args.steps, 3)
            err = int(reduce_over_ranks(float(epz.device_errors() | sbb.device_errors(device)),
                                        world, "max"))
            ids_all = [b[1].cpu().numpy() for b in gb]
            per_rank = []
            for r in range(world):
                b0, c = ep_mod.expert_shard(E, world, r)
                per_rank.append(sum(int(((x >= b0) & (x < b0 + c)).sum()) for x in ids_all)
                                / len(ids_all))
            mean_r = sum(per_rank) / world
            routes = sum(int((x >= 0).sum()) for x in ids_all) / len(ids_all)
            tfl = 2.0 * routes * 3 * I * D / world / (ms * 1e-3) / 1e12
            peak = tf_peak * (4.0 if w4 else 1.0)
            out[workload_name(Tz, "zipf", w4) + f", experts sharded over {world} GPUs"] = {
                "value": Tz / (ms * 1e-3) if err == 0 else None, "unit": "tokens/s",
                "ms_per_step": ms, "steps": args.steps, "timing": "eager calls, max over ranks",
                "loop_spread_ms": spread,
                "load_imbalance": {"routes_per_rank": per_rank,
                                   "max_over_mean": max(per_rank) / mean_r if mean_r else None},
                "roofline": {"bound": "tensor", "achieved": tfl, "peak": peak,
                             "unit": "TFLOP/s", "frac": tfl / peak,
                             "kernel": "whole expert-parallel step per GPU",
                             "peak_source": "measured bf16_tflops_sustained" +
                                            (" x4 (FP4 rate)" if w4 else "")},
                "device_errors": err}
            epz.close()
            del lay, bat, gb, o
            torch.cuda.empty_cache()
            ok = ok and err == 0
        del zl
        torch.cuda.empty_cache()
    except Exception as exc:  # recorded, and the stack below is skipped
        out["error"] = f"config 4: {type(exc).__name__}: {str(exc)[:160]}"
        ok = False
    if not agreed(ok):
        return out if rank == 0 else None

    # config 3: the 46-layer stack, sharded
    try:
        ep_dec = ep_mod.ExpertParallel(rank=rank, world=world, device=local,
                                       max_tokens=64 // world, top_k=TOP_K, E=E, K=D, I=I)
        st = stack_layers(device, 46, ep_dec)
        for t, steps, e in ((64, args.steps, ep_dec), (32768, 3, None)):
            if e is None:
                e = ep_mod.ExpertParallel(rank=rank, world=world, device=local,
                                          max_tokens=t // world, top_k=TOP_K, E=E, K=D, I=I)
            sl = measure_stack(args, sbb, rank, world, local, t, st, e, steps, 3)
            if rank == 0:
                out[sl["config"]["workload"]] = {
                    k: sl[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup",
                                       "ms_per_layer", "roofline", "e2e", "clocks",
                                       "gpu_launches", "device_errors", "weights_gb")}
            e.close()
            torch.cuda.empty_cache()
        del st
        torch.cuda.empty_cache()
        ok = True
    except Exception as exc:
        out["error"] = f"config 3: {type(exc).__name__}: {str(exc)[:160]}"
        ok = False
    agreed(ok)
    return out if rank == 0 else None


# --------------------------------------------------------------------------
# config 3: layer stack
# --------------------------------------------------------------------------

def run_stack(args, sbb, rank, world, local):
    """Config 3: a stack of args.stack routed-expert layers (46 ->
    69.2 GB of NVFP4 weights, independent seeded layers) run back to back per
    step on T tokens (the attention blocks between the MoE layers are outside
    this path, so every layer reads the same hidden rows), routing per layer
    from its own seeded logits. One GPU holds every layer; with N GPUs each
    layer's experts are sharded (expert parallel, strong scaling: the T
    tokens split over the ranks). value = T / step time; one CUDA graph per
    step holds all layers."""
    import importlib

    import torch
    device = torch.device("cuda", local)
    T = args.tokens
    if T % world:
        raise SystemExit(f"--tokens {T} must divide evenly over {world} ranks")
    ep = None
    if world > 1:
        ep_mod = importlib.import_module(sbb.__name__ + ".ep")
        ep = ep_mod.ExpertParallel(rank=rank, world=world, device=local, max_tokens=T // world,
                                   top_k=TOP_K, E=E, K=D, I=I, w4a4=args.w4a4)
    layers = stack_layers(device, args.stack, ep)
    line = measure_stack(args, sbb, rank, world, local, T, layers, ep, args.steps, args.warmup)
    if ep is not None:
        ep.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def stack_layers(device, Ls, ep=None):
    """The Ls independent seeded layers of config 3 (this rank's expert shard
    of each when expert parallel)."""
    import torch
    layers = []
    for l in range(Ls):
        lw = make_layers(device, 1, seed=5000 + l)[0]
        layers.append(tuple(ep.local_experts(t).contiguous() for t in lw) if ep else lw)
        del lw
    torch.cuda.empty_cache()
    return layers


def measure_stack(args, sbb, rank, world, local, T, layers, ep, steps, warmup):
    """One config-3 measurement: every layer of `layers` per step on T
    tokens. Returns the bench line (rank 0's values)."""
    import torch
    device = torch.device("cuda", local)
    Ls = len(layers)
    Tr = T // world
    routing = args.routing or default_routing(T)
    routes, gids = [], []
    for l in range(Ls):
        h, ids, w = make_batch(device, T, seed=7000 + l, routing=routing)
        gids.append(ids.cpu().numpy())
        routes.append((ids[rank * Tr:(rank + 1) * Tr].contiguous(),
                       w[rank * Tr:(rank + 1) * Tr].contiguous()))
        if l == 0:
            hidden = h[rank * Tr:(rank + 1) * Tr].contiguous()
    out = torch.empty((Tr, D), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    timer = StepTimer(stream, world)

    def layer(l, x, o):
        ids, w = routes[l]
        if ep is not None:
            return ep.forward(x, ids, w, *layers[l], out=o)
        if args.w4a4:
            return sbb.nvfp4_moe_w4a4(x, ids, w, *layers[l], out=o)
        return sbb._nvfp4_moe_impl(x, ids, w, *layers[l], True, torch.bfloat16, out=o)

    def stack_step(_i=0):
        for l in range(Ls):
            layer(l, hidden, out)

    for _ in range(max(warmup, 3)):
        stack_step()
    torch.cuda.synchronize()
    barrier(world)
    graph = None
    if not args.eager:
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            stack_step()  # the capture stream's workspace exists before capture
        torch.cuda.synchronize()
        barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            stack_step()
        torch.cuda.synchronize()
        barrier(world)
        graph.replay()
    run = (lambda _i: graph.replay()) if graph is not None else stack_step
    est = timer.loop_ms(run, 1)
    repeats = timer.repeats_for(est, steps, 0.0, lo=3, hi=3)
    clk = ClockSampler(local).start()
    ms, spread = timer.run(run, steps, repeats)
    clk.stop()

    # end to end: this rank's hidden rows and every layer's routing in from
    # pinned host memory, the last layer's output back
    host_h = hidden.cpu().pin_memory()
    host_r = [(i.cpu().pin_memory(), w.cpu().pin_memory()) for i, w in routes]
    host_out = torch.empty((Tr, D), dtype=torch.bfloat16).pin_memory()
    dh = torch.empty_like(hidden)
    dr = [(torch.empty_like(i), torch.empty_like(w)) for i, w in routes]

    def e2e_step(_i=0):
        dh.copy_(host_h, non_blocking=True)
        for (di, dw), (hi, hw) in zip(dr, host_r):
            di.copy_(hi, non_blocking=True)
            dw.copy_(hw, non_blocking=True)
        for l in range(Ls):
            ids, w = dr[l]
            if ep is not None:
                o = ep.forward(dh, ids, w, *layers[l], out_dtype=torch.bfloat16)
            elif args.w4a4:
                o = sbb.nvfp4_moe_w4a4(dh, ids, w, *layers[l], out_dtype=torch.bfloat16)
            else:
                o = sbb.nvfp4_moe(dh, ids, w, *layers[l], out_dtype=torch.bfloat16)
        host_out.copy_(o, non_blocking=True)

    e2e_step()
    n_e2e = max(1, steps // 2)
    e2e_ms, _ = timer.run(e2e_step, n_e2e, 1)
    errors = (ep.device_errors() if ep is not None else 0) | sbb.device_errors(device)
    errors = int(reduce_over_ranks(float(errors), world, "max"))

    peaks = load_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    byts = sum(algorithmic_bytes(g, T)[0] for g in gids)
    per_gpu_gbs = byts / world / (ms * 1e-3) / 1e9
    fl = 2.0 * T * TOP_K * 3 * I * D * Ls
    tf_peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    tflops = fl / world / (ms * 1e-3) / 1e12
    roofline = ({"bound": "hbm", "achieved": per_gpu_gbs, "peak": hbm_peak, "unit": "GB/s",
                 "frac": per_gpu_gbs / hbm_peak} if T < 1024 else
                {"bound": "tensor", "achieved": tflops, "peak": tf_peak, "unit": "TFLOP/s",
                 "frac": tflops / tf_peak})
    roofline.update({"traffic": None, "kernel": f"whole {Ls}-layer stack per GPU",
                     "peak_source": "measured" if peaks else "fallback"})
    per_layer = ep.kernels_per_step() if ep is not None else sbb.kernels_per_call(T, E, TOP_K, D, I)
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": T / (ms * 1e-3) if errors == 0 else None,
            "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "nvfp4 W4A4 (dynamic per-row activation globals)" if args.w4a4 else
                     W4A16_DTYPE,
            "data": "synthetic",
            "config": {"workload": f"config3-stack {Ls} layers E={E} d={D} I={I} top{TOP_K} "
                                   f"T={T} routing={routing}",
                       "global_batch": T,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       "l2": "inputs larger than L2: every layer's weights are read each step"},
            "tokens_per_gpu": Tr, "weights_gb": Ls * E * EXPERT_BYTES / 1e9,
            "timing": ("CUDA graph replay (one graph per stack step)" if graph is not None
                       else "eager calls") + f"; median of {spread['repeats']} loops",
            "ms_per_layer": ms / Ls,
            "roofline": roofline, "cpu_baseline": None,
            "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": Tr * D * 2 + Ls * Tr * TOP_K * 8,
                    "d2h_bytes_per_step": Tr * D * 2, "ms_per_step": e2e_ms,
                    "copies": "serial, on the compute stream before and after the stack step"},
            "gpu_launches": per_layer * Ls * steps, "device_errors": errors,
            "clocks": clk.summary(),
        }
    del graph
    return line


# --------------------------------------------------------------------------
# single GPU
# --------------------------------------------------------------------------

class LayerBench:
    """One single-GPU workload (T tokens, routing, W4A16 or W4A4) over the
    shared rotating layers: graph replay timing, eager timing, per-stage
    events for the dominant kernel."""

    def __init__(self, sbb, device, layers, T, routing, w4a4, args, seed_base=2000):
        import torch
        self.sbb, self.device, self.layers = sbb, device, layers
        self.T, self.routing, self.w4a4, self.args = T, routing, w4a4, args
        self.n = len(layers)
        self.batches = [make_batch(device, T, seed=seed_base + 17 * i, routing=routing)
                        for i in range(self.n)]
        self.out = torch.empty((T, D), dtype=torch.bfloat16, device=device)
        self.stream = torch.cuda.current_stream(device)
        self.timer = StepTimer(self.stream, 1)

    def forward(self, h, ids, w, lw, out=None, stage_events=None, out_dtype=None):
        import torch
        out_dtype = out_dtype or torch.bfloat16
        if self.w4a4:
            return self.sbb.nvfp4_moe_w4a4(h, ids, w, *lw, out_dtype=out_dtype, out=out,
                                           stage_events=stage_events)
        if out is None and stage_events is None:
            return self.sbb.nvfp4_moe(h, ids, w, *lw, out_dtype=out_dtype)  # the public op
        return self.sbb._nvfp4_moe_impl(h, ids, w, *lw, True, out_dtype, out=out,
                                        stage_events=stage_events)

    def step(self, i):
        h, ids, w = self.batches[i % self.n]
        self.forward(h, ids, w, self.layers[i % self.n], out=self.out)

    def measure(self, steps, warmup, seconds, clk=None, eager=False):
        import torch
        for i in range(max(warmup, 3)):
            self.step(i)
        est = self.timer.loop_ms(self.step, max(warmup, 3))
        self.graphs = []
        if not eager:
            cap = torch.cuda.Stream(self.device)
            cap.wait_stream(self.stream)
            with torch.cuda.stream(cap):
                for i in range(self.n):
                    self.step(i)  # the capture stream's workspace exists before capture
            torch.cuda.synchronize()
            for i in range(self.n):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=cap):
                    self.step(i)
                self.graphs.append(gr)
            for i in range(max(warmup, 3)):
                self.graphs[i % self.n].replay()
            run = lambda i: self.graphs[i % self.n].replay()  # noqa: E731
        else:
            run = self.step
        repeats = self.timer.repeats_for(est, steps, seconds)
        if clk is not None:
            clk.start()
        ms, spread = self.timer.run(run, steps, repeats)
        if clk is not None:
            clk.stop()
        eager_ms = ms if eager else self.timer.run(self.step, steps, 3)[0]
        self.graphs = []
        # per-stage timing: the same calls with the C-ABI's stage events
        # recorded on the launching stream
        evsets = [self.sbb.stage_events(self.stream) for _ in range(steps)]
        torch.cuda.synchronize()
        for i in range(steps):
            h, ids, w = self.batches[i % self.n]
            self.forward(h, ids, w, self.layers[i % self.n], out=self.out,
                         stage_events=evsets[i])
        torch.cuda.synchronize()
        stage_ms = {name: statistics.mean(evs[j].elapsed_time(evs[j + 1]) for evs in evsets)
                    for j, name in enumerate(self.sbb.STAGE_NAMES)}
        return ms, eager_ms, spread, stage_ms

    def roofline(self, ms, stage_ms, peaks):
        """Dominant-kernel roofline (the gate/up GEMM): HBM for decode sizes,
        tensor pipe from 1,024 tokens."""
        T = self.T
        ids_all = [b[1].cpu().numpy() for b in self.batches]
        byts = [algorithmic_bytes(x, T) for x in ids_all]
        avg_bytes = sum(b for b, _ in byts) / len(byts)
        avg_distinct = sum(d for _, d in byts) / len(byts)
        hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
        peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
        step_gbs = avg_bytes / (ms * 1e-3) / 1e9
        gu_bytes = avg_distinct * W13_EXPERT_BYTES + T * D * 2
        dn_bytes = avg_distinct * W2_EXPERT_BYTES
        gu_gbs = gu_bytes / (stage_ms["gate_up"] * 1e-3) / 1e9
        dn_gbs = dn_bytes / (stage_ms["h_split+down"] * 1e-3) / 1e9
        info = {"distinct_experts_avg": avg_distinct, "algorithmic_bytes_per_step": avg_bytes}
        if T < 1024:
            traffic = profiled_traffic(T) if not self.w4a4 else None
            roof = {"bound": "hbm", "achieved": gu_gbs, "peak": hbm_peak, "unit": "GB/s",
                    "frac": gu_gbs / hbm_peak, "traffic": traffic,
                    "kernel": "moe_gemm_bs_kernel<gate/up> (w13 weight stream + SwiGLU)",
                    "algorithmic_bytes_per_launch": gu_bytes,
                    "launch_ms": stage_ms["gate_up"], "peak_source": f"{peak_src} hbm_gbs",
                    "stages_ms": stage_ms, "down_gbs": dn_gbs,
                    "whole_step_gbs": step_gbs, "whole_step_frac": step_gbs / hbm_peak}
            if traffic is not None:
                roof["traffic_launch_algorithmic_bytes"] = (
                    byts[0][1] * W13_EXPERT_BYTES + T * D * 2)
            return roof, info
        # prefill sizes: algorithmic FLOPs 2 * routes * 2I * d (gate/up) and
        # 2 * routes * d * I (down); W4A16 work counts against the measured
        # bf16 rate, W4A4 against the FP4 rate (4x). The kernels run inside a
        # seconds-long loop, so the sustained figure applies.
        routes = sum(int((x >= 0).sum()) for x in ids_all) / len(ids_all)
        fl_gu = 2.0 * routes * 2 * I * D
        fl_all = fl_gu * 1.5
        tf_peak = float(peaks.get("bf16_tflops_sustained", 1400.0)) * (4.0 if self.w4a4 else 1.0)
        tf_src = ("measured bf16_tflops_sustained" if "bf16_tflops_sustained" in peaks
                  else "fallback 1.4 PF sustained") + (" x4 (FP4 rate)" if self.w4a4 else "")
        gu_tf = fl_gu / (stage_ms["gate_up"] * 1e-3) / 1e12
        dn_tf = fl_gu / 2 / (stage_ms["h_split+down"] * 1e-3) / 1e12
        step_tf = fl_all / (ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": gu_tf, "peak": tf_peak, "unit": "TFLOP/s",
                "frac": gu_tf / tf_peak, "traffic": None,
                "kernel": "moe_gemm_bs_kernel<gate/up> (grouped GEMM + SwiGLU)",
                "algorithmic_flops_per_launch": fl_gu, "launch_ms": stage_ms["gate_up"],
                "peak_source": tf_src, "stages_ms": stage_ms, "down_tflops": dn_tf,
                "whole_step_tflops": step_tf, "whole_step_frac": step_tf / tf_peak,
                "bf16_burst_peak": float(peaks.get("bf16_tflops", 1590.0))}
        return roof, info


def run_single(args, sbb, rank, world, local):
    import torch
    device = torch.device("cuda", local)
    T = args.tokens
    N_LAYERS = args.layers
    routing = args.routing or default_routing(T)
    peaks = load_peaks()
    layers = make_layers(device, N_LAYERS, seed=1000 + rank)
    head = LayerBench(sbb, device, layers, T, routing, args.w4a4, args, seed_base=2000 + rank)
    clk = ClockSampler(local)
    ms, eager_ms, spread, stage_ms = head.measure(args.steps, args.warmup, args.min_timed_s,
                                                  clk=clk, eager=args.eager)
    clocks = clk.summary()
    roofline, info = head.roofline(ms, stage_ms, peaks)

    # ---- end-to-end through the public op with host buffers ---------------
    host_in = [(h.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory())
               for (h, ids, w) in head.batches]
    pipe = CopyPipeline(device, host_in, (T, D),
                        lambda i, x: head.forward(*x, layers[i % N_LAYERS]))
    for i in range(max(args.warmup, 3)):
        pipe.step(i)
    e2e_ms, _ = head.timer.run(pipe.step, args.steps, 3, finish=pipe.finish)
    h2d, d2h = pipe.bytes_per_step()
    # the same steps with the copies in line on the compute stream, for
    # comparison (what the overlap saves)
    dev_in = pipe.dev[0]

    def serial_step(i):
        for d, x in zip(dev_in, host_in[i % N_LAYERS]):
            d.copy_(x, non_blocking=True)
        o = head.forward(*dev_in, layers[i % N_LAYERS])
        pipe.host_out.copy_(o, non_blocking=True)

    serial_step(0)
    serial_ms, _ = head.timer.run(serial_step, args.steps, 3)

    # host copies for the CPU baseline (layer 0, batch 0), taken before the
    # stack measurement below frees the rotating layers
    cpu_in = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_in = (layer_to_host(layers[0]), host_batch(head.batches[0]))

    # ---- the other single-GPU workloads of the configurations -------------
    workloads = {}
    if not args.no_extras and world == 1 and not args.w4a4 and T == 64 and not args.eager:
        extras = [(1, "uniform", False), (8, "uniform", False), (32, "uniform", False),
                  (8192, "biased", False), (4096, "zipf", False), (4096, "zipf", True)]
        for (t, r, w4) in extras:
            lb = LayerBench(sbb, device, layers, t, r, w4, args, seed_base=3000 + t)
            xclk = ClockSampler(local)
            xms, xeager, xspread, xstage = lb.measure(args.steps, args.warmup, 0.25, clk=xclk)
            xroof, xinfo = lb.roofline(xms, xstage, peaks)
            workloads[workload_name(t, r, w4)] = {
                "value": t / (xms * 1e-3), "unit": "tokens/s", "ms_per_step": xms,
                "eager_ms_per_step": xeager, "loop_spread_ms": xspread,
                "roofline": xroof, **xinfo, "clocks": xclk.summary(),
                "gpu_launches": sbb.kernels_per_call(t, E, TOP_K, D, I) * args.steps}
            del lb
            torch.cuda.empty_cache()
        # config 3 on one GPU: the 46-layer stack (69 GB of weights), decode
        # T = 64 and a 32,768-token prefill (three timed steps: 0.5 s each)
        if args.stack_extras:
            head.batches = []
            del head
            layers.clear()
            torch.cuda.empty_cache()
            st_layers = stack_layers(device, 46)
            for t, st_steps in ((64, args.steps), (32768, 3)):
                sl = measure_stack(args, sbb, rank, world, local, t, st_layers, None, st_steps,
                                   3)
                workloads[sl["config"]["workload"]] = {
                    k: sl[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup",
                                       "ms_per_layer", "roofline", "e2e", "clocks",
                                       "gpu_launches", "device_errors", "weights_gb")}
                torch.cuda.empty_cache()
            del st_layers
            torch.cuda.empty_cache()
    errors = sbb.device_errors(device)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import nvfp4 as O
            if not O.reference_available():
                O.build(ref=True)
            if O.reference_available() and cpu_in is not None:
                hb, hids, hw = cpu_in[1]
                tps, sample, threads, _, _ = cpu_reference_run(
                    cpu_in[0], hb, hids, hw, args.cpu_seconds)
                cpu_baseline = {"value": tps, "unit": "tokens/s", "cores": threads,
                                "kind": "reference", "sample": sample, "isa": cpu_isa()}
        except Exception as exc:  # the baseline is reported, never required
            cpu_baseline = {"error": str(exc)[:200]}

    launches_per_step = sbb.kernels_per_call(T, E, TOP_K, D, I)
    if rank == 0:
        line = {
            "metric": METRIC, "value": world * T / (ms * 1e-3) if errors == 0 else None,
            "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("nvfp4 W4A4: e2m1 weights x e2m1 activations (dynamic per-row globals), "
                      "mxf4nvf4 MMA, fp32 accumulate") if args.w4a4 else
                     W4A16_DTYPE,
            "data": "synthetic",
            "config": single_config(T, routing, args.w4a4),
            "tokens_per_gpu": T,
            "replicas": world if world > 1 else None,
            **info,
            "timing": ("CUDA graph replay" if not args.eager else "eager calls")
                      + f"; median of {spread['repeats']} loops of {args.steps} steps, each "
                        "after one untimed step",
            "loop_spread_ms": spread,
            "eager_ms_per_step": eager_ms,
            "weight_stream_gbs": roofline.get("whole_step_gbs"),
            "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "copies": CopyPipeline.DESCRIPTION,
                    "serial_copies": {"value": world * T / (serial_ms * 1e-3),
                                      "ms_per_step": serial_ms,
                                      "copies": "in line on the compute stream before and "
                                                "after each step"}},
            "gpu_launches": launches_per_step * args.steps,
            "device_errors": errors,
            "clocks": clocks,
            "workloads": workloads or None,
        }
        if errors:
            line["invalid"] = "device error bits set during the run; no value reported"
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference_arm(args)
        return
    import torch
    import __graft_entry__ as g

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sbb = g.load_package()
    if args.stack:
        run_stack(args, sbb, rank, world, local)
    elif world > 1 and not args.replicas:
        run_expert_parallel(args, sbb, rank, world, local)
    else:
        run_single(args, sbb, rank, world, local)


if __name__ == "__main__":
    main()
