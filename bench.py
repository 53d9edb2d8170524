"""Benchmark of the routed-expert NVFP4 MoE layer on B200.

Headline workload (decode-shaped full layer): E=170 routed
experts, hidden d=4096, expert intermediate I=1280, top-8, T=64 tokens, NVFP4
weights (bf16 N(0, 0.02) quantised with per-tensor global amax/(448*6)),
bf16 N(0, 1) activations, uniform-random top-8 routing with softmax-
renormalised weights. Synthetic seeded data; the weights are random-init.

A "step" is one routed-expert layer forward over one batch of T tokens. Four
independent layers (4 x 1.5 GB) rotate across steps so consecutive steps
never find their weights in the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T]
    python bench.py --impl reference ...   # the reference's CPU expert tier

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

E, D, I, TOP_K = 170, 4096, 1280, 8
N_LAYERS = 4
EXPERT_BYTES = 2 * I * D // 2 + 2 * I * D // 16 + D * I // 2 + D * I // 16 + 8
METRIC = "routed-expert tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
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


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------
# synthetic inputs
# --------------------------------------------------------------------------

_E2M1_THRESH = None


def quantize_plane_torch(w, G):
    """NVFP4 quantisation of a [rows, cols] plane with plain torch ops (vLLM
    ref_nvfp4_quant semantics): data generation shared by both bench arms, so
    they see identical bytes; the library's own quantiser is not used here."""
    import torch
    rows, cols = w.shape
    x = w.float().reshape(rows, cols // 16, 16)
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
        for e in range(E):
            for (q, sf, g, shape) in ((w13, s13, g13, (2 * I, D)), (w2, s2, g2, (D, I))):
                w = (torch.randn(shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)
                amax = w.float().abs().max()
                G = torch.tensor(2688.0, device=device) / amax
                g[e] = amax / 2688.0
                qe, se = quantize_plane_torch(w, G)
                q[e].copy_(qe)
                sf[e].copy_(se)
        layers.append((w13, s13, g13, w2, s2, g2))
    return layers


def layer_to_host(tensors):
    from oracle import nvfp4 as O
    w13, s13, g13, w2, s2, g2 = (t.cpu().numpy() for t in tensors)
    return O.Layer(E, D, I, w13, s13, g13, w2, s2, g2)


def make_batch(device, T, seed):
    """bf16 N(0,1) hidden [T, d]; uniform-random top-8 (distinct experts, the
    top-8 of N(0,1) logits) with softmax-renormalised weights."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    hidden = torch.randn((T, D), generator=gen, device=device).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen, device=device)
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

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

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
# CPU baselines (reference CPU expert tier, compiled from its source)
# --------------------------------------------------------------------------

def cpu_reference_run(layer_host, hidden_bits, ids, w, seconds):
    """Time the reference's CPU expert tier (sb_cpu_moe_forward, compiled from
    its source) on one 170-expert layer of the headline workload with all host
    threads. Returns (tokens/s, sample description, threads, seconds/call)."""
    from oracle import nvfp4 as O
    threads = os.cpu_count() or 1
    T = hidden_bits.shape[0]
    tier = O.ReferenceCpuTier(layer_host, threads=threads)
    tier.forward(hidden_bits, ids, w)  # warm-up: first touch of the arena
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        tier.forward(hidden_bits, ids, w)
        times.append(time.perf_counter() - t0)
        if len(times) >= 500:
            break
    tier.close()
    per_call = statistics.median(times)
    return T / per_call, (f"median of {len(times)} sb_cpu_moe_forward calls on one 170-expert "
                          f"layer, T={T}"), threads, per_call


def host_batch(batch):
    """(bf16 bits, ids, weights) numpy copies of a device batch."""
    import torch
    h, ids, w = batch
    return (h.view(torch.int16).cpu().numpy().view("uint16"), ids.cpu().numpy(),
            w.cpu().numpy())


# --------------------------------------------------------------------------
# main
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
    hb, ids, w = host_batch(make_batch(device, T, seed=2000))
    tps, sample, threads, per_call = cpu_reference_run(layer_host, hb, ids, w, args.cpu_seconds)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_call * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config1-decode E={E} d={D} I={I} top{TOP_K} T={T}",
                   "global_batch": T, "parallelism": "host threads"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference_arm(args)
        return
    import numpy as np
    import torch
    import __graft_entry__ as g

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    sbb = g.load_package()
    T = args.tokens

    layers = make_layers(device, N_LAYERS, seed=1000 + rank)
    batches = [make_batch(device, T, seed=2000 + 17 * i + rank) for i in range(N_LAYERS)]
    out = torch.empty((T, D), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    def step(i):
        lw = layers[i % N_LAYERS]
        h, ids, w = batches[i % N_LAYERS]
        sbb._nvfp4_moe_impl(h, ids, w, *lw, True, torch.bfloat16, out=out)

    # ---- device-resident timing ------------------------------------------
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ev0.elapsed_time(ev1), world) / args.steps
    clocks = clk.summary()

    # ---- per-stage timing for the roofline: the same calls with the C-ABI's
    # stage events recorded on the launching stream ------------------------
    evsets = [sbb.stage_events(stream) for _ in range(args.steps)]
    torch.cuda.synchronize()
    for i in range(args.steps):
        lw = layers[i % N_LAYERS]
        h, ids, w = batches[i % N_LAYERS]
        sbb._nvfp4_moe_impl(h, ids, w, *lw, True, torch.bfloat16, out=out, stage_events=evsets[i])
    torch.cuda.synchronize()
    stage_ms = {name: statistics.mean(evs[j].elapsed_time(evs[j + 1]) for evs in evsets)
                for j, name in enumerate(sbb.STAGE_NAMES)}

    # ---- end-to-end through the public op with host buffers ---------------
    host_in = []
    for (h, ids, w) in batches:
        host_in.append((h.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory()))
    host_out = torch.empty((T, D), dtype=torch.bfloat16).pin_memory()
    dh = torch.empty_like(batches[0][0])
    di = torch.empty_like(batches[0][1])
    dw = torch.empty_like(batches[0][2])

    def e2e_step(i):
        hh, hi, hw = host_in[i % N_LAYERS]
        dh.copy_(hh, non_blocking=True)
        di.copy_(hi, non_blocking=True)
        dw.copy_(hw, non_blocking=True)
        o = sbb.nvfp4_moe(dh, di, dw, *layers[i % N_LAYERS], out_dtype=torch.bfloat16)
        host_out.copy_(o, non_blocking=True)

    for i in range(max(args.warmup, 3)):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    h2d = T * D * 2 + T * TOP_K * 4 + T * TOP_K * 4
    d2h = T * D * 2

    # ---- algorithmic bytes and roofline -----------------------------------
    ids_all = [b[1].cpu().numpy() for b in batches]
    byts = [algorithmic_bytes(x, T) for x in ids_all]
    avg_bytes = sum(b for b, _ in byts) / len(byts)
    avg_distinct = sum(d for _, d in byts) / len(byts)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    achieved_step = avg_bytes / (ms * 1e-3) / 1e9

    # dominant kernel: gate/up + SwiGLU streams w13 (2/3 of the weight bytes)
    distinct_bytes_w13 = avg_distinct * (2 * I * D // 2 + 2 * I * D // 16 + 4) + T * D * 2
    distinct_bytes_w2 = avg_distinct * (D * I // 2 + D * I // 16 + 4)
    gu_gbs = distinct_bytes_w13 / (stage_ms["gate_up"] * 1e-3) / 1e9
    dn_gbs = distinct_bytes_w2 / (stage_ms["down"] * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": gu_gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": gu_gbs / hbm_peak, "traffic": None,
                "kernel": "gate/up + SwiGLU (w13 weight stream)",
                "algorithmic_bytes_per_launch": distinct_bytes_w13,
                "launch_ms": stage_ms["gate_up"], "peak_source": f"{peak_src} hbm_gbs",
                "stages_ms": stage_ms, "down_gbs": dn_gbs,
                "whole_step_gbs": achieved_step, "whole_step_frac": achieved_step / hbm_peak}

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import nvfp4 as O
            if not O.reference_available():
                O.build(ref=True)
            if O.reference_available():
                hb, hids, hw = host_batch(batches[0])
                tps, sample, threads, _ = cpu_reference_run(layer_to_host(layers[0]), hb, hids,
                                                            hw, args.cpu_seconds)
                cpu_baseline = {"value": tps, "unit": "tokens/s", "cores": threads,
                                "kind": "reference", "sample": sample}
        except Exception as exc:  # the baseline is reported, never required
            cpu_baseline = {"error": str(exc)[:200]}

    launches_per_step = sbb.kernels_per_call(T * TOP_K)
    if rank == 0:
        line = {
            "metric": METRIC, "value": world * T / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16/bf16 MMA operands, fp32 accumulate (NVFP4 W4A16)",
            "data": "synthetic",
            "config": {"workload": f"config1-decode E={E} d={D} I={I} top{TOP_K} T={T}",
                       "global_batch": world * T, "tokens_per_gpu": T,
                       "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": f"{N_LAYERS} rotating layers of {E * EXPERT_BYTES / 1e9:.2f} GB",
                       "distinct_experts_avg": avg_distinct,
                       "algorithmic_bytes_per_step": avg_bytes},
            "weight_stream_gbs": achieved_step,
            "roofline": roofline,
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
