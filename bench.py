#!/usr/bin/env python
"""MoE-layer throughput of the B200 Qwen3-MoE hot path (one JSON line).

Workload (N=1): the sparse-MoE block of the config-1 decoder layer -- prefill
batch 1 x seq 1024 = 1024 tokens, hidden 2048, 128 experts, top-8,
moe_intermediate 768, bf16, random-init weights ~N(0, 0.02), activations
~N(0, 1).  A step = one MoE-layer forward (router -> permutation -> gate/up +
SiLU*up -> down + weighted combine -> bf16 output) over the 1024 tokens, with
inputs resident in HBM.  The 1.2 GB of expert weights are larger than L2
(126 MB), so every step streams them from HBM again.

N>1 (torchrun): expert parallel over peer memory -- rank r owns experts
[r*E/N, (r+1)*E/N) and its own 1024 tokens; each (token, slot) row is stored
straight into its expert owner's receive buffer over NVLink and comes back
weighted from the owner's down-GEMM epilogue (weak scaling).  value = tokens
of all ranks / max-over-ranks device time (whole job).  Every rank draws the
same full expert set from one seed, and after timing one step is compared
with the single-GPU forward on the same tokens ("parity" on the line; the
run exits non-zero if it fails).

Also reported on the same line:
  e2e          same metric through the public module API with the step's
               input copied from pinned host memory and its output read back
  roofline     N=1: moe_fused_kernel (gate/up + down in one kernel) against
               the measured HBM copy rate; N>1: the local experts kernel
               against the measured bf16 tensor peak, with the step's
               tensor / NVLink / weight-stream target times
  cpu_baseline the reference CPU path (HF transformers Qwen3MoeSparseMoeBlock,
               the module the reference uses in CPU mode) on the host cores
  extras       N=1: decode-sized layers (B = 1..64 tokens, CUDA graph), the
               config-2 48-layer decode step, the Zipf-skewed (config 4) and a
               uniform 16,384-token block, the config-1 decoder layer, the
               config-3 48-layer prefill of 8 x 2048 tokens; N>1: config 4 and
               config 3 expert-parallel, each with a parity block

``--impl reference`` times only the reference CPU path (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

H, E, K_TOP, I_MOE = 2048, 128, 8, 768
GATE_UP_BYTES_PER_EXPERT = 2 * I_MOE * H * 2   # 6,291,456
DOWN_BYTES_PER_EXPERT = H * I_MOE * 2          # 3,145,728
METRIC = "MoE-layer tokens/s/GPU (prefill & decode) at 1-8 B200; % of HBM/tensor roofline"
UNIT = "tokens/s (whole job, all GPUs)"
MAX_REL_ERR = 2e-2   # activations: max |ours - ref| / max |ref| (bf16 outputs, fp32 accumulation)
# A token routed differently after last-bit differences upstream of the
# router must be a near tie: its k-th and (k+1)-th fp32 logits within this
# (a bf16 ulp of the router input moves the logits by ~2e-3; the median
# k-th/(k+1)-th gap at these shapes is ~0.04)
FLIP_GAP_MAX = 2e-2


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--extras", default=None,
                    help="comma list of extras to run (decode_layer, decode_step, cfg4, uniform16k, "
                         "cfg1_layer, cfg3); default all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--clock-settle-s", type=float, default=1.0,
                    help="untimed load before warm-up so clocks settle and get sampled")
    ap.add_argument("--prefill-attention", default=None, metavar="BxS",
                    help="profiling aid: only run the flash-prefill attention kernel on B sequences of S "
                         "tokens (32 query / 4 KV heads of 128) for --steps launches and print its time")
    ap.add_argument("--decode-model", type=int, default=0, metavar="LAYERS",
                    help="profiling aid: only run the config-2 decode step of a LAYERS-layer model "
                         "(--tokens = batch) for --steps graph replays and print its time")
    return ap.parse_args()


# ----------------------------------------------------------------------------
# peaks, clocks
# ----------------------------------------------------------------------------

def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", 0)), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), util=float(parts[4]),
                                 hw=parts[6], hwt=parts[7], swt=parts[8], pcap=parts[9]))
            except ValueError:
                continue
        os.unlink(self.path)
        loaded = [r for r in rows if r["util"] >= 50] or rows
        if not loaded:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        reasons = set()
        for r in loaded:
            if r["hw"] == "Active":
                reasons.add("hw_slowdown")
            if r["hwt"] == "Active":
                reasons.add("hw_thermal_slowdown")
            if r["swt"] == "Active":
                reasons.add("sw_thermal_slowdown")
            if r["pcap"] == "Active":
                reasons.add("sw_power_cap")
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["smax"] for r in loaded), "reasons": sorted(reasons),
                "samples": len(loaded)}


BAD_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


# ----------------------------------------------------------------------------
# reference CPU path (HF transformers, the reference's CPU-mode module)
# ----------------------------------------------------------------------------

def make_hf_block(w_router, w_gate_up, w_down):
    import torch
    from transformers import Qwen3MoeConfig as HFConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeSparseMoeBlock

    cfg = HFConfig(hidden_size=H, num_experts=E, num_experts_per_tok=K_TOP, moe_intermediate_size=I_MOE,
                   norm_topk_prob=True, hidden_act="silu")
    blk = Qwen3MoeSparseMoeBlock(cfg).to(torch.bfloat16)
    with torch.no_grad():
        blk.gate.weight.copy_(w_router.cpu())
        blk.experts.gate_up_proj.copy_(w_gate_up.cpu())
        blk.experts.down_proj.copy_(w_down.cpu())
    return blk.eval()


def time_cpu_reference(blk, x_cpu, budget_s: float, min_runs: int = 3):
    """Median seconds of HF forward on x_cpu (1, T, H), all host threads."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    with torch.no_grad():
        blk(x_cpu)  # warm-up
        times = []
        t_start = time.perf_counter()
        while len(times) < min_runs or (time.perf_counter() - t_start) < budget_s * 0.5:
            t0 = time.perf_counter()
            blk(x_cpu)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > budget_s:
                break
    return statistics.median(times), len(times)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    T = args.tokens
    # Weights drawn on the host (same distributions as the GPU arm).
    g = torch.Generator().manual_seed(0)
    w_router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    w_gate_up = (torch.randn(E, 2 * I_MOE, H, generator=g) * 0.02).to(torch.bfloat16)
    w_down = (torch.randn(E, H, I_MOE, generator=g) * 0.02).to(torch.bfloat16)
    blk = make_hf_block(w_router, w_gate_up, w_down)
    torch.set_num_threads(os.cpu_count() or 1)
    x_full = torch.randn(1, T, H, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        t0 = time.perf_counter()
        blk(x_full)
        t1 = time.perf_counter() - t0
    # bounded sample: K steps of at most ~120 s in total
    budget = 120.0
    per_step_tokens = T
    if (args.steps + args.warmup) * t1 > budget:
        per_step_tokens = max(8, int(T * budget / ((args.steps + args.warmup) * t1)))
    x = x_full[:, :per_step_tokens].contiguous()
    with torch.no_grad():
        for _ in range(args.warmup):
            blk(x)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            blk(x)
        el = time.perf_counter() - t0
    value = per_step_tokens * args.steps / el
    cores = torch.get_num_threads()
    sample = (f"HF transformers Qwen3MoeSparseMoeBlock (eager experts, bf16) on {per_step_tokens} of the "
              f"{T} tokens per step, {args.steps} steps, {cores} threads on {cpu_model()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights and activations)",
        "config": {"workload": f"qwen3-moe sparse block, cfg1 prefill 1x{T} tokens (reference CPU path)",
                   "hidden": H, "experts": E, "top_k": K_TOP, "moe_intermediate": I_MOE},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------

def _events(n):
    import torch

    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def _max_over_ranks(v: float, dev, world: int) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _want(args, name: str) -> bool:
    return args.extras is None or name in args.extras.split(",")


def run_ours(args):
    import torch
    import torch.distributed as dist

    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.moe import MoEPlan, MoEWeights, Qwen3MoeSparseMoeBlock

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _C.lib()

    cfg = Qwen3MoeConfig()
    T = args.tokens
    weights = MoEWeights.random(cfg, seed=0, device=dev)
    from nki_moe_7013_b200.synth import normal_bf16_device

    x = normal_bf16_device(1000 + rank, (T, H), 1.0, dev)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    plan = MoEPlan(weights, T, K_TOP)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sampler = ClockSampler() if rank == 0 else None

    def timed_run():
        # load phase: settle clocks and give the sampler samples (untimed)
        t_end = time.perf_counter() + args.clock_settle_s
        while time.perf_counter() < t_end:
            for _ in range(20):
                plan.run(x, out)
            torch.cuda.synchronize()
        for _ in range(args.warmup):
            plan.run(x, out)
        # timed region: K steps, events only at its two ends so consecutive
        # kernels keep their programmatic-launch overlap
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e_start.record()
        for _ in range(args.steps):
            plan.run(x, out)
        e_end.record()
        barrier()
        span_ms = e_start.elapsed_time(e_end)
        # stage pass: the same K steps again with an event between every
        # kernel, for the per-kernel durations (roofline) and the breakdown
        ns = len(plan.stages)
        ev = [_events(ns + 1) for _ in range(args.steps)]
        barrier()
        for s_ in range(args.steps):
            plan.run(x, out, events=ev[s_])
        barrier()
        stage_ms = [statistics.mean(ev[s_][i].elapsed_time(ev[s_][i + 1]) for s_ in range(args.steps))
                    for i in range(ns)]
        return span_ms, stage_ms

    if sampler:
        sampler.start()
    span_ms, stage_ms = timed_run()
    clocks = sampler.stop() if sampler else None
    if clocks and set(clocks["reasons"]) & BAD_REASONS:
        sampler.start()
        span_ms, stage_ms = timed_run()
        clocks = sampler.stop()
        clocks["remeasured"] = True
    torch.cuda.synchronize()
    dev_err = _C.device_error()
    if dev_err:
        raise RuntimeError(f"device error word {dev_err} set during the timed steps")

    span_ms = _max_over_ranks(span_ms, dev, world)
    ms_per_step = span_ms / args.steps
    value = T * world * args.steps / (span_ms / 1e3)

    # routing statistics of this workload (distinct experts hit)
    counts = plan.counts.cpu()
    U = int((counts > 0).sum().item())
    R = T * K_TOP
    hbm_gbs, tf_burst, tf_sust, peak_kind = load_peaks()
    if plan.fused:
        # dominant kernel: gate/up + down in one persistent kernel.
        # Algorithmic bytes: the hit experts' weights (9,437,184 B each) and
        # the token rows in and out.  The kernel's own intermediates (the
        # permuted row copy, the SwiGLU activations written and read back,
        # the fp32 combine rows) are not counted; they show in `traffic`.
        kern_name = "moe_fused_kernel (gate/up + down)"
        kern_bytes = U * (GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT) + 2 * T * H * 2
        inter_bytes = R * H * 2 + 2 * R * I_MOE * 2 + T * H * 4
        kern_us = stage_ms[plan.stages.index("experts")] * 1e3
    else:
        kern_name = "grouped_gemm_kernel<gate_up>"
        kern_bytes = U * GATE_UP_BYTES_PER_EXPERT + T * H * 2
        inter_bytes = R * I_MOE * 2
        kern_us = stage_ms[plan.stages.index("gate_up")] * 1e3
    achieved = kern_bytes / (kern_us * 1e-6) / 1e9
    layer_bytes = U * (GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT) + E * H * 2 + 4 * T * H + 8 * T * K_TOP
    layer_gbs = layer_bytes / (ms_per_step * 1e-3) / 1e9

    # ---------------- e2e through the public module API ----------------
    # Each step copies its input from pinned host memory, runs the module and
    # reads the output back to pinned host memory.  Copies run on their own
    # streams so step i's compute overlaps step i+1's upload and step i-1's
    # download (double-buffered), as a serving loop would.
    block = Qwen3MoeSparseMoeBlock(cfg, weights=weights, device=dev)
    x_host = x.reshape(1, T, H).cpu().pin_memory()
    y_host = [torch.empty((1, T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty((1, T, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def e2e_steps(n):
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_used = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for ev in ev_used + ev_out:
            ev.record(comp)
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        with torch.cuda.stream(s_in):
            xd[0].copy_(x_host, non_blocking=True)
            ev_in[0].record(s_in)
        for i in range(n):
            b = i & 1
            if i + 1 < n:  # upload the next step's input while this one computes
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_used[b ^ 1])
                    xd[b ^ 1].copy_(x_host, non_blocking=True)
                    ev_in[b ^ 1].record(s_in)
            comp.wait_event(ev_in[b])
            comp.wait_event(ev_out[b])  # y_host[b] free again
            y = block(xd[b])[0]
            ev_used[b].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[b])
                y_host[b].copy_(y, non_blocking=True)
                y.record_stream(s_out)
                ev_out[b].record(s_out)
        comp.wait_stream(s_out)

    e2e_steps(max(args.warmup, 3))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_steps(args.steps)
    e1.record()
    barrier()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dev, world)
    e2e_value = T * world * args.steps / (e2e_ms / 1e3)
    y_check = y_host[(args.steps - 1) & 1].to(dev).float().reshape(T, H)
    y_ref = block(x.reshape(1, T, H))[0].float().reshape(T, H)
    if float((y_check - y_ref).abs().max() / y_ref.abs().max()) > 1e-2:
        raise RuntimeError("e2e output differs from the device-resident run")

    # ---------------- traffic from the committed ncu capture ----------------
    traffic = None
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            tr = json.load(f)
        ent = tr.get(f"{'experts' if plan.fused else 'gate_up'}_T{T}")
        if ent:
            traffic = float(ent["dram_bytes_per_launch"])
    except Exception:
        pass

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights ~N(0,0.02), activations ~N(0,1))",
        "config": {"workload": f"qwen3-moe sparse block of the cfg1 decoder layer, prefill 1x{T} tokens",
                   "tokens_per_gpu": T, "hidden": H, "experts": E, "top_k": K_TOP,
                   "moe_intermediate": I_MOE, "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2: 1.21 GB of expert weights streamed per step"},
        "value_per_gpu": value / world,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "api": "Qwen3MoeSparseMoeBlock.forward(hidden_states)[0], pinned host in/out, "
                       "uploads and downloads on their own streams overlapping compute"},
        "gpu_launches": plan.launches_per_run * args.steps,
        "stage_us": dict(zip(plan.stages, [round(s * 1e3, 2) for s in stage_ms])),
        "stage_note": "per-kernel CUDA-event times from a second pass of the K steps with an event "
                      "between every kernel; value uses events at the ends of the timed region only",
        "roofline": {"bound": "hbm", "kernel": kern_name,
                     "achieved": achieved, "peak": hbm_gbs, "unit": "GB/s", "frac": achieved / hbm_gbs,
                     "peak_kind": peak_kind, "traffic": traffic,
                     "algorithmic_bytes_per_launch": kern_bytes,
                     "algorithmic_bytes": "experts hit x 9,437,184 B of weights + token rows in and out",
                     "kernel_intermediate_bytes_per_launch": inter_bytes,
                     "kernel_us": kern_us, "experts_hit": U},
        "layer_roofline": {"bound": "hbm", "achieved": layer_gbs, "peak": hbm_gbs, "unit": "GB/s",
                           "frac": layer_gbs / hbm_gbs, "algorithmic_bytes_per_step": layer_bytes},
        "device_error": dev_err,
        "clocks": clocks,
    }

    if rank == 0 and not args.no_extras:
        line["extras"] = run_extras(args, cfg, weights, dev, hbm_gbs, tf_burst)

    if rank == 0 and not args.no_cpu_baseline:
        blk = make_hf_block(weights.router, weights.gate_up, weights.down)
        med, runs = time_cpu_reference(blk, x.reshape(1, T, H).cpu(), args.cpu_budget_s)
        import torch as _t

        line["cpu_baseline"] = {
            "value": T / med, "unit": UNIT, "cores": _t.get_num_threads(), "kind": "reference",
            "sample": (f"HF transformers Qwen3MoeSparseMoeBlock (the module the reference uses in CPU "
                       f"mode, qwen.py:35-37), bf16, same weights and {T} tokens, median of {runs} runs "
                       f"on {cpu_model()}")}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def prefill_block_line(weights, T, dev, tf_burst, bias=None, x_seed=4242):
    """One prefill-sized MoE layer (T tokens): device time per layer, stage
    times, and the expert GEMMs' FLOP rate against the measured bf16 peak."""
    import torch

    from nki_moe_7013_b200.moe import MoEPlan
    from nki_moe_7013_b200.synth import normal_bf16_device

    plan = MoEPlan(weights, T, K_TOP, bias=bias)
    x = normal_bf16_device(x_seed, (T, H), 1.0, dev)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        plan.run(x, out)
    e0, e1 = _events(2)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(10):
        plan.run(x, out)
    e1.record()
    torch.cuda.synchronize()
    total_ms = e0.elapsed_time(e1) / 10
    ns = len(plan.stages)
    ev = [_events(ns + 1) for _ in range(10)]
    for s in range(10):
        plan.run(x, out, events=ev[s])
    torch.cuda.synchronize()
    stage = [statistics.mean(ev[s][i].elapsed_time(ev[s][i + 1]) for s in range(10)) for i in range(ns)]
    counts = plan.counts.cpu()
    flops_gemm = T * 6 * K_TOP * H * I_MOE
    gemm_ms = sum(v for name, v in zip(plan.stages, stage) if name in ("experts", "gate_up", "down"))
    tflops = flops_gemm / (gemm_ms * 1e-3) / 1e12
    return {
        "ms_per_layer": round(total_ms, 3), "tokens_per_s": T / (total_ms * 1e-3),
        "stage_us": dict(zip(plan.stages, [round(v * 1e3, 1) for v in stage])),
        "expert_gemm_tflops": tflops, "tensor_frac": tflops / tf_burst, "tensor_peak_tflops": tf_burst,
        "layer_tflops": T * 76021760 / (total_ms * 1e-3) / 1e12,
        "max_expert_rows": int(counts.max().item()), "mean_expert_rows": float(counts.float().mean().item()),
    }


def decoder_layer_line(cfg, weights, dev, tf_burst, S=1024):
    """Config 1: the full decoder layer (input RMSNorm, QKV projection, QK-norm
    + RoPE + cache append, causal GQA flash prefill, O projection, add & norm,
    MoE, residual) on 1 x S tokens: layer time, per-stage times, the
    attention kernel's FLOP rate."""
    import torch

    from nki_moe_7013_b200.attention import StageTimer
    from nki_moe_7013_b200.decoder import Qwen3MoeDecoderLayer
    from nki_moe_7013_b200.synth import normal_bf16_device

    layer = Qwen3MoeDecoderLayer(cfg, moe_weights=weights, device=dev, seed=5)
    x = normal_bf16_device(55, (1, S, H), 1.0, dev)
    cache = layer.self_attn.new_cache(1, S)
    for _ in range(3):
        layer(x, past_key_value=cache.reset())
    n = 10
    e0, e1 = _events(2)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(n):
        layer(x, past_key_value=cache.reset())
    e1.record()
    torch.cuda.synchronize()
    layer_ms = e0.elapsed_time(e1) / n
    timers = []
    for _ in range(n):
        t = StageTimer()
        layer(x, past_key_value=cache.reset(), timer=t)
        timers.append(t)
    torch.cuda.synchronize()
    stages = {}
    for t in timers:
        for k_, v in t.totals_ms().items():
            stages[k_] = stages.get(k_, 0.0) + v / n
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    attn_flops = 4 * hd * nh * S * (S + 1) // 2          # causal QK^T and PV
    proj_flops = 2 * S * H * (nh + 2 * nkv) * hd + 2 * S * nh * hd * H
    a_ms = stages.get("attention", float("nan"))
    return {
        "tokens": S, "ms_per_layer": round(layer_ms, 4), "tokens_per_s": S / (layer_ms * 1e-3),
        "stage_us": {k_: round(v * 1e3, 1) for k_, v in stages.items()},
        "attention_kernel_tflops": attn_flops / (a_ms * 1e-3) / 1e12,
        "attention_tensor_frac": attn_flops / (a_ms * 1e-3) / 1e12 / tf_burst,
        "attention_flops": attn_flops, "projection_flops": proj_flops,
        "note": "stage_us from a second pass with CUDA events around every stage; ms_per_layer has events "
                "only at the ends of 10 layer calls",
    }


def prefill_model_line(cfg, dev, world, rank, group=None, batch=8, seq=2048, layers=None, runs=3):
    """Config 3: batch x seq tokens through the 48-layer random-init model
    (embedding, 48 decoder layers, final norm, LM head on each sequence's
    last position).  world == 1: one GPU holds everything; world > 1: the
    experts are sharded over the ranks (EP) and each rank runs batch/world
    sequences (attention data-parallel).  Returns the line, the model and
    this rank's token ids."""
    import torch

    from nki_moe_7013_b200.attention import StageTimer
    from nki_moe_7013_b200.model import Qwen3MoeModel

    nl = cfg.num_hidden_layers if layers is None else layers
    b_local = batch // world
    T_local = b_local * seq
    g = torch.Generator(device=dev)
    g.manual_seed(333)
    ids = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g, device=dev, dtype=torch.int32)
    ids_local = ids[rank * b_local:(rank + 1) * b_local].contiguous()
    if world == 1:
        model = Qwen3MoeModel(cfg, num_layers=nl, device=dev, seed=3)
    else:
        model = Qwen3MoeModel.expert_parallel(cfg, T_local, group=group, num_layers=nl, device=dev, seed=3)
    caches = model.new_caches(b_local, seq)

    def run(timer=None):
        for c in caches:
            c.reset()
        if timer is None:
            return model.forward(ids_local, caches, last_only=True)[0]
        x, _ = model.hidden_states(ids_local, caches, timer=timer)
        return x

    run()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier(group=group)
    e0, e1 = _events(2)
    e0.record()
    for _ in range(runs):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / runs, dev, world)
    timer = StageTimer()
    run(timer)
    torch.cuda.synchronize()
    st = {k_: round(v, 3) for k_, v in timer.totals_ms().items()}
    moe_flops = batch * seq * nl * 76021760
    line = {
        "batch": batch, "seq": seq, "layers": nl, "tokens": batch * seq, "tokens_per_gpu": T_local,
        "parallelism": f"ep{world} (attention data-parallel)" if world > 1 else "single",
        "ms_per_prefill": round(ms, 3), "tokens_per_s": batch * seq / (ms * 1e-3),
        "tokens_per_s_per_gpu": batch * seq / (ms * 1e-3) / world,
        "moe_tflops_per_gpu": moe_flops / world / (ms * 1e-3) / 1e12,
        "stage_ms_rank0_summed_over_layers": st,
        "note": "device time of the whole prefill (max over ranks); stage times from a second pass with "
                "CUDA events around every layer stage (without the LM head)",
    }
    return line, model, ids_local


def run_extras(args, cfg, weights, dev, hbm_gbs, tf_burst):
    """Decode-sized MoE layers (CUDA graph replay), the config-4 skewed block,
    a uniform 16,384-token block, the config-1 decoder layer, the config-2
    decode step and the config-3 prefill on one GPU."""
    import torch

    from nki_moe_7013_b200.moe import MoEPlan
    from nki_moe_7013_b200.synth import normal_bf16_device, zipf_expert_bias

    res = {}
    if _want(args, "decode_layer"):
        dec = {}
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 2x L2
        # 5 and 40 tokens: speculative-decoding verify steps (1 and 8 sequences x
        # 5 tokens), between decode and prefill
        for B in (1, 5, 8, 32, 40, 64):
            plan = MoEPlan(weights, B, K_TOP)
            x = normal_bf16_device(77 + B, (B, H), 1.0, dev)
            out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(3):
                    plan.run(x, out)
            torch.cuda.current_stream(dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                plan.run(x, out)
            for _ in range(5):
                g.replay()
            torch.cuda.synchronize()
            # The experts one small batch hits can fit in L2 (8 x 9.4 MB at B=1),
            # so L2 is flushed before every replay and each replay is timed alone.
            n = 50
            ev = [_events(2) for _ in range(n)]
            for i in range(n):
                flush.zero_()
                ev[i][0].record()
                g.replay()
                ev[i][1].record()
            torch.cuda.synchronize()
            us = statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3
            # the same layer without the graph, an event between stages
            ns = len(plan.stages)
            st = [_events(ns + 1) for _ in range(n)]
            for i in range(n):
                flush.zero_()
                plan.run(x, out, events=st[i])
            torch.cuda.synchronize()
            stage = [statistics.median(st[i][j].elapsed_time(st[i][j + 1]) for i in range(n)) * 1e3
                     for j in range(ns)]
            U = int((plan.counts.cpu() > 0).sum().item())
            byts = U * (GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT) + E * H * 2 + 4 * B * H + 8 * B * K_TOP
            dec[str(B)] = {"us_per_layer": round(us, 2), "tokens_per_s": B / (us * 1e-6),
                           "experts_hit": U, "hbm_frac": byts / (us * 1e-6) / 1e9 / hbm_gbs,
                           "stage_us_eager": dict(zip(plan.stages, [round(v, 1) for v in stage]))}
            if B in (5, 40):
                dec[str(B)]["shape"] = f"spec-verify step: {B // 5} sequence(s) x 5 tokens"
            del g
        del flush
        res["decode_moe_layer_cuda_graph"] = dec
    if _want(args, "decode_step"):
        res["decode_step_cfg2"] = run_decode_model(cfg, dev, hbm_gbs)
    if _want(args, "cfg4"):
        bias = zipf_expert_bias(0, E).to(dev)
        res["cfg4_zipf_T16384"] = prefill_block_line(weights, 16384, dev, tf_burst, bias=bias)
    if _want(args, "uniform16k"):
        res["uniform_T16384"] = prefill_block_line(weights, 16384, dev, tf_burst, x_seed=4343)
    if _want(args, "cfg1_layer"):
        res["cfg1_decoder_layer_1x1024"] = decoder_layer_line(cfg, weights, dev, tf_burst)
    if _want(args, "cfg3"):
        torch.cuda.empty_cache()
        line, model, _ = prefill_model_line(cfg, dev, 1, 0)
        res["cfg3_prefill_8x2048_48l"] = line
        del model
        torch.cuda.empty_cache()
    return res


def run_decode_model(cfg, dev, hbm_gbs, batches=(1, 8, 32, 64), context=4096):
    """Config 2: the 48-layer model (random weights ~N(0,0.02), vocab 151,936)
    decoding one token per sequence per step with 4,096 cached tokens per
    sequence (~N(0,1)); the whole step (embedding, 48 layers, final norm, LM
    head, greedy pick) replays as one CUDA graph.  60 GB of weights: no step
    finds its weights in L2."""
    import torch

    from nki_moe_7013_b200.model import DecodeSession, Qwen3MoeModel

    model = Qwen3MoeModel(cfg, device=dev, seed=1)
    nl, V = len(model.layers), model.vocab_size
    attn_bytes = sum(l.self_attn.w.wqkv.numel() + l.self_attn.w.wo.numel() for l in model.layers) * 2
    out = {}
    for B in batches:
        sess = DecodeSession(model, B, context=context, max_new=64, seed=B)
        sess.capture()
        for _ in range(2):
            sess.step()
        torch.cuda.synchronize()
        n = 10
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            sess.step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        U = sum(p.experts_hit() for p in sess.plans)
        kv_len = context + sess.steps_done
        byts = (U * (GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT) + nl * E * H * 2 + attn_bytes
                + V * H * 2 + nl * B * cfg.num_key_value_heads * kv_len * cfg.head_dim * 2 * 2)
        out[str(B)] = {"ms_per_step": round(ms, 3), "tokens_per_s": B / (ms * 1e-3),
                       "experts_hit_per_layer": round(U / nl, 1), "hbm_bytes_per_step": byts,
                       "hbm_frac": byts / (ms * 1e-3) / 1e9 / hbm_gbs}
        sess.release()
        del sess
        torch.cuda.empty_cache()
    return {"layers": nl, "vocab": V, "context": context, "per_batch": out,
            "note": "one CUDA graph per step: embedding, 48 x (norm, QKV, QK-norm+RoPE+append, split-KV "
                    "attention, O proj, add&norm, MoE), final norm, LM head, greedy pick"}


def _ep_parity(moe_out, ref_out, idx_ep, idx_ref, dev, world):
    """Parity of an expert-parallel step against the single-GPU forward on
    the same tokens and full weights, reduced over the ranks."""
    import torch
    import torch.distributed as dist

    from nki_moe_7013_b200 import _C

    torch.cuda.synchronize()
    a, b = moe_out.float(), ref_out.float()
    err = float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))
    same = 1.0 if torch.equal(idx_ep, idx_ref) else 0.0
    code = float(_C.device_error())
    t = torch.tensor([err, -same, code], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    err, same, code = float(t[0]), -float(t[1]), int(t[2])
    return {"max_rel_err": err, "routing_equal": bool(same == 1.0), "device_error": code,
            "tolerance": MAX_REL_ERR, "ok": bool(err <= MAX_REL_ERR and same == 1.0 and code == 0)}


def run_ours_ep(args):
    """N>1: the expert-parallel MoE layer over peer memory (NCCL for set-up)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from nki_moe_7013_b200 import _C, ops
    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.ep import PeerExpertParallelMoE
    from nki_moe_7013_b200.moe import MoEWeights
    from nki_moe_7013_b200.synth import normal_bf16_device

    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _C.lib()
    cfg = Qwen3MoeConfig()
    T = args.tokens
    el = E // world
    # every rank draws the same full expert set (one seed) and keeps its
    # slice; the full set stays for the parity check against one GPU
    full = MoEWeights.random(cfg, seed=0, device=dev)
    router = full.router
    local = MoEWeights(router, full.gate_up[rank * el:(rank + 1) * el].clone(),
                       full.down[rank * el:(rank + 1) * el].clone())
    moe = PeerExpertParallelMoE(cfg, router, local, max_tokens=T)
    x = normal_bf16_device(1000 + rank, (T, H), 1.0, dev)
    for _ in range(2):
        moe(x)  # eager steps: every kernel's attributes set before capture
    torch.cuda.synchronize()
    moe.capture(x)  # one CUDA graph per parity, each with its own input / output

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    sampler = ClockSampler() if rank == 0 else None

    def timed_run():
        # load phase: the same number of steps on every rank (each step's
        # exchange waits for every peer's same step), about clock_settle_s
        for _ in range(int(args.clock_settle_s * 3000)):
            moe.replay()
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            moe.replay()
        e0, e1 = _events(2)
        barrier()
        e0.record()
        for _ in range(args.steps):
            moe.replay()
        e1.record()
        barrier()
        return e0.elapsed_time(e1)

    if sampler:
        sampler.start()
    span_ms = timed_run()
    clocks = sampler.stop() if sampler else None
    torch.cuda.synchronize()
    err_timed = _max_over_ranks(_C.device_error(), dev, world)
    # stage pass (eager steps, an event between stages; every rank does it)
    ns = len(PeerExpertParallelMoE.STAGES)
    evs = [_events(ns + 1) for _ in range(10)]
    barrier()
    for i in range(10):
        moe(x, events=evs[i])
    barrier()
    stage_us = {name: round(statistics.median(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(10)) * 1e3, 1)
                for j, name in enumerate(PeerExpertParallelMoE.STAGES)}
    span_ms = _max_over_ranks(span_ms, dev, world)
    ms_per_step = span_ms / args.steps
    value = T * world * args.steps / (span_ms / 1e3)
    hbm_gbs, tf_burst, tf_sust, peak_kind = load_peaks()
    recv_rows = int(moe.recv_rows.item())
    idx = moe.topk_idx[:T]
    remote_sent = int((idx // el != rank).sum().item())     # my (token, slot) rows served elsewhere
    local_rows = T * K_TOP - remote_sent
    remote_recv = recv_rows - local_rows                    # (token, slot) rows other ranks sent me
    # dispatch sends each token row once per destination rank
    present = torch.zeros((T, world), dtype=torch.int32, device=dev).scatter_(1, idx.long() // el, 1)
    tok_to = present.sum(0)
    tok_in = tok_to.clone()
    if world > 1:
        torch.distributed.all_reduce(tok_in)
    tok_sent_remote = int(tok_to.sum().item() - tok_to[rank].item())
    tok_recv_remote = int(tok_in[rank].item() - tok_to[rank].item())
    # expert GEMM FLOPs of this rank's experts, and the bytes that must
    # cross NVLink per direction: token rows out (dispatch) + weighted rows I
    # return out, and token rows in + my weighted rows coming back
    flops_rank = recv_rows * 6 * H * I_MOE
    nvl_out = (tok_sent_remote + remote_recv) * H * 2
    nvl_in = (tok_recv_remote + remote_sent) * H * 2
    nvl_gbs_ref = 770.0
    t_tensor_us = flops_rank / (tf_burst * 1e12) * 1e6
    t_nvlink_us = max(nvl_out, nvl_in) / (nvl_gbs_ref * 1e9) * 1e6
    t_weights_us = el * (GATE_UP_BYTES_PER_EXPERT + DOWN_BYTES_PER_EXPERT) / (hbm_gbs * 1e9) * 1e6
    target_us = max(t_tensor_us, t_nvlink_us, t_weights_us)
    experts_us = stage_us["experts"]
    exp_tflops = flops_rank / (experts_us * 1e-6) / 1e12
    step_tflops = flops_rank / (ms_per_step * 1e-3) / 1e12

    # ---------------- e2e: module step with host copies, double-buffered ----------------
    # Each step uploads its input from pinned host memory into the static
    # input of its parity's graph and reads that graph's output back; the
    # upload of step i+1 and the download of step i run on their own streams
    # while step i computes (each parity has its own input and output).
    x_host = x.cpu().pin_memory()
    y_host = [torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def e2e_steps(n):
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for ev in ev_done + ev_out:
            ev.record(comp)
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        par = (moe.steps + 1) & 1
        with torch.cuda.stream(s_in):
            moe.static_input(1).copy_(x_host, non_blocking=True)
            ev_in[par].record(s_in)
        for i in range(n):
            par = (moe.steps + 1) & 1
            comp.wait_event(ev_in[par])
            comp.wait_event(ev_out[par])     # this parity's last output read back
            y = moe.replay()
            ev_done[par].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[par])
                y_host[par].copy_(y, non_blocking=True)
                ev_out[par].record(s_out)
            if i + 1 < n:  # next step's input: its buffer was last read by step i-1
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_done[par ^ 1])
                    moe.static_input(1).copy_(x_host, non_blocking=True)
                    ev_in[par ^ 1].record(s_in)
        comp.wait_stream(s_out)
        comp.wait_stream(s_in)
        return par

    e2e_steps(max(args.warmup, 3))
    barrier()
    e0, e1 = _events(2)
    e0.record()
    last_par = e2e_steps(args.steps)
    e1.record()
    barrier()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dev, world)
    e2e_value = T * world * args.steps / (e2e_ms / 1e3)
    y_e2e = y_host[last_par].to(dev)

    # what the host's copy paths give when every rank copies at once: the
    # same pinned 4 MB input up and output down, back to back, no compute
    def copy_rate(up: bool) -> float:
        buf = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        c0, c1 = _events(2)
        barrier()
        c0.record()
        for _ in range(args.steps):
            if up:
                buf.copy_(x_host, non_blocking=True)
            else:
                y_host[0].copy_(buf, non_blocking=True)
        c1.record()
        barrier()
        return _max_over_ranks(c0.elapsed_time(c1) / args.steps, dev, world)

    def copy_rate_both() -> float:
        # upload and download at once on their own streams, as the e2e loop does
        buf_in = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        buf_out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        c0, c1 = _events(2)
        s_in.wait_stream(torch.cuda.current_stream(dev))
        s_out.wait_stream(torch.cuda.current_stream(dev))
        barrier()
        c0.record()
        s_in.wait_event(c0)
        s_out.wait_event(c0)
        for _ in range(args.steps):
            with torch.cuda.stream(s_in):
                buf_in.copy_(x_host, non_blocking=True)
            with torch.cuda.stream(s_out):
                y_host[1].copy_(buf_out, non_blocking=True)
        torch.cuda.current_stream(dev).wait_stream(s_in)
        torch.cuda.current_stream(dev).wait_stream(s_out)
        c1.record()
        barrier()
        return _max_over_ranks(c0.elapsed_time(c1) / args.steps, dev, world)

    h2d_ms, d2h_ms = copy_rate(True), copy_rate(False)
    both_ms = copy_rate_both()
    host_copy = {"h2d_gbs_per_gpu": T * H * 2 / (h2d_ms * 1e-3) / 1e9,
                 "d2h_gbs_per_gpu": T * H * 2 / (d2h_ms * 1e-3) / 1e9, "concurrent_ranks": world,
                 "copy_bound_tokens_per_s": T * world / (max(h2d_ms, d2h_ms) * 1e-3),
                 "both_directions_ms_per_step": both_ms,
                 "copy_bound_both_directions_tokens_per_s": T * world / (both_ms * 1e-3),
                 "note": "all ranks copying 4 MB pinned host buffers at once, no compute (max over ranks); "
                         "both_directions: each rank uploads and downloads 4 MB at once per step, as the e2e "
                         "loop does"}

    # ---------------- parity: one eager step vs the single-GPU forward ----------------
    y_ep = moe(x)
    idx_ep = moe.topk_idx[:T].clone()
    y_ref, idx_ref, _ = ops.moe_forward(x, router, full.gate_up, full.down, K_TOP, return_routing=True)
    parity = _ep_parity(y_ep, y_ref, idx_ep, idx_ref, dev, world)
    parity["device_error_timed"] = int(err_timed)
    e2e_err = _max_over_ranks(float((y_e2e.float() - y_ref.float()).abs().max() / y_ref.float().abs().max()),
                              dev, world)
    parity["e2e_max_rel_err"] = e2e_err
    parity["ok"] = bool(parity["ok"] and err_timed == 0 and e2e_err <= MAX_REL_ERR)
    parity["reference"] = "qmoe_moe_forward on one GPU, same tokens, full expert set (routing bit-exact)"

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights ~N(0,0.02), activations ~N(0,1))",
        "config": {"workload": f"qwen3-moe sparse block, expert parallel, {T} tokens per GPU",
                   "tokens_per_gpu": T, "hidden": H, "experts": E, "experts_per_gpu": el, "top_k": K_TOP,
                   "moe_intermediate": I_MOE, "parallelism": f"ep{world}",
                   "l2": "inputs larger than L2: expert weights and exchange buffers streamed per step"},
        "value_per_gpu": value / world,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2,
                "api": "PeerExpertParallelMoE step (CUDA graph replay of its forward, one graph and input/output "
                       "per parity), pinned host in/out, uploads and downloads on their own streams",
                "host_copy": host_copy},
        "gpu_launches": moe.launches_per_step(T) * args.steps,
        "stage_us_rank0": stage_us,
        "parity": parity,
        "roofline": {"bound": "tensor", "kernel": "moe_fused_kernel<return> (this rank's experts, rank 0)",
                     "achieved": exp_tflops, "peak": tf_burst, "unit": "TFLOP/s", "frac": exp_tflops / tf_burst,
                     "peak_kind": peak_kind, "traffic": None, "kernel_us": experts_us,
                     "algorithmic_flops_per_launch": flops_rank, "rows_received": recv_rows,
                     "step_tflops": step_tflops, "step_tensor_frac": step_tflops / tf_burst,
                     "step_tensor_frac_of_sustained": step_tflops / tf_sust if tf_sust else None,
                     "nvlink": {"bytes_out_per_step": nvl_out, "bytes_in_per_step": nvl_in,
                                "link_gbs_reference": nvl_gbs_ref,
                                "dispatch_token_rows_out": tok_sent_remote,
                                "dispatch_rows_undeduplicated": remote_sent,
                                "dispatch_gbs": (tok_sent_remote * H * 2) / (stage_us["dispatch"] * 1e-6) / 1e9},
                     "step_target_us": target_us,
                     "step_target": {"tensor_us": t_tensor_us, "nvlink_us": t_nvlink_us, "weights_us": t_weights_us},
                     "step_frac_of_target": target_us / (ms_per_step * 1e3)},
        "clocks": clocks,
    }
    del full
    torch.cuda.empty_cache()
    extras = {}
    if not args.no_extras and _want(args, "cfg4"):
        extras["cfg4_zipf_T16384"] = ep_zipf_line(cfg, dev, world, rank, tf_burst)
    if not args.no_extras and _want(args, "cfg3"):
        torch.cuda.empty_cache()
        extras["cfg3_prefill_8x2048_48l"] = ep_prefill_model_line(cfg, dev, world, rank)
    if extras:
        line["extras"] = extras
    ok = parity["ok"] and all(v.get("parity", {}).get("ok", True) for v in extras.values())
    if rank == 0:
        print(json.dumps(line))
    dist.barrier()
    moe.close()
    dist.barrier()
    dist.destroy_process_group()
    if not ok:
        print("expert-parallel parity failed", file=sys.stderr)
        return 1
    return 0


def ep_zipf_line(cfg, dev, world, rank, tf_burst, T_total=16384):
    """Config 4 under expert parallelism: the 16,384-token Zipf-skewed block
    split over the ranks (T_total / world tokens each), the experts sharded."""
    import torch
    import torch.distributed as dist

    from nki_moe_7013_b200 import ops
    from nki_moe_7013_b200.ep import PeerExpertParallelMoE
    from nki_moe_7013_b200.moe import MoEWeights
    from nki_moe_7013_b200.synth import normal_bf16_device, zipf_expert_bias

    el = E // world
    T = T_total // world
    full = MoEWeights.random(cfg, seed=0, device=dev)
    local = MoEWeights(full.router, full.gate_up[rank * el:(rank + 1) * el].clone(),
                       full.down[rank * el:(rank + 1) * el].clone())
    bias = zipf_expert_bias(0, E).to(dev)
    moe = PeerExpertParallelMoE(cfg, full.router, local, max_tokens=T)
    moe.router_bias = bias
    x = normal_bf16_device(4242, (T_total, H), 1.0, dev)[rank * T:(rank + 1) * T].contiguous()
    for _ in range(2):
        moe(x)
    torch.cuda.synchronize()
    dist.barrier()
    n = 10
    e0, e1 = _events(2)
    e0.record()
    for _ in range(n):
        moe(x)
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1) / n, dev, world)
    ns = len(PeerExpertParallelMoE.STAGES)
    evs = [_events(ns + 1) for _ in range(n)]
    for i in range(n):
        moe(x, events=evs[i])
    torch.cuda.synchronize()
    stage_us = {name: round(statistics.median(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(n)) * 1e3, 1)
                for j, name in enumerate(PeerExpertParallelMoE.STAGES)}
    rows = torch.tensor([int(moe.recv_rows.item())], dtype=torch.int64, device=dev)
    all_rows = [torch.zeros_like(rows) for _ in range(world)]
    dist.all_gather(all_rows, rows)
    y_ep = moe(x)
    idx_ep = moe.topk_idx[:T].clone()
    y_ref, idx_ref, _ = ops.moe_forward(x, full.router, full.gate_up, full.down, K_TOP, bias=bias,
                                        return_routing=True)
    parity = _ep_parity(y_ep, y_ref, idx_ep, idx_ref, dev, world)
    dist.barrier()
    moe.close()
    flops = T_total * 6 * K_TOP * H * I_MOE
    return {"tokens": T_total, "tokens_per_gpu": T, "ms_per_layer": round(ms, 3),
            "tokens_per_s": T_total / (ms * 1e-3), "stage_us_rank0": stage_us,
            "rows_received_per_rank": [int(r.item()) for r in all_rows],
            "expert_gemm_tflops_per_gpu": flops / world / (ms * 1e-3) / 1e12,
            "step_tensor_frac": flops / world / (ms * 1e-3) / 1e12 / tf_burst,
            "parity": parity,
            "note": "eager steps (device time max over ranks); the hottest rank bounds the step"}


def ep_prefill_model_line(cfg, dev, world, rank):
    """Config 3 under expert parallelism, with parity of a 2-layer cut
    against the same model on one GPU (each rank checks its own sequences)."""
    import torch
    import torch.distributed as dist

    from nki_moe_7013_b200 import _C
    from nki_moe_7013_b200.model import Qwen3MoeModel, routing_agreement

    line, model, ids_local = prefill_model_line(cfg, dev, world, rank)
    # parity: hidden states after 2 layers, EP model vs the 2-layer model on
    # one GPU.  Layer 1 sees identical inputs (routing bit-exact); the EP
    # combine rounds each weighted expert row to bf16 before summing, so a
    # near-tie token may pick another 8th expert in layer 2: the hidden
    # states are compared on the tokens routed alike in both layers.
    mi_ep = []
    h_ep, _ = model.hidden_states(ids_local, model.new_caches(ids_local.shape[0], ids_local.shape[1]),
                                  num_layers=2, moe_inputs=mi_ep)
    r_ep = model.routing_of(mi_ep)
    torch.cuda.synchronize()
    dist.barrier()
    model.close()
    del model, mi_ep
    torch.cuda.empty_cache()
    ref = Qwen3MoeModel(cfg, num_layers=2, device=dev, seed=3)
    mi_ref = []
    h_ref, _ = ref.hidden_states(ids_local, moe_inputs=mi_ref)
    r_ref = ref.routing_of(mi_ref, with_logits=True)
    same1 = bool(torch.equal(r_ep[0], r_ref[0][0]))
    ag = routing_agreement(r_ep[1], r_ref[1][0], r_ref[1][1], K_TOP)
    agree = ag["agree"] & (r_ep[0] == r_ref[0][0]).all(1)
    hv_ep = h_ep.reshape(-1, H).float()
    hv_ref = h_ref.reshape(-1, H).float()
    err = float((hv_ep[agree] - hv_ref[agree]).abs().max() / hv_ref.abs().max())
    frac = float(agree.float().mean())
    code = float(_C.device_error())
    err = _max_over_ranks(err, dev, world)
    code = int(_max_over_ranks(code, dev, world))
    frac = -_max_over_ranks(-frac, dev, world)
    gap = _max_over_ranks(ag["max_flip_gap"], dev, world)
    same1 = _max_over_ranks(0.0 if same1 else 1.0, dev, world) == 0.0
    line["parity"] = {"cut_layers": 2, "layer1_routing_equal": same1, "layer2_routing_agree_frac": frac,
                      "layer2_max_flip_logit_gap": gap, "layer2_median_logit_gap": ag["median_gap"],
                      "max_rel_err_on_tokens_routed_alike": err, "device_error": code, "tolerance": MAX_REL_ERR,
                      "ok": bool(same1 and frac >= 0.9 and gap <= FLIP_GAP_MAX and err <= MAX_REL_ERR and code == 0),
                      "reference": "the same seeded model, 2 layers, on one GPU, same sequences",
                      "rule": "layer-1 routing bit-exact; every layer-2 routing difference a near tie (k-th vs "
                              "(k+1)-th fp32 logit within layer2_max_flip_logit_gap <= %g) and >= 90 %% of tokens "
                              "routed alike; hidden states of those tokens within the tolerance" % FLIP_GAP_MAX}
    del ref
    torch.cuda.empty_cache()
    return line


def run_decode_model_only(args):
    import torch

    from nki_moe_7013_b200.config import Qwen3MoeConfig
    from nki_moe_7013_b200.model import DecodeSession, Qwen3MoeModel

    dev = torch.device("cuda", 0)
    model = Qwen3MoeModel(Qwen3MoeConfig(), num_layers=args.decode_model, device=dev, seed=1)
    sess = DecodeSession(model, args.tokens, context=4096, max_new=args.steps + args.warmup + 4, seed=1)
    sess.capture()
    for _ in range(args.warmup):
        sess.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        sess.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    print(json.dumps({"decode_model_layers": args.decode_model, "batch": args.tokens, "ms_per_step": ms,
                      "us_per_layer": ms * 1e3 / args.decode_model}))
    return 0


def run_prefill_attention_only(args):
    """The flash-prefill kernel alone on seeded q / K / V (~N(0,1) bf16), causal
    over each sequence from an empty cache: device time per launch and the
    causal FLOP rate against the measured bf16 peak."""
    import torch

    from nki_moe_7013_b200 import _C, ops

    B, S = (int(v) for v in args.prefill_attention.lower().split("x"))
    nh, nkv, hd = 32, 4, 128
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    k = torch.randn(B, nkv, S, hd, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(B, nkv, S, hd, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B * S, nh, hd, generator=g, device=dev).to(torch.bfloat16)
    qs = torch.zeros(B, dtype=torch.int32, device=dev)
    for _ in range(max(args.warmup, 1)):
        ops.attention_prefill(q, k, v, qs, B, S)
    torch.cuda.synchronize()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(args.steps):
        ops.attention_prefill(q, k, v, qs, B, S)
    e1.record()
    torch.cuda.synchronize()
    if _C.device_error():
        raise RuntimeError("device error word set")
    us = e0.elapsed_time(e1) / max(args.steps, 1) * 1e3
    flops = B * 4 * hd * nh * S * (S + 1) // 2
    _, tf_burst, _, _ = load_peaks()
    print(json.dumps({"prefill_attention": f"{B}x{S}", "us_per_launch": us, "causal_flops": flops,
                      "tflops": flops / (us * 1e-6) / 1e12, "tensor_frac": flops / (us * 1e-6) / 1e12 / tf_burst}))
    return 0


def main():
    args = parse_args()
    if args.prefill_attention:
        return run_prefill_attention_only(args)
    if args.decode_model:
        return run_decode_model_only(args)
    if args.impl == "reference":
        return run_reference(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_ours_ep(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
