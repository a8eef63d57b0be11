#!/usr/bin/env python
"""Benchmark of the B200 MoE layer of Qwen3.6-35B-A3B (lightreason edge35b).

Metric: MoE-layer us/step at decode, tokens/s at prefill, and
the fraction of the HBM / tensor-core roofline.  The JSON line's `value` is
whole-job throughput in tokens/s; `ms_per_step` gives the step time.

Default workload (no flags): BASELINE configs[1], one MoE layer at the
speculative-verify width T=16 with seeded synthetic weights and N(0,1)
activations.
  * value: device-timed steps with every input already resident in HBM;
  * e2e:   the same step through the C ABI (moe_layer_forward) with HOST
           buffers -- activations copied in from pinned memory and the result
           read back each step, and all 256 experts resident in pinned host
           RAM, of which only the union of selected experts is gathered into
           HBM slots every step (configs[1]'s gather + compute);
  * roofline: the dominant kernel of `value`, from CUDA events recorded at the
           stage boundaries inside moe_layer_forward during the timed steps;
  * cpu_baseline: the reference's own CPU path (edge35b/cpu_experts.c built from
           the reference sources into oracle/_ref, torch-CPU router / shared
           expert / ordered combine) on a bounded sample of the same workload.
L2 is flushed between timed steps by reading a 256 MiB buffer (twice the L2),
outside each step's CUDA-event window.

--impl reference times that CPU path alone as the reference arm.
--gpus N > 1 (under torchrun) runs BASELINE configs[4], the expert-parallel
layer: 512 tokens per rank, 256/N experts per rank, NCCL all-to-all dispatch
and combine, step time = max over ranks of the device-timed steps.  The same
workload runs on one GPU with --config 4.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from lightreason_b200 import synthetic as S  # noqa: E402

HIDDEN, INNER, EXPERTS, TOP_K = S.HIDDEN, S.INNER, S.EXPERTS, S.TOP_K
GATE_UP_BYTES = 2 * INNER * HIDDEN * 2       # 4,194,304 B per expert
DOWN_BYTES = HIDDEN * INNER * 2              # 2,097,152 B per expert
EXPERT_BYTES = GATE_UP_BYTES + DOWN_BYTES    # 6,291,456 B
STAGES = ("router", "route", "gather", "xs", "experts", "combine", "unused")
KERNEL_NAMES = {"router": "router_split_kernel (T <= 16) | router_tc_kernel",
                "route": "route_decode_kernel (T <= 16) | router_select+permute+grouped_plan kernels",
                "gather": "stage_experts_kernel", "xs": "gather_tokens_kernel (T > 64)",
                "experts": "swiglu_grouped_kernel (tcgen05 gate/up + down; + token gather and combine at T <= 64)",
                "combine": "combine_kernel (T > 64)", "unused": "-"}
# up to this width the layer runs its experts as one fused_decode_kernel
# (gate/up, down and the ordered combine in one persistent launch)
FUSED_DECODE_MAX_TOKENS = 2


def kernel_name(stage: str, tokens: int) -> str:
    if stage == "experts" and tokens <= FUSED_DECODE_MAX_TOKENS:
        return "fused_decode_kernel (routing, gate/up, down, ordered combine in one persistent launch, T <= 2)"
    return KERNEL_NAMES[stage]


def launches_per_step(tokens: int) -> int:
    """Kernels of one moe_layer_forward call with HBM-resident experts."""
    if tokens <= FUSED_DECODE_MAX_TOKENS:
        return 2  # router_split, fused_decode (which selects and plans in every CTA)
    if tokens <= 16:
        return 3  # router_split, route_decode, grouped (gathers and combines itself)
    routes = tokens * TOP_K
    permute = 1 if routes <= 2048 else 3  # one-CTA sort, or count + column scan + place
    if tokens <= 64:
        return 4 + permute  # router_tc, router_select, permute, grouped_plan, grouped
    return 6 + permute  # router_tc, router_select, permute, grouped_plan, gather_tokens, grouped, combine

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the dominant kernel, from the ncu captures summarised under profiles/.
PROFILED_TRAFFIC = {
    0: (57_046_528, "profiles/launches_layer_config0_T1.md (fused_decode_kernel)"),
    1: (454_122_240, "profiles/swiglu_grouped_kernel_T16_config1.md"),
    3: (2_062_540_000, "profiles/launches_layer_config3_T4096.md"),
}

CACHE_SLOTS = 128  # experts the e2e_cached variant keeps in HBM (half of the bank, ~0.8 GB)

CONFIGS = {
    0: dict(tokens=1, bias="normal", workload="config0: one MoE layer, decode T=1"),
    2: dict(tokens=64, bias="zipf", layers=40,
            workload="config2: 40-layer MoE stack, decode B=64 tokens per step, all experts HBM-resident"),
    1: dict(tokens=16, bias="normal",
            workload="config1: one MoE layer, speculative-verify width T=16; experts in pinned host RAM (e2e)"),
    3: dict(tokens=4096, bias="zipf", workload="config3: one MoE layer, prefill T=4096, Zipf(1.1) routing"),
    4: dict(tokens=512, bias="zipf", workload="config4: expert-parallel MoE layer, 512 tokens per GPU, experts "
                                               "sharded evenly over the ranks, NCCL all-to-all dispatch/combine"),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.15)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def to_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


# ------------------------------------------------------------ our arm ---

def build_layer(cfg, dev, seed):
    from lightreason_b200 import native

    w = S.layer_weights(seed, bias=cfg["bias"])
    gu, dn = w.stacked()
    d = lambda a: to_dev(a, dev)  # noqa: E731
    sh = [d(w.sh_gate), d(w.sh_up), d(w.sh_down), d(w.sh_gate_w)]
    bias = torch.from_numpy(w.bias).to(dev)
    router = d(w.router)
    hbm = native.Layer(router=router, gate_up=d(gu), down=d(dn), bias=bias, shared_gate=sh[0], shared_up=sh[1],
                       shared_down=sh[2], shared_gate_w=sh[3])
    host = cached = None
    if cfg.get("e2e_host_experts", True):
        # all experts in pinned host RAM in the packed BF16 layout
        # (the lossless row codec the reference streams over PCIe)
        banks = native.PackedHostBanks(gu, dn, dev)
        host = native.Layer(router=router, bias=bias, shared_gate=sh[0], shared_up=sh[1], shared_down=sh[2],
                            shared_gate_w=sh[3], host_packed=banks)
        # the same banks behind a device expert cache of CACHE_SLOTS experts
        cached = native.Layer(router=router, bias=bias, shared_gate=sh[0], shared_up=sh[1], shared_down=sh[2],
                              shared_gate_w=sh[3], host_packed=banks,
                              cache_slots=max(CACHE_SLOTS, min(EXPERTS, cfg["tokens"] * TOP_K)))
    return w, gu, dn, hbm, host, cached


def timed_steps(run_step, steps, warmup, flush, world, stage_events=None):
    """Per-step CUDA-event timing with an L2 flush outside each step window.

    Each timed step is one CUDA-graph replay (captured beforehand, with its own
    step and stage events inside the graph), so the window holds device work
    only; the flush is launched eagerly between replays."""
    for i in range(warmup):
        flush()
        run_step(i, None)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    # stage_events: indices of the moe_layer_forward stage boundaries to record
    # (each external event node costs a few microseconds, so the step-time
    # loop records none and the roofline loop only brackets one kernel)
    stg = None
    if stage_events:
        stg = [[torch.cuda.Event(enable_timing=True) if j in stage_events else None for j in range(8)]
               for _ in range(steps)]
        for row in stg:
            for e in row:
                if e is not None:
                    e.record()  # create the CUDA events before capture
    graphs = []
    for i in range(steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_step(warmup + i, stg[i] if stg else None)
        graphs.append(g)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        flush()
        ev[i][0].record()
        graphs[i].replay()
        ev[i][1].record()
    torch.cuda.synchronize()
    barrier(world)
    wall = time.perf_counter() - t0
    ms = [s.elapsed_time(e) for s, e in ev]
    stage_ms = None
    if stg:
        stage_ms = {name: [row[j].elapsed_time(row[j + 1]) for row in stg] for j, name in enumerate(STAGES)
                    if row_has(stg, j) and row_has(stg, j + 1)}
    return ms, stage_ms, wall


def row_has(stg, j):
    return all(row[j] is not None for row in stg)


def cpu_reference_layer(w, gu, dn, x_bits, threads):
    """The reference's CPU implementation of one layer step on host cores:
    torch-CPU router (modeling_qwen3_5_moe.py:762-770 + bias) and shared expert
    (:698-711, :788), edge35b/cpu_experts.c expert_block_rows for T <= 16
    (cpu_experts.c:74-105, as edge35b/block_experts.py:52-86 binds it) or the
    eager expert loop (:727-751) beyond, and the ordered BF16 combine
    (edge35b/cpu_route.py:66-68)."""
    from oracle import oracle as O

    F = torch.nn.functional
    torch.set_num_threads(threads)
    t_bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    x = t_bf(x_bits)
    router, sg, su, sd, sgw = (t_bf(a) for a in (w.router, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w))
    bias = torch.from_numpy(w.bias)
    with torch.no_grad():
        logits = F.linear(x, router)
        probs = F.softmax(logits.float() + bias, dim=-1)
        top_v, top_i = torch.topk(probs, TOP_K, dim=-1)
        scores = (top_v / top_v.sum(-1, keepdim=True)).to(torch.bfloat16)
        shared = F.linear(F.silu(F.linear(x, sg)) * F.linear(x, su), sd)
        gate = torch.sigmoid(F.linear(x, sgw.reshape(1, -1)))
        result = torch.zeros_like(x)
        tokens = x.shape[0]
        ids = top_i.numpy()
        pairs = [(int(ids[t, s]), s, t) for s in range(TOP_K) for t in range(tokens)]
        pairs.sort(key=lambda p: p[0])
        if tokens <= 16 and O.ref_experts_lib() is not None:
            y = O.ref_expert_block_rows(x_bits, [gu[e] for e, _, _ in pairs], [dn[e] for e, _, _ in pairs],
                                        np.array([t for _, _, t in pairs], dtype=np.int32), threads=threads)
            yt = t_bf(y)
            for i, (e, s, t) in enumerate(pairs):
                result[t].add_(yt[i] * scores[t, s])
        else:
            for e in sorted(set(e for e, _, _ in pairs)):
                sel = [(s, t) for ee, s, t in pairs if ee == e]
                tok = torch.tensor([t for _, t in sel])
                slot = torch.tensor([s for s, _ in sel])
                g, u = F.linear(x[tok], t_bf(gu[e])).chunk(2, dim=-1)
                cur = F.linear(F.silu(g) * u, t_bf(dn[e])) * scores[tok, slot, None]
                result.index_add_(0, tok, cur.to(result.dtype))
        out = result + gate * shared
    return out


def cpu_baseline(cfg, w, gu, dn, seed, budget_s=15.0):
    from oracle import oracle as O

    threads = len(os.sched_getaffinity(0))
    tokens = cfg["tokens"]
    sample_tokens = tokens if tokens <= 16 else 256
    kind = "reference" if (sample_tokens <= 16 and O.ref_experts_lib() is not None) else "port"
    xs = [S.hidden_states(seed + 1000 + i, sample_tokens) for i in range(4)]
    cpu_reference_layer(w, gu, dn, xs[0], threads)          # warm-up
    times, t_start, i = [], time.perf_counter(), 0
    while (time.perf_counter() - t_start < budget_s and i < 50) or i < 2:
        t = time.perf_counter()
        cpu_reference_layer(w, gu, dn, xs[i % len(xs)], threads)
        times.append(time.perf_counter() - t)
        i += 1
    step_s = statistics.median(times)
    sample = (f"{len(times)} steps of {sample_tokens} tokens through the reference CPU layer "
              f"(cpu_experts.c expert_block_rows + torch-CPU router/shared/combine)" if kind == "reference" else
              f"{len(times)} steps of {sample_tokens} tokens through the eager torch-CPU expert loop")
    return {"value": sample_tokens / step_s, "unit": "tokens/s", "cores": threads, "kind": kind, "sample": sample,
            "ms_per_step": step_s * 1e3}


def run_ours(args, cfg, world, rank, local):
    from lightreason_b200 import native

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    native.device_check(local)
    hbm_peak, tensor_peak, peak_src = peaks()
    tokens = cfg["tokens"]
    seed = 1 + rank
    t_setup = time.perf_counter()
    w, gu, dn, hbm, host, cached = build_layer(cfg, dev, seed)
    pool = 16
    xs_np = [S.hidden_states(seed, tokens, step=i) for i in range(pool)]
    xs = [to_dev(a, dev) for a in xs_np]
    xs_host = [torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).pin_memory() for a in xs_np]
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
    out_host = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory()
    idx_buf = [torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev) for _ in range(pool)]
    # L2 flush between steps: read a 256 MiB buffer (twice the L2).  Reading
    # evicts every line without leaving ~126 MB of dirty lines behind, whose
    # write-back would otherwise land inside the next timed step.
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    flush_out = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        torch.sum(flush_buf, 0, out=flush_out)
    log(f"[bench] setup {time.perf_counter() - t_setup:.1f}s, tokens={tokens}")

    def hbm_step(i, stage):
        hbm(xs[i % pool], out=out, idx_out=idx_buf[i % pool], stage_events=stage)

    xin = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)

    def e2e_step(i, stage):
        xin.copy_(xs_host[i % pool], non_blocking=True)
        host(xin, out=out, stage_events=stage)
        out_host.copy_(out, non_blocking=True)

    def e2e_cached_step(i, stage):
        xin.copy_(xs_host[i % pool], non_blocking=True)
        cached(xin, out=out, stage_events=stage)
        out_host.copy_(out, non_blocking=True)

    sampler = ClockSampler(local)
    with sampler:
        # step time: no stage events inside the steps
        ms, _, wall = timed_steps(hbm_step, args.steps, args.warmup, flush, world)
        # dominant-kernel time: events only around the expert kernel (stage 4 -> 5)
        _, kernel_ms, _ = timed_steps(hbm_step, args.steps, args.warmup, flush, world, stage_events=(4, 5))
        # full stage breakdown (informational; every boundary recorded)
        _, stage_ms, _ = timed_steps(hbm_step, args.steps, args.warmup, flush, world,
                                     stage_events=tuple(range(8)))
        e2e_ms = None
        if host is not None:
            e2e_ms, _, _ = timed_steps(e2e_step, args.steps, args.warmup, flush, world)
            _, e2e_stage, _ = timed_steps(e2e_step, args.steps, args.warmup, flush, world, stage_events=(2, 3))
            cache_before = cached.cache_stats()
            e2e_cached_ms, _, _ = timed_steps(e2e_cached_step, args.steps, args.warmup, flush, world)
            cache_after = cached.cache_stats()
    clocks = sampler.summary()

    total_ms = dist_max(sum(ms), world)
    value = world * tokens * args.steps / (total_ms / 1e3)
    # routing actually realised in the timed steps
    used = [(args.warmup + i) % pool for i in range(args.steps)]
    u_per_step = [len(set(idx_buf[j].cpu().numpy().reshape(-1).tolist())) for j in used]
    u_mean = float(np.mean(u_per_step))
    routes = tokens * TOP_K
    # algorithmic bytes per launch of each expert kernel (groups = U routed + shared)
    rows = routes + tokens
    fused = FUSED_DECODE_MAX_TOKENS < tokens <= 64   # the grouped kernel runs the combine itself at decode widths
    combine_bytes = rows * HIDDEN * 2 + tokens * HIDDEN * 2 + routes * 6
    if tokens <= FUSED_DECODE_MAX_TOKENS:
        # fused_decode_kernel: every selected expert's weights (+ shared) once,
        # the router partials in, the token rows in, activations out and back
        # in, the layer output out (per-route outputs stay in shared memory)
        expert_algo = [(u + 1) * EXPERT_BYTES + 4 * tokens * (EXPERTS + 1) * 4 + 2 * tokens * HIDDEN * 2
                       + 2 * rows * INNER * 2 for u in u_per_step]
    else:
        # grouped kernel: every selected expert's weights (+ shared) once, the
        # routed token rows in, activations out and back in, per-route outputs
        # out (+ the combine at decode widths: per-route outputs read back, the
        # layer output written)
        expert_algo = [(u + 1) * EXPERT_BYTES + rows * HIDDEN * 2 + 2 * rows * INNER * 2 + rows * HIDDEN * 2
                       + (combine_bytes if fused else 0) for u in u_per_step]
    algo = {
        "experts": expert_algo,
        "combine": [combine_bytes] * len(used),
        "router": [EXPERTS * HIDDEN * 2 + HIDDEN * 2 + tokens * HIDDEN * 2 + tokens * EXPERTS * 2] * len(used),
    }
    totals = {k: sum(v) for k, v in stage_ms.items()}
    dominant = max(totals, key=totals.get)
    if dominant == "experts":
        dur_ms = statistics.mean(kernel_ms["experts"])
    else:
        dur_ms = statistics.mean(stage_ms[dominant])
    bytes_per_launch = statistics.mean(algo.get(dominant, [0]))
    achieved = bytes_per_launch / (dur_ms / 1e3) / 1e9
    layer_bytes = [u * EXPERT_BYTES + EXPERT_BYTES + EXPERTS * HIDDEN * 2 + HIDDEN * 2 + tokens * HIDDEN * 4
                   for u in u_per_step]
    layer_gbs = statistics.mean(b / (m / 1e3) / 1e9 for b, m in zip(layer_bytes, ms))
    n_launches = launches_per_step(tokens)
    result = {
        "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "us_per_step": round(1e3 * total_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations, N(0,0.5) router bias)",
        "config": {"workload": cfg["workload"], "tokens_per_step": tokens, "hidden": HIDDEN, "inner": INNER,
                   "experts": EXPERTS, "top_k": TOP_K, "shared_expert": True,
                   "distinct_experts_per_step": round(u_mean, 2),
                   "parallelism": "single-gpu" if world == 1 else f"replicas{world}",
                   "l2": "flushed between timed steps by reading a 256 MiB buffer, outside each step's event window"},
        "roofline": {"bound": "hbm", "kernel": kernel_name(dominant, tokens), "achieved": round(achieved, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else
                     "fallback 6650 GB/s",
                     "traffic": PROFILED_TRAFFIC.get(args.config, (None, None))[0] if dominant == "experts" else None,
                     "traffic_source": PROFILED_TRAFFIC.get(args.config, (None, None))[1],
                     "algorithmic_bytes_per_launch": int(bytes_per_launch),
                     "launch_us": round(dur_ms * 1e3, 2),
                     "layer_gbs": round(layer_gbs, 1), "layer_frac": round(layer_gbs / hbm_peak, 4),
                     "stage_us_with_event_overhead": {k: round(1e3 * statistics.mean(v), 2)
                                                      for k, v in stage_ms.items()}},
        "gpu_launches": n_launches * args.steps,
        "clocks": clocks,
        "wall_s_timed_loop": round(wall, 4),
    }
    if e2e_ms is not None:
        e2e_total = dist_max(sum(e2e_ms), world)
        banks = host.host_packed
        gathered = statistics.mean(sum(banks.expert_bytes(e) for e in set(idx_buf[j].cpu().numpy().reshape(-1).tolist()))
                                   for j in used)
        result["e2e"] = {
            "value": round(world * tokens * args.steps / (e2e_total / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(e2e_total / args.steps, 4),
            "h2d_bytes_per_step": int(tokens * HIDDEN * 2 + gathered),
            "d2h_bytes_per_step": tokens * HIDDEN * 2,
            "h2d_expert_bytes_per_step": int(gathered),
            "gather_us": round(1e3 * statistics.mean(e2e_stage["gather"]), 2),
            "gather_gbs": round(gathered / (statistics.mean(e2e_stage["gather"]) / 1e3) / 1e9, 2),
            "path": "moe_layer_forward with host_descriptors (pinned banks in the lossless row codec, decoded "
                    "in registers into HBM slots), x H2D + out D2H per step",
        }
        uses = cache_after["uses"] - cache_before["uses"]
        misses = cache_after["misses"] - cache_before["misses"]
        e2e_cached_total = dist_max(sum(e2e_cached_ms), world)
        result["e2e_cached"] = {
            "value": round(world * tokens * args.steps / (e2e_cached_total / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(e2e_cached_total / args.steps, 4), "cache_slots": cached.cache_slots,
            "hit_rate": round((uses - misses) / uses, 4) if uses else None,
            "path": f"as e2e, with a device expert cache (LRU over {cached.cache_slots} HBM slots, the B200 form "
                    "of the reference's cached ExpertPool mode): only missing experts cross the host link",
        }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg, w, gu, dn, seed)
    return result


def run_ep(args, cfg, world, rank, local):
    """one expert-parallel step per timed step.

    transport "p2p" (default on N > 1 GPUs): the NVLink peer-memory exchange,
    no host synchronisation, every timed step one CUDA-graph replay; "nccl":
    the all_to_all_single exchange, eager steps (the split sizes are read on
    the host every step).  On one GPU the exchange is a device copy."""
    from lightreason_b200 import native
    from lightreason_b200.expert_parallel import (ExpertParallelLayer, PeerExchange, TorchExchange,
                                                  run_virtual_ranks, shard)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    native.device_check(local)
    hbm_peak, tensor_peak, peak_src = peaks()
    tokens = cfg["tokens"]
    transport = args.transport if world > 1 else "local"
    seed = 4                                   # one layer, the same on every rank
    t_setup = time.perf_counter()
    w = S.layer_weights(seed, bias=cfg["bias"])
    mine = shard(EXPERTS, world, rank)
    d = lambda a: to_dev(a, dev)  # noqa: E731
    gu = torch.empty((len(mine), 2 * INNER, HIDDEN), dtype=torch.bfloat16, device=dev)
    dn = torch.empty((len(mine), HIDDEN, INNER), dtype=torch.bfloat16, device=dev)
    for j, e in enumerate(mine):
        gu[j].copy_(d(S.expert_gate_up(seed, 0, e)))
        dn[j].copy_(d(S.expert_down(seed, 0, e)))
    peer = None
    if transport == "p2p":
        peer = PeerExchange(world=world, rank=rank, tokens=tokens, top_k=TOP_K, hidden=HIDDEN, experts=EXPERTS,
                            device=dev)
        exchange = peer
    else:
        exchange = TorchExchange() if world > 1 else None
    layer = ExpertParallelLayer(router=d(w.router), gate_up=gu, down=dn, shared_gate=d(w.sh_gate),
                                shared_up=d(w.sh_up), shared_down=d(w.sh_down), shared_gate_w=d(w.sh_gate_w),
                                bias=torch.from_numpy(w.bias).to(dev), rank=rank, world=world, tokens=tokens,
                                exchange=exchange)
    del gu, dn
    pool = 8
    xs_np = [S.hidden_states(100 + 17 * rank, tokens, step=i) for i in range(pool)]
    xs = [to_dev(a, dev) for a in xs_np]
    xs_host = [torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).pin_memory() for a in xs_np]
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
    out_host = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory()
    xin = torch.empty_like(out)
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    flush_out = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        torch.sum(flush_buf, 0, out=flush_out)
    log(f"[bench] ep setup {time.perf_counter() - t_setup:.1f}s, rank {rank}/{world}, experts "
        f"{mine.start}..{mine.stop - 1}, transport {transport}")

    def step(x, o, stage=None):
        if world > 1:
            layer(x, out=o, stage_events=stage)
        else:
            run_virtual_ranks([layer], [x], outs=[o], stage_events=stage)

    def loop(kind, stage_idx=None):
        """Eager steps (the NCCL exchange reads its split sizes on the host)."""
        for i in range(args.warmup):
            step(xs[i % pool], out)
        torch.cuda.synchronize()
        barrier(world)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        stg = [[torch.cuda.Event(enable_timing=True) if stage_idx and j in stage_idx else None for j in range(8)]
               for _ in range(args.steps)]
        for i in range(args.steps):
            flush()
            j = (args.warmup + i) % pool
            ev[i][0].record()
            if kind == "e2e":
                xin.copy_(xs_host[j], non_blocking=True)
                step(xin, out, stg[i] if stage_idx else None)
                out_host.copy_(out, non_blocking=True)
            else:
                step(xs[j], out, stg[i] if stage_idx else None)
            ev[i][1].record()
        torch.cuda.synchronize()
        barrier(world)
        ms = [a.elapsed_time(b) for a, b in ev]
        kern = [row[4].elapsed_time(row[5]) for row in stg] if stage_idx else None
        return ms, kern

    sampler = ClockSampler(local)
    with sampler:
        if transport == "p2p":
            def dev_step(i, stage):
                layer(xs[i % pool], out=out, stage_events=stage)

            def e2e_step(i, stage):
                xin.copy_(xs_host[i % pool], non_blocking=True)
                layer(xin, out=out, stage_events=stage)
                out_host.copy_(out, non_blocking=True)
            for i in range(args.warmup):          # buffers and workspaces exist before capture
                dev_step(i, None)
            torch.cuda.synchronize()
            ms, _, _ = timed_steps(dev_step, args.steps, args.warmup, flush, world)
            _, stage_ms, _ = timed_steps(dev_step, args.steps, args.warmup, flush, world, stage_events=(4, 5))
            kern_ms = stage_ms["experts"]
            e2e_ms, _, _ = timed_steps(e2e_step, args.steps, args.warmup, flush, world)
            peer.check()
        else:
            ms, _ = loop("device")
            _, kern_ms = loop("device", stage_idx=(4, 5))
            e2e_ms, _ = loop("e2e")
    clocks = sampler.summary()
    total_ms = dist_max(sum(ms), world)
    e2e_total = dist_max(sum(e2e_ms), world)
    value = world * tokens * args.steps / (total_ms / 1e3)
    # this rank's work in the last timed step
    if transport == "p2p":
        ids = layer.p_route_in[peer.own_rows:, 0].cpu().numpy()
        local_ids = ids[ids >= 0]
        received = int(local_ids.size)
        sent = layer.offsets.cpu().numpy()
        el = EXPERTS // world
        leaving = int(sent[EXPERTS] - (sent[(rank + 1) * el] - sent[rank * el]))
    else:
        m = layer.last_splits if layer.last_splits is not None else [[int(layer.send_counts.sum())]]
        received = sum(m[s][rank] for s in range(world))
        leaving = sum(m[rank][dd] for dd in range(world) if dd != rank)
        local_ids = layer.recv_meta[:received].cpu().numpy()
    u_local = len(set(local_ids.tolist()))
    rows = tokens + received
    kernel_bytes = ((u_local + 1) * EXPERT_BYTES + rows * HIDDEN * 2 + 2 * rows * INNER * 2 + 2 * rows * HIDDEN * 2
                    + rows * HIDDEN * 2)
    kernel_flops = rows * 2 * (2 * INNER * HIDDEN + HIDDEN * INNER)
    dur_ms = statistics.mean(kern_ms)          # this rank's launches, with this rank's bytes
    gbs = kernel_bytes / (dur_ms / 1e3) / 1e9
    tfs = kernel_flops / (dur_ms / 1e3) / 1e12
    t_hbm, t_tc = kernel_bytes / (hbm_peak * 1e9), kernel_flops / (tensor_peak * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    achieved, peak, unit = (gbs, hbm_peak, "GB/s") if bound == "hbm" else (tfs, tensor_peak, "TFLOP/s")
    # router tc + select, permute (3 when wide), dispatch, collect, local permute/plan/gather/grouped, return,
    # finish, combine  (NCCL: dispatch, unpack instead of collect/return/finish)
    # router_tc + router_select, permute (count, column scan, place), the
    # exchange's own kernels (p2p: dispatch, collect, return, finish; NCCL and
    # one rank: ep_dispatch, ep_unpack), the local layer in rows mode
    # (permute x3, plan, gather, grouped), the ordered combine
    launches = 16 if transport == "p2p" else 14
    if peer is not None:
        peer.close()
    timing = ("each timed step one CUDA-graph replay of the whole rank step (no host synchronisation), CUDA "
              "events around it, max over ranks of the summed step times" if transport == "p2p" else
              "CUDA events around each whole step on the compute stream (includes the host read of the "
              "all-to-all split sizes), max over ranks of the summed step times")
    return {
        "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "us_per_step": round(1e3 * total_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations, Zipf(1.1) router bias)",
        "config": {"workload": cfg["workload"], "tokens_per_gpu": tokens, "hidden": HIDDEN, "inner": INNER,
                   "experts": EXPERTS, "experts_per_gpu": len(mine), "top_k": TOP_K, "shared_expert": True,
                   "parallelism": f"ep{world}", "transport": transport, "rank0_rows_received": received,
                   "rank0_routes_leaving": leaving, "rank0_nvlink_bytes_per_step": 2 * leaving * HIDDEN * 2,
                   "l2": "flushed between timed steps by reading a 256 MiB buffer, outside each step's event window",
                   "timing": timing},
        "roofline": {"bound": bound, "kernel": "swiglu_grouped_kernel (local experts + shared, rank 0 rows)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
                     "traffic": None, "algorithmic_bytes_per_launch": int(kernel_bytes),
                     "algorithmic_flops_per_launch": int(kernel_flops), "launch_us": round(dur_ms * 1e3, 2),
                     "hbm_frac": round(gbs / hbm_peak, 4), "tensor_frac": round(tfs / tensor_peak, 4)},
        "e2e": {"value": round(world * tokens * args.steps / (e2e_total / 1e3), 2), "unit": "tokens/s",
                "ms_per_step": round(e2e_total / args.steps, 4), "h2d_bytes_per_step": tokens * HIDDEN * 2,
                "d2h_bytes_per_step": tokens * HIDDEN * 2,
                "path": "ExpertParallelLayer.forward per rank, x H2D from pinned memory + out D2H per step"},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }


def run_stack(args, cfg, world, rank, local):
    """the 40-layer stack at decode width, every step one
    CUDA-graph replay of all layers.  Each layer reads its own N(0,1) token
    activations -- the normalised residual stream a MoE block sees; the mixer
    layers between them are out of scope, and feeding one MoE output straight
    into the next would collapse the activations and the routing.  Weights
    are drawn on the GPU from seeded generators (~61 GiB; one layer's parity is
    what the tests check)."""
    from lightreason_b200 import native

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    native.device_check(local)
    hbm_peak, _, peak_src = peaks()
    tokens, n_layers = cfg["tokens"], cfg["layers"]
    t_setup = time.perf_counter()
    layers, u_all = [], []
    for li in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + li)
        rnd = lambda *shape: (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * 0.02).to(  # noqa: E731
            torch.bfloat16)
        gate_up = rnd(EXPERTS, 2 * INNER, HIDDEN)
        down = rnd(EXPERTS, HIDDEN, INNER)
        bias = torch.from_numpy(S.router_bias(7, li, cfg["bias"])).to(dev)
        layers.append(native.Layer(router=rnd(EXPERTS, HIDDEN), gate_up=gate_up, down=down, bias=bias,
                                   shared_gate=rnd(INNER, HIDDEN), shared_up=rnd(INNER, HIDDEN),
                                   shared_down=rnd(HIDDEN, INNER), shared_gate_w=rnd(HIDDEN)))
    xs = [to_dev(S.hidden_states(7 + li, tokens), dev) for li in range(n_layers)]
    acts = [torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev) for _ in range(n_layers)]
    idx = [torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev) for _ in range(n_layers)]
    log(f"[bench] stack setup {time.perf_counter() - t_setup:.1f}s, {n_layers} layers, "
        f"{torch.cuda.memory_allocated(dev) / 2**30:.1f} GiB allocated")

    def stack_step(i, stage):
        for li, layer in enumerate(layers):
            layer(xs[li], out=acts[li], idx_out=idx[li])

    def no_flush():
        pass  # every step streams ~55 GB of weights: far larger than L2
    sampler = ClockSampler(local)
    with sampler:
        ms, _, _ = timed_steps(stack_step, args.steps, args.warmup, no_flush, world)
    clocks = sampler.summary()
    total_ms = dist_max(sum(ms), world)
    u = [len(set(t.cpu().numpy().reshape(-1).tolist())) for t in idx]
    layer_bytes = [(ui + 1) * EXPERT_BYTES + EXPERTS * HIDDEN * 2 + HIDDEN * 2 + tokens * HIDDEN * 4 for ui in u]
    step_ms = total_ms / args.steps
    gbs = sum(layer_bytes) / (step_ms / 1e3) / 1e9
    return {
        "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": round(world * tokens * args.steps / (total_ms / 1e3), 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5),
        "us_per_step": round(step_ms * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded GPU-drawn N(0,0.02) weights, N(0,1) activations, Zipf(1.1) router bias)",
        "config": {"workload": cfg["workload"], "layers": n_layers, "tokens_per_step": tokens, "hidden": HIDDEN,
                   "inner": INNER, "experts": EXPERTS, "top_k": TOP_K, "shared_expert": True,
                   "distinct_experts_per_layer": round(float(np.mean(u)), 1),
                   "l2": "not flushed: every step streams the selected experts of 40 layers (far above L2)",
                   "parallelism": "single-gpu"},
        "roofline": {"bound": "hbm", "kernel": "whole 40-layer step (all kernels)", "achieved": round(gbs, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
                     "traffic": None, "algorithmic_bytes_per_step": int(sum(layer_bytes))},
        "gpu_launches": launches_per_step(tokens) * n_layers * args.steps,
        "clocks": clocks,
    }


def run_profile(args, cfg):
    """--profile N: N eager steps of the HBM-resident layer on one GPU, no CUDA
    graphs and no timing, for a profiler's launch list or kernel capture."""
    from lightreason_b200 import native

    dev = torch.device("cuda", 0)
    native.device_check(0)
    cfg = dict(cfg, e2e_host_experts=False)
    w, gu, dn, hbm, _, _ = build_layer(cfg, dev, 1)
    xs = [to_dev(S.hidden_states(1, cfg["tokens"], step=i), dev) for i in range(min(args.profile, 4))]
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    for i in range(args.profile):
        flush_buf.sum()
        hbm(xs[i % len(xs)])
    torch.cuda.synchronize()
    return {"profile_steps": args.profile, "workload": cfg["workload"], "tokens": cfg["tokens"]}


def run_encode(args):
    """--encode: the device codec encoders over one 35B layer's expert banks
    (gate_up [256, 1024, 2048] + down [256, 2048, 512] BF16, N(0, 0.02) drawn
    on the GPU, 1.5 GiB): row codec plan + pack and tile codec pack per step,
    CUDA events per encoder, inputs far above L2.  Reported as GB/s of BF16
    input; the roofline counts the algorithmic bytes of each encoder (row
    codec: the bank read twice + packed bytes written; tile codec: the bank
    read once + 3/4 of it written + one base byte per tile)."""

    from lightreason_b200 import bf16_expert_codec as codec
    from lightreason_b200 import native

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    native.device_check(0)
    hbm_peak, _, peak_src = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    banks = [(torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * 0.02).to(torch.bfloat16)
             .view(torch.int16) for shape in ((EXPERTS, 2 * INNER, HIDDEN), (EXPERTS, HIDDEN, INNER))]
    L = native.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    row = []
    for bank in banks:
        rows, n = bank.shape[0], bank[0].numel()
        ws = torch.empty(L.moe_rowcodec_workspace_bytes(rows, n), dtype=torch.uint8, device=dev)
        meta = torch.empty((rows, 3), dtype=torch.int64, device=dev)
        total = torch.empty(1, dtype=torch.int64, device=dev)
        native.check(L.moe_rowcodec_plan(bank.data_ptr(), rows, n, meta.data_ptr(), total.data_ptr(), ws.data_ptr(),
                                         ws.numel(), stream), "moe_rowcodec_plan")
        packed = torch.zeros(max(int(total.item()), 16), dtype=torch.uint8, device=dev)
        row.append((bank, rows, n, ws, meta, total, packed))
    tiles = [(bank, bank.numel() // 256, torch.empty((bank.numel() // 256, 384), dtype=torch.uint8, device=dev),
              torch.empty(bank.numel() // 256, dtype=torch.uint8, device=dev)) for bank in banks]
    encoded = torch.zeros(1, dtype=torch.int64, device=dev)

    def row_step():
        for bank, rows, n, ws, meta, total, packed in row:
            native.check(L.moe_rowcodec_plan(bank.data_ptr(), rows, n, meta.data_ptr(), total.data_ptr(),
                                             ws.data_ptr(), ws.numel(), stream), "moe_rowcodec_plan")
            native.check(L.moe_rowcodec_pack(bank.data_ptr(), rows, n, meta.data_ptr(), packed.data_ptr(),
                                             ws.data_ptr(), ws.numel(), stream), "moe_rowcodec_pack")

    def tile_step():
        for bank, nt, packed, bases in tiles:
            native.check(L.moe_tilecodec_pack(bank.data_ptr(), nt, packed.data_ptr(), bases.data_ptr(),
                                              encoded.data_ptr(), stream), "moe_tilecodec_pack")

    def timed(step):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        ms = []
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            b.synchronize()
            ms.append(a.elapsed_time(b))
        return statistics.median(ms)

    with ClockSampler(0) as clk:
        row_ms = timed(row_step)
        tile_ms = timed(tile_step)
    in_bytes = sum(b.numel() * 2 for b in banks)
    packed_bytes = sum(int(r[5].item()) for r in row)
    row_alg = 2 * in_bytes + packed_bytes
    n_tiles = sum(t[1] for t in tiles)
    tile_alg = in_bytes + n_tiles * 384 + n_tiles
    # the host encoder (numpy, all host threads) on 8 experts of the gate_up bank
    host_bank = banks[0][:8].cpu().numpy().view(np.uint16)
    t = time.perf_counter()
    codec.pack_bank(host_bank)
    host_s = time.perf_counter() - t
    threads = min(32, os.cpu_count() or 1)
    plans = [r[4].cpu().tolist() for r in row]
    raw_rows = sum(1 for p in plans for o, _, _ in p if o < 0)
    return {
        "metric": "expert-bank encode throughput (GB/s of BF16 input), row codec",
        "value": round(in_bytes / row_ms / 1e6, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(row_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16", "data": "synthetic",
        "config": {"workload": "one 35B layer's gate_up + down banks (1.5 GiB BF16), device encoders",
                   "l2": "inputs 1.5 GiB, far above L2"},
        "roofline": {"bound": "hbm", "achieved": round(row_alg / row_ms / 1e6, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(row_alg / row_ms / 1e6 / hbm_peak, 4), "traffic": None,
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else
                     "fallback"},
        "tile_codec": {"value": round(in_bytes / tile_ms / 1e6, 2), "unit": "GB/s", "ms_per_step": round(tile_ms, 4),
                       "achieved": round(tile_alg / tile_ms / 1e6, 1),
                       "frac": round(tile_alg / tile_ms / 1e6 / hbm_peak, 4),
                       "encoded_tiles": int(encoded.item()) // (args.warmup + args.steps)},
        "packed_bytes": packed_bytes, "raw_rows": raw_rows,
        "cpu_baseline": {"value": round(host_bank.nbytes / host_s / 1e9, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": "bf16_expert_codec.pack_bank (numpy) on 8 gate_up experts"},
        "gpu_launches": args.steps * (2 * 4 + 2), "clocks": clk.summary(),
    }


def run_reference(args, cfg, world, rank):
    """Reference arm: the reference's CPU implementation on the host cores."""
    if rank != 0:
        return None
    tokens = cfg["tokens"]
    seed = 1
    w = S.layer_weights(seed, bias=cfg["bias"])
    gu, dn = w.stacked()
    threads = len(os.sched_getaffinity(0))
    from oracle import oracle as O

    sample_tokens = tokens if tokens <= 16 else 256
    xs = [S.hidden_states(seed, sample_tokens, step=i) for i in range(8)]
    for i in range(args.warmup):
        cpu_reference_layer(w, gu, dn, xs[i % 8], threads)
    times = []
    for i in range(args.steps):
        t = time.perf_counter()
        cpu_reference_layer(w, gu, dn, xs[i % 8], threads)
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = sample_tokens * args.steps / total
    kind = "reference" if (sample_tokens <= 16 and O.ref_experts_lib() is not None) else "port"
    return {
        "impl": "reference", "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg["workload"], "tokens_per_step": sample_tokens},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{args.steps} steps of {sample_tokens} tokens"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    # The one JSON line goes to the real stdout; anything libraries print there
    # (NCCL's version banner, for one) is sent to stderr instead.
    json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=None,
                    help="BASELINE config: 1 by default on one GPU, 4 (expert parallel) on more")
    ap.add_argument("--tokens", type=int, default=None, help="override the config's tokens per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--transport", choices=("p2p", "nccl"), default="p2p",
                    help="expert-parallel exchange on N > 1 GPUs: NVLink peer memory (default) or NCCL all_to_all")
    ap.add_argument("--encode", action="store_true",
                    help="time the device codec encoders on one layer's expert banks instead of the layer")
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="run N eager layer steps of the config on one GPU (for ncu) and print a short status line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    n = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if args.config is None:
        args.config = 1 if n == 1 else 4
    cfg = dict(CONFIGS[args.config])
    if args.tokens:
        cfg["tokens"] = args.tokens
        cfg["workload"] += f" (tokens overridden to {args.tokens})"
    if args.impl == "reference":
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        res = run_reference(args, cfg, world, rank)
        if res is not None:
            print(json.dumps(res), file=json_out, flush=True)
        return
    if args.profile:
        print(json.dumps(run_profile(args, cfg)), file=json_out, flush=True)
        return
    if args.encode:
        print(json.dumps(run_encode(args)), file=json_out, flush=True)
        return
    world, rank, local = dist_setup()
    try:
        if args.config == 4:
            res = run_ep(args, cfg, world, rank, local)
        elif args.config == 2:
            res = run_stack(args, cfg, world, rank, local)
        else:
            res = run_ours(args, cfg, world, rank, local)
        if rank == 0 and world == 1 and args.config == 4 and not args.no_cpu_baseline:
            w = S.layer_weights(4, bias=cfg["bias"])
            gu, dn = w.stacked()
            res["cpu_baseline"] = cpu_baseline(cfg, w, gu, dn, 4)
        if rank == 0:
            print(json.dumps(res), file=json_out, flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
