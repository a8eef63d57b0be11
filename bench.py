#!/usr/bin/env python
"""Benchmark of the B200 MoE layer of Qwen3.6-35B-A3B (lightreason edge35b).

Metric: MoE-layer us/step at decode, tokens/s at prefill, and
the fraction of the HBM / tensor-core roofline.  The JSON line's `value` is
whole-job throughput in tokens/s; `ms_per_step` gives the step time.

Default workload at every N: BASELINE configs[4], the expert-parallel layer --
512 tokens per GPU, the 256 experts sharded evenly over the N ranks (all of
them on the one rank at N = 1), tokens and their rows exchanged over NVLink
peer memory, step time = max over ranks of the device-timed steps, so the
per-N values form one weak-scaling series.
  * value:    device-timed steps (one CUDA-graph replay per step), inputs in HBM;
  * e2e:      the same step through ExpertParallelLayer.forward with the
              activations copied in from pinned host memory and the result
              copied out, every step;
  * roofline: the expert kernel of the step (CUDA events inside the step);
  * parity:   after the timed steps every rank rebuilds the single-GPU layer
              with all 256 experts and requires its output of the last timed
              step bit for bit, and its expert ids, to equal the
              expert-parallel ones; the ids are also checked against the torch
              CPU router on a token sample (near ties of one BF16 ulp excused
              and counted).  A mismatch makes every rank exit non-zero;
  * ep_stages_us: per-phase times of the rank step (route -- the router,
              which also publishes the own routes to their owners --,
              experts -- the owner's plan and the grouped kernel,
              which pulls the token rows over NVLink and stores the expert
              rows into their senders' memory -- finish, combine) and the
              NVLink bytes the rank moves;
  * cpu_baseline (rank 0, N = 1): the reference's CPU path of the same
              workload on the host cores;
  * configs (N = 1): configs[0..3] as sub-records, each with its step time,
              roofline (HBM and tensor fractions) and CPU baseline:
              config0 (decode T=1), config1_hbm (T=16, experts in HBM),
              config1_e2e (T=16 with all experts in pinned host RAM, the
              union gathered every step, against a measured host-link peak),
              config2 (40-layer decode stack, B=64) and config3 (prefill
              T=4096).
L2 is flushed between timed steps by reading a 256 MiB buffer (twice the L2),
outside each step's CUDA-event window.

--impl reference times the reference's CPU path alone as the reference arm,
with the same inputs, repeat count and statistic (median) as cpu_baseline.
--config 0|1|2|3 runs one of the other workloads as the main line.
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
from concurrent.futures import ThreadPoolExecutor
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
EXPERT_FLOPS_PER_ROW = 2 * (2 * INNER * HIDDEN + HIDDEN * INNER)   # gate/up + down per routed row
STAGES = ("router", "route", "gather", "xs", "experts", "combine", "unused")
KERNEL_NAMES = {"router": "router_split_kernel (T <= 16) | router_tc_kernel",
                "route": "route_decode_kernel (T <= 16) | router_select+permute+grouped_plan kernels",
                "gather": "stage_experts_kernel | stage_row_codec_kernel", "xs": "gather_tokens_kernel (T > 64)",
                "experts": "swiglu_grouped_kernel (tcgen05 gate/up + down; + token gather and combine at T <= 64)",
                "combine": "combine_kernel (T > 64)", "unused": "-"}
# up to this width the layer runs its experts as one fused_decode_kernel
# (gate/up, down and the ordered combine in one persistent launch)
FUSED_DECODE_MAX_TOKENS = 2
CACHE_SLOTS = 128  # experts the e2e_cached variant keeps in HBM (half of the bank, ~0.8 GB)
POOL = 8           # distinct inputs cycled through by the steps of both legs

CONFIGS = {
    0: dict(index=0, tokens=1, bias="normal", seed=1, workload="config0: one MoE layer, decode T=1"),
    1: dict(index=1, tokens=16, bias="normal", seed=1,
            workload="config1: one MoE layer, speculative-verify width T=16 (e2e: experts in pinned host RAM)"),
    2: dict(index=2, tokens=64, bias="zipf", layers=40,
            workload="config2: 40-layer MoE stack, decode B=64 tokens per step, all experts HBM-resident"),
    3: dict(index=3, tokens=4096, bias="zipf", seed=1, cpu_sample=512,
            workload="config3: one MoE layer, prefill T=4096, Zipf(1.1) routing"),
    4: dict(index=4, tokens=512, bias="zipf", seed=4, ep=True,
            workload="config4: expert-parallel MoE layer, 512 tokens per GPU, 256 experts sharded evenly over "
                     "the GPUs, token rows exchanged over NVLink peer memory"),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tensor": float(d["bf16_tflops"]),
                "tensor_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm": 6650.0, "tensor": 1590.0, "tensor_sustained": 1400.0, "source": "fallback"}


def grouped_mode(width: int) -> str:
    """Which grouped kernel layout the library runs at this width (tokens of
    a layer, rows of an expert-parallel owner)."""
    import os

    from lightreason_b200 import native
    if native.lib().moe_grouped_paired(width, INNER, HIDDEN):
        return "CTA pairs (cta_group::2, weights as M = 256)"
    if width > 512 and os.environ.get("LRB_GROUPED_SWAP") != "1":
        return "tokens as M = 128, weights as N = 256"
    return "weights as M = 128, tokens as N"


def profiled_traffic(key: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of a
    kernel from an ncu capture, as recorded in profiles/dram_traffic.json
    (entry: bytes_per_launch, the summary it comes from)."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None, None
    entry = json.loads(p.read_text()).get(key)
    if not entry:
        return None, None
    return int(entry["bytes_per_launch"]), entry["summary"]


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


def dist_all(flag: bool, world: int) -> bool:
    """True on every rank iff `flag` is true on every rank."""
    if world == 1:
        return flag
    import torch.distributed as dist

    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def to_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def pinned(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).pin_memory()


def l2_flusher(dev):
    """Read a 256 MiB buffer (twice the L2).  Reading evicts every line without
    leaving ~126 MB of dirty lines behind, whose write-back would otherwise
    land inside the next timed step."""
    buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    out = torch.empty((), dtype=torch.float32, device=dev)
    return lambda: torch.sum(buf, 0, out=out)


def spread(ms) -> dict:
    a = np.asarray(ms, dtype=np.float64)
    return {"median_ms": round(float(np.median(a)), 5), "p10_ms": round(float(np.percentile(a, 10)), 5),
            "p90_ms": round(float(np.percentile(a, 90)), 5), "min_ms": round(float(a.min()), 5),
            "max_ms": round(float(a.max()), 5), "samples": int(a.size)}


def timed_steps(run_step, steps, warmup, flush, world, n_events=0, event_slots=()):
    """Per-step CUDA-event timing with an L2 flush outside each step window.

    Each timed step is one CUDA-graph replay (captured beforehand, with its own
    step and stage events inside the graph), so the window holds device work
    only; the flush is launched eagerly between replays.  run_step(i, events)
    gets None, or a list of n_events CUDA events (None outside event_slots) to
    record inside the step; each external event node costs a few
    microseconds, so the step-time loop records none.  Returns (step ms, the
    per-step event lists, wall seconds of the timed loop)."""
    for i in range(warmup):
        flush()
        run_step(i, None)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    rows = None
    if n_events:
        # external: an event recorded from Python inside the capture becomes an
        # external event node, which the host can time after a replay
        rows = [[torch.cuda.Event(enable_timing=True, external=True) if j in event_slots else None
                 for j in range(n_events)] for _ in range(steps)]
        for row in rows:
            for e in row:
                if e is not None:
                    e.record()  # create the CUDA events before capture
    graphs = []
    for i in range(steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_step(warmup + i, rows[i] if rows else None)
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
    del graphs
    return [s.elapsed_time(e) for s, e in ev], rows, wall


def pipelined_e2e(step, xs_host, shape, dev, steps, warmup, world, capture=True):
    """ms for `steps` steps through lightreason_b200.pipeline.HostStream: each
    step's input copied host -> device and its output device -> host on side
    streams, overlapped with the neighbouring steps' compute; every copy inside
    the timed window, which is one CUDA-graph replay of all the steps
    (eager when capture=False).  No L2 flush between steps: each step streams
    expert banks larger than L2."""
    from lightreason_b200.pipeline import HostStream

    hs = HostStream(shape, shape, device=dev)
    outs = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    pool = len(xs_host)

    def run(first, n):
        hs.run(step, [xs_host[(first + i) % pool] for i in range(n)], [outs[i % 2] for i in range(n)])
    run(0, warmup)
    torch.cuda.synchronize()
    g = None
    if capture:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run(warmup, steps)
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    if g is not None:
        g.replay()
    else:
        run(warmup, steps)
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    del g
    return a.elapsed_time(b)


def between(rows, a, b):
    """Per-step ms between event slots a and b."""
    return [row[a].elapsed_time(row[b]) for row in rows]


def stage_times(rows, names):
    """{name: per-step ms} for consecutive recorded slots of the layer's stages."""
    out = {}
    for j, name in enumerate(names):
        if j + 1 < len(rows[0]) and rows[0][j] is not None and rows[0][j + 1] is not None:
            out[name] = between(rows, j, j + 1)
    return out


def roofline(kernel: str, bytes_: float, flops: float, dur_ms: float, pk: dict, *, sustained=False,
             traffic=None, traffic_source=None, **extra) -> dict:
    """The kernel's achieved rate against the measured peaks: bound = the
    roofline (HBM or tensor) whose time floor for these bytes and flops is
    larger; both fractions are reported."""
    tensor_peak = pk["tensor_sustained"] if sustained else pk["tensor"]
    gbs = bytes_ / (dur_ms / 1e3) / 1e9
    tfs = flops / (dur_ms / 1e3) / 1e12
    t_hbm, t_tc = bytes_ / (pk["hbm"] * 1e9), flops / (tensor_peak * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    achieved, peak, unit = (gbs, pk["hbm"], "GB/s") if bound == "hbm" else (tfs, tensor_peak, "TFLOP/s")
    src = ("measured (MEASURED_PEAKS.json hbm_gbs / " + ("bf16_tflops_sustained)" if sustained else "bf16_tflops)")
           if pk["source"] == "measured" else "fallback 6650 GB/s, 1590 TFLOP/s")
    r = {"bound": bound, "kernel": kernel, "achieved": round(achieved, 1), "peak": peak, "unit": unit,
         "frac": round(achieved / peak, 4), "peak_source": src, "traffic": traffic,
         "traffic_source": traffic_source, "algorithmic_bytes_per_launch": int(bytes_),
         "algorithmic_flops_per_launch": int(flops), "launch_us": round(dur_ms * 1e3, 2),
         "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm"], 4), "tflops": round(tfs, 1),
         "tensor_frac": round(tfs / tensor_peak, 4)}
    r.update(extra)
    return r


def host_link_peak(dev) -> dict:
    """Pinned host -> HBM copy rate (cudaMemcpyAsync of 256 MiB, best of 5),
    the ceiling of any per-step gather over the host link."""
    n = 256 << 20
    src = torch.empty(n, dtype=torch.uint8).pin_memory()
    dst = torch.empty(n, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(6):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, n / (a.elapsed_time(b) / 1e3) / 1e9)
    return {"h2d_gbs": round(best, 2), "how": "pinned host -> HBM cudaMemcpyAsync of 256 MiB, best of 6"}


# ------------------------------------------------- the reference CPU path ---

def cpu_reference_layer(w, gu, dn, x_bits, threads):
    """The reference's CPU implementation of one layer step on host cores:
    torch-CPU router (modeling_qwen3_5_moe.py:762-770 + bias) and shared expert
    (:698-711, :788), edge35b/cpu_experts.c expert_block_rows for T <= 16
    (cpu_experts.c:74-105, as edge35b/block_experts.py:52-86 binds it) or the
    eager expert loop (:727-751) beyond, and the ordered BF16 combine
    (edge35b/cpu_route.py:66-68).  Returns (out, top-k ids, z = logits + bias)."""
    from oracle import oracle as O

    F = torch.nn.functional
    torch.set_num_threads(threads)
    t_bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    x = t_bf(x_bits)
    router, sg, su, sd, sgw = (t_bf(a) for a in (w.router, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w))
    bias = torch.from_numpy(w.bias) if w.bias is not None else torch.zeros(router.shape[0])
    with torch.no_grad():
        logits = F.linear(x, router)
        z = logits.float() + bias
        probs = F.softmax(z, dim=-1)
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
    return out, ids, z.numpy()


def cpu_kind(tokens: int) -> str:
    from oracle import oracle as O

    return "reference" if (tokens <= 16 and O.ref_experts_lib() is not None) else "port"


def time_cpu_reference(w, gu, dn, xs, steps, warmup, threads=None) -> dict:
    """The reference's CPU layer on the host cores, timed the same way in both
    legs: `warmup` untimed calls, then `steps` timed calls cycling through the
    inputs `xs`; the statistic is the median (the spread is reported)."""
    threads = threads or len(os.sched_getaffinity(0))
    for i in range(warmup):
        cpu_reference_layer(w, gu, dn, xs[i % len(xs)], threads)
    ms = []
    for i in range(steps):
        t = time.perf_counter()
        cpu_reference_layer(w, gu, dn, xs[(warmup + i) % len(xs)], threads)
        ms.append((time.perf_counter() - t) * 1e3)
    tokens = xs[0].shape[0]
    sp = spread(ms)
    kind = cpu_kind(tokens)
    path = ("cpu_experts.c expert_block_rows + torch-CPU router/shared/combine" if kind == "reference" else
            "the eager torch-CPU expert loop + torch-CPU router/shared/combine")
    return {"value": round(tokens / (sp["median_ms"] / 1e3), 2), "unit": "tokens/s", "cores": threads,
            "kind": kind, "ms_per_step": sp["median_ms"], "spread": sp, "tokens_per_step": tokens,
            "sample": f"median of {steps} steps (after {warmup} warm-up) of {tokens} tokens through {path}"}


_BANKS = {}


def host_layer(seed: int, bias: str):
    """(LayerWeights, gate_up [E, 2I, H], down [E, H, I]) on the host; the
    expert banks depend on the seed only (the bias is drawn separately), so
    configs with one seed share one draw."""
    if seed not in _BANKS:
        _BANKS.clear()
        _BANKS[seed] = S.layer_weights(seed).stacked()
    gu, dn = _BANKS[seed]
    return S.layer_weights(seed, bias=bias), gu, dn


def cpu_inputs(cfg):
    """Weights (host) and the input pool of rank 0, shared by the cpu_baseline
    leg and the reference arm."""
    seed = cfg["seed"]
    w, gu, dn = host_layer(seed, cfg["bias"])
    tokens = cfg.get("cpu_sample", cfg["tokens"])
    xs = [S.hidden_states(input_seed(cfg, 0), cfg["tokens"], step=i)[:tokens] for i in range(POOL)]
    return w, gu, dn, xs


def input_seed(cfg, rank: int) -> int:
    return 100 + 17 * rank if cfg.get("ep") else cfg["seed"]


# ------------------------------------------------------- configs 0, 1, 3 ---

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


def layer_algo(tokens, u):
    """Algorithmic bytes and flops of the expert kernel of one layer call with
    u distinct routed experts: every selected expert's weights (+ the shared
    expert) once; the routed token rows in, the activations out and back in
    and the per-route rows out -- at decode widths the kernel also gathers the
    token rows and runs the combine (per-route rows read back, the layer
    output written); the fused decode kernel (T <= 2) reads the router's
    FP32 partials and keeps the per-route rows in shared memory."""
    routes = tokens * TOP_K
    rows = routes + tokens
    combine = rows * HIDDEN * 2 + tokens * HIDDEN * 2 + routes * 6
    if tokens <= FUSED_DECODE_MAX_TOKENS:
        b = (u + 1) * EXPERT_BYTES + 4 * tokens * (EXPERTS + 1) * 4 + 2 * tokens * HIDDEN * 2 + 2 * rows * INNER * 2
    else:
        b = (u + 1) * EXPERT_BYTES + rows * HIDDEN * 2 + 2 * rows * INNER * 2 + rows * HIDDEN * 2
        if tokens <= 64:
            b += combine
    return b, rows * EXPERT_FLOPS_PER_ROW


def layer_bytes(tokens, u):
    """Whole-layer algorithmic bytes: selected experts + shared expert + router
    + shared gate + activations in and out."""
    return u * EXPERT_BYTES + EXPERT_BYTES + EXPERTS * HIDDEN * 2 + HIDDEN * 2 + tokens * HIDDEN * 4


def run_layer(args, cfg, dev, *, with_cpu=True, cpu_steps=None, cpu_warmup=None) -> dict:
    """One MoE layer (configs 0, 1, 3) on one GPU."""
    from lightreason_b200 import native

    pk = peaks()
    tokens, seed = cfg["tokens"], cfg["seed"]
    t_setup = time.perf_counter()
    w, gu, dn = host_layer(seed, cfg["bias"])
    d = lambda a: to_dev(a, dev)  # noqa: E731
    sh = dict(shared_gate=d(w.sh_gate), shared_up=d(w.sh_up), shared_down=d(w.sh_down), shared_gate_w=d(w.sh_gate_w))
    bias = torch.from_numpy(w.bias).to(dev)
    router = d(w.router)
    hbm = native.Layer(router=router, gate_up=d(gu), down=d(dn), bias=bias, **sh)
    host = cached = None
    if cfg.get("host_experts"):
        # all experts in pinned host RAM in the packed BF16 layout
        # (the lossless row codec the reference streams over PCIe)
        banks = native.PackedHostBanks(gu, dn, dev)
        host = native.Layer(router=router, bias=bias, host_packed=banks, **sh)
        # the same banks behind a device expert cache of CACHE_SLOTS experts
        cached = native.Layer(router=router, bias=bias, host_packed=banks,
                              cache_slots=max(CACHE_SLOTS, min(EXPERTS, tokens * TOP_K)), **sh)
    pool = 16
    xs_np = [S.hidden_states(seed, tokens, step=i) for i in range(pool)]
    xs = [to_dev(a, dev) for a in xs_np]
    xs_host = [pinned(a) for a in xs_np]
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
    out_host = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory()
    xin = torch.empty_like(out)
    idx_buf = [torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev) for _ in range(pool)]
    flush = l2_flusher(dev)
    log(f"[bench] {cfg['workload'][:8]} setup {time.perf_counter() - t_setup:.1f}s, tokens={tokens}")

    def hbm_step(i, ev):
        hbm(xs[i % pool], out=out, idx_out=idx_buf[i % pool], stage_events=ev)

    def e2e_step_of(layer):
        def step(i, ev):
            xin.copy_(xs_host[i % pool], non_blocking=True)
            layer(xin, out=out, stage_events=ev)
            out_host.copy_(out, non_blocking=True)
        return step

    e2e_layer = host if host is not None else hbm
    steps, warmup = args.steps, args.warmup
    sampler = ClockSampler(dev.index or 0)
    with sampler:
        ms, _, wall = timed_steps(hbm_step, steps, warmup, flush, 1)
        _, krows, _ = timed_steps(hbm_step, steps, warmup, flush, 1, n_events=8, event_slots=(4, 5))
        _, srows, _ = timed_steps(hbm_step, steps, warmup, flush, 1, n_events=8, event_slots=tuple(range(8)))
        e2e_ms, _, _ = timed_steps(e2e_step_of(e2e_layer), steps, warmup, flush, 1)
        pipe_ms = None
        # overlapped only where a step's working set exceeds L2 (no flush between
        # its steps): from T = 512 a step reads nearly all 256 experts (1.6 GB);
        # at decode widths (57 MB at T = 1) it would sit in the 126 MB L2
        if host is None and tokens >= 512:
            pipe_ms = pipelined_e2e(lambda x, o: hbm(x, out=o), xs_host, (tokens, HIDDEN), dev, steps, warmup, 1)
        e2e_stage = None
        if host is not None:
            _, grows, _ = timed_steps(e2e_step_of(host), steps, warmup, flush, 1, n_events=8, event_slots=(2, 3))
            e2e_stage = between(grows, 2, 3)
            cache_before = cached.cache_stats()
            cached_ms, _, _ = timed_steps(e2e_step_of(cached), steps, warmup, flush, 1)
            cache_after = cached.cache_stats()
    clocks = sampler.summary()
    stage_ms = stage_times(srows, STAGES)
    kernel_ms = between(krows, 4, 5)

    used = [(warmup + i) % pool for i in range(steps)]
    u_per_step = [len(set(idx_buf[j].cpu().numpy().reshape(-1).tolist())) for j in used]
    algo = [layer_algo(tokens, u) for u in u_per_step]
    totals = {k: sum(v) for k, v in stage_ms.items()}
    dominant = max(totals, key=totals.get)
    kname = ("fused_decode_kernel (routing, gate/up, down, ordered combine in one persistent launch, T <= 2)"
             if dominant == "experts" and tokens <= FUSED_DECODE_MAX_TOKENS else KERNEL_NAMES[dominant])
    if dominant == "experts":
        dur = statistics.mean(kernel_ms)
        b = statistics.mean(a[0] for a in algo)
        f = statistics.mean(a[1] for a in algo)
    else:
        dur = statistics.mean(stage_ms[dominant])
        b = EXPERTS * HIDDEN * 2 + tokens * HIDDEN * 2 if dominant == "router" else 0
        f = 2 * tokens * EXPERTS * HIDDEN if dominant == "router" else 0
    key = f"config{cfg['index']}_{'fused_decode' if tokens <= FUSED_DECODE_MAX_TOKENS else 'grouped'}"
    traffic, traffic_src = profiled_traffic(key) if dominant == "experts" else (None, None)
    lb = [layer_bytes(tokens, u) for u in u_per_step]
    layer_gbs = statistics.mean(x / (m / 1e3) / 1e9 for x, m in zip(lb, ms))
    total_ms = sum(ms)
    rec = {
        "workload": cfg["workload"], "value": round(tokens * steps / (total_ms / 1e3), 2), "unit": "tokens/s",
        "ms_per_step": round(total_ms / steps, 5), "us_per_step": round(1e3 * total_ms / steps, 2),
        "residency": "all experts in HBM",
        "distinct_experts_per_step": round(float(np.mean(u_per_step)), 2),
        "grouped_kernel": grouped_mode(tokens),
        "roofline": roofline(kname, b, f, dur, pk, traffic=traffic, traffic_source=traffic_src,
                             layer_gbs=round(layer_gbs, 1), layer_frac=round(layer_gbs / pk["hbm"], 4),
                             stage_us_with_event_overhead={k: round(1e3 * statistics.mean(v), 2)
                                                           for k, v in stage_ms.items()}),
        "gpu_launches": launches_per_step(tokens) * steps, "clocks": clocks, "wall_s_timed_loop": round(wall, 4),
    }
    e2e_total = sum(e2e_ms)
    rec["e2e"] = {"value": round(tokens * steps / (e2e_total / 1e3), 2), "unit": "tokens/s",
                  "ms_per_step": round(e2e_total / steps, 4), "h2d_bytes_per_step": tokens * HIDDEN * 2,
                  "d2h_bytes_per_step": tokens * HIDDEN * 2,
                  "path": "moe_layer_forward, experts in HBM, x H2D from pinned memory + out D2H per step"}
    if pipe_ms is not None:
        rec["e2e"].update({
            "value": round(tokens * steps / (pipe_ms / 1e3), 2), "ms_per_step": round(pipe_ms / steps, 4),
            "serial_ms_per_step": round(e2e_total / steps, 4),
            "serial_value": round(tokens * steps / (e2e_total / 1e3), 2),
            "path": ("moe_layer_forward over pinned host batches through lightreason_b200.pipeline.HostStream: "
                     "each step's x H2D and out D2H on side streams overlapped with the neighbouring steps; the "
                     "steps as one CUDA-graph replay, no L2 flush between them (the expert banks streamed every "
                     "step exceed L2); serial_*: one step at a time, copies in line, L2 flushed between steps")})
    if host is not None:
        banks = host.host_packed
        gathered = statistics.mean(sum(banks.expert_bytes(e) for e in set(idx_buf[j].cpu().numpy().reshape(-1)
                                                                           .tolist())) for j in used)
        link = host_link_peak(dev)
        g_us = 1e3 * statistics.mean(e2e_stage)
        g_gbs = gathered / (g_us / 1e6) / 1e9
        rec["e2e"] = {
            "value": round(tokens * steps / (e2e_total / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(e2e_total / steps, 4), "residency": "all 256 experts in pinned host RAM",
            "h2d_bytes_per_step": int(tokens * HIDDEN * 2 + gathered), "d2h_bytes_per_step": tokens * HIDDEN * 2,
            "h2d_expert_bytes_per_step": int(gathered), "gather_us": round(g_us, 2), "gather_gbs": round(g_gbs, 2),
            "host_link_peak": link, "gather_frac": round(g_gbs / link["h2d_gbs"], 4),
            "path": "moe_layer_forward with host descriptors (pinned banks in the lossless row codec, decoded in "
                    "registers into HBM slots; the union of the selected experts every step), x H2D + out D2H",
        }
        uses = cache_after["uses"] - cache_before["uses"]
        misses = cache_after["misses"] - cache_before["misses"]
        rec["e2e_cached"] = {
            "value": round(tokens * steps / (sum(cached_ms) / 1e3), 2), "unit": "tokens/s",
            "ms_per_step": round(sum(cached_ms) / steps, 4), "cache_slots": cached.cache_slots,
            "hit_rate": round((uses - misses) / uses, 4) if uses else None,
            "path": f"as e2e, with a device expert cache (LRU over {cached.cache_slots} HBM slots, the B200 form "
                    "of the reference's cached ExpertPool mode): only missing experts cross the host link"}
        host.release()
        cached.release()
    if with_cpu:
        n = cfg.get("cpu_sample", tokens)
        xs_cpu = [a[:n] for a in xs_np[:POOL]]
        rec["cpu_baseline"] = time_cpu_reference(w, gu, dn, xs_cpu, cpu_steps or steps, cpu_warmup or warmup)
    return rec


def run_decode_widths(args, dev, widths=(2, 4, 8)) -> dict:
    """The decode widths between configs[0] (T = 1) and configs[1] (T = 16):
    the same layer (configs[0]/[1] weights, experts in HBM), each width timed
    as those are (one CUDA-graph replay per step, L2 flushed between steps),
    with the whole layer's bytes over the step time and the expert kernel's
    algorithmic bytes over its own event-bracketed time."""
    from lightreason_b200 import native

    pk = peaks()
    cfg = CONFIGS[0]
    w, gu, dn = host_layer(cfg["seed"], cfg["bias"])
    d = lambda a: to_dev(a, dev)  # noqa: E731
    layer = native.Layer(router=d(w.router), gate_up=d(gu), down=d(dn), bias=torch.from_numpy(w.bias).to(dev),
                         shared_gate=d(w.sh_gate), shared_up=d(w.sh_up), shared_down=d(w.sh_down),
                         shared_gate_w=d(w.sh_gate_w))
    flush = l2_flusher(dev)
    out = {}
    for tokens in widths:
        xs = [d(S.hidden_states(cfg["seed"], tokens, step=i)) for i in range(POOL)]
        y = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
        idx = [torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev) for _ in range(POOL)]

        def step(i, ev):
            layer(xs[i % POOL], out=y, idx_out=idx[i % POOL], stage_events=ev)

        for i in range(args.warmup):
            step(i, None)
        ms, _, _ = timed_steps(step, args.steps, args.warmup, flush, 1)
        _, krows, _ = timed_steps(step, args.steps, args.warmup, flush, 1, n_events=8, event_slots=(4, 5))
        kernel_ms = between(krows, 4, 5)
        used = [(args.warmup + i) % POOL for i in range(args.steps)]
        u = [len(set(idx[j].cpu().numpy().reshape(-1).tolist())) for j in used]
        kb = statistics.mean(layer_algo(tokens, x)[0] for x in u)
        layer_gbs = statistics.mean(layer_bytes(tokens, x) / (m / 1e3) / 1e9 for x, m in zip(u, ms))
        kernel_gbs = kb / (statistics.mean(kernel_ms) / 1e3) / 1e9
        out[f"T{tokens}"] = {
            "tokens": tokens, "us_per_step": round(1e3 * statistics.mean(ms), 2),
            "value": round(tokens / (statistics.mean(ms) / 1e3), 2), "unit": "tokens/s",
            "distinct_experts_per_step": round(float(np.mean(u)), 2),
            "expert_kernel": ("fused_decode_kernel" if tokens <= FUSED_DECODE_MAX_TOKENS else
                              "swiglu_grouped_kernel (" + grouped_mode(tokens) + ")"),
            "expert_kernel_us": round(1e3 * statistics.mean(kernel_ms), 2),
            "expert_kernel_hbm_frac": round(kernel_gbs / pk["hbm"], 4),
            "layer_gbs": round(layer_gbs, 1), "layer_hbm_frac": round(layer_gbs / pk["hbm"], 4),
            "gpu_launches": launches_per_step(tokens) * args.steps,
        }
    del layer
    return {"workload": "one MoE layer at the decode widths between configs[0] (T=1) and configs[1] (T=16), "
                        "experts in HBM, seeded as configs[0]",
            "peak_hbm_gbs": pk["hbm"], "l2": "flushed between timed steps by reading a 256 MiB buffer",
            "widths": out}


# -------------------------------------------------------------- config 2 ---

def run_stack(args, cfg, dev, *, with_cpu=True, cpu_steps=None, cpu_warmup=None) -> dict:
    """the 40-layer stack at decode width, every step one
    CUDA-graph replay of all layers.  Each layer reads its own N(0,1) token
    activations -- the normalised residual stream a MoE block sees; the mixer
    layers between them are out of scope, and feeding one MoE output straight
    into the next would collapse the activations and the routing.  Weights
    are drawn on the GPU from seeded generators (~61 GiB); the CPU baseline
    runs layer 0's weights copied back to the host."""
    from lightreason_b200 import native

    pk = peaks()
    tokens, n_layers = cfg["tokens"], cfg["layers"]
    t_setup = time.perf_counter()
    layers = []
    host_layer0 = None
    for li in range(n_layers):
        g = torch.Generator(device=dev)
        g.manual_seed(1000 + li)
        rnd = lambda *shape: (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * 0.02).to(  # noqa: E731
            torch.bfloat16)
        gate_up = rnd(EXPERTS, 2 * INNER, HIDDEN)
        down = rnd(EXPERTS, HIDDEN, INNER)
        bias = torch.from_numpy(S.router_bias(7, li, cfg["bias"])).to(dev)
        parts = dict(router=rnd(EXPERTS, HIDDEN), shared_gate=rnd(INNER, HIDDEN), shared_up=rnd(INNER, HIDDEN),
                     shared_down=rnd(HIDDEN, INNER), shared_gate_w=rnd(HIDDEN))
        layers.append(native.Layer(gate_up=gate_up, down=down, bias=bias, **parts))
        if li == 0 and with_cpu:
            hb = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
            host_layer0 = (S.LayerWeights(seed=0, layer=0, router=hb(parts["router"]), bias=bias.cpu().numpy(),
                                          sh_gate=hb(parts["shared_gate"]), sh_up=hb(parts["shared_up"]),
                                          sh_down=hb(parts["shared_down"]), sh_gate_w=hb(parts["shared_gate_w"])),
                           hb(gate_up), hb(down))
    xs_np = [S.hidden_states(7 + li, tokens) for li in range(n_layers)]
    xs = [to_dev(a, dev) for a in xs_np]
    acts = [torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev) for _ in range(n_layers)]
    idx = [torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev) for _ in range(n_layers)]
    log(f"[bench] stack setup {time.perf_counter() - t_setup:.1f}s, {n_layers} layers, "
        f"{torch.cuda.memory_allocated(dev) / 2**30:.1f} GiB allocated")

    def stack_step(i, ev):
        for li, layer in enumerate(layers):
            layer(xs[li], out=acts[li], idx_out=idx[li])

    def no_flush():
        pass  # every step streams ~55 GB of weights: far larger than L2
    sampler = ClockSampler(dev.index or 0)
    with sampler:
        ms, _, _ = timed_steps(stack_step, args.steps, args.warmup, no_flush, 1)
    clocks = sampler.summary()
    u = [len(set(t.cpu().numpy().reshape(-1).tolist())) for t in idx]
    lb = [layer_bytes(tokens, ui) for ui in u]
    flops = sum((tokens * TOP_K + tokens) * EXPERT_FLOPS_PER_ROW + 2 * tokens * EXPERTS * HIDDEN for _ in u)
    step_ms = sum(ms) / args.steps
    rec = {
        "workload": cfg["workload"], "value": round(tokens / (step_ms / 1e3), 2), "unit": "tokens/s",
        "ms_per_step": round(step_ms, 5), "us_per_step": round(step_ms * 1e3, 2),
        "residency": "all experts of 40 layers in HBM", "distinct_experts_per_layer": round(float(np.mean(u)), 1),
        "l2": "not flushed: every step streams the selected experts of 40 layers (far above L2)",
        "roofline": roofline("whole 40-layer step (all kernels)", sum(lb), flops, step_ms, pk, sustained=True),
        "gpu_launches": launches_per_step(tokens) * n_layers * args.steps, "clocks": clocks,
    }
    del layers
    torch.cuda.empty_cache()
    if with_cpu:
        w0, gu0, dn0 = host_layer0
        per_layer = time_cpu_reference(w0, gu0, dn0, [xs_np[0]], cpu_steps or args.steps, cpu_warmup or args.warmup)
        stack_ms = per_layer["ms_per_step"] * n_layers
        rec["cpu_baseline"] = dict(per_layer, value=round(tokens / (stack_ms / 1e3), 2), ms_per_step=round(stack_ms, 3),
                                   sample=per_layer["sample"] + f" (layer 0 of the stack; the 40-layer step is "
                                                               f"{n_layers} x the median)")
    return rec


# ---------------------------------------------------- config 4 (default) ---

def ep_weights(cfg, mine, dev):
    """The experts `mine` [El, 2I, H] / [El, H, I] on the device (each expert
    drawn from its own seed, on a thread pool) and the replicated parts."""
    seed = cfg["seed"]
    w = S.layer_weights(seed, bias=cfg["bias"])
    gu = torch.empty((len(mine), 2 * INNER, HIDDEN), dtype=torch.bfloat16, device=dev)
    dn = torch.empty((len(mine), HIDDEN, INNER), dtype=torch.bfloat16, device=dev)

    def draw(j):
        e = mine[j]
        return j, S.expert_gate_up(seed, 0, e), S.expert_down(seed, 0, e)
    with ThreadPoolExecutor(min(16, os.cpu_count() or 1)) as pool:
        for j, a, b in pool.map(draw, range(len(mine))):
            gu[j].copy_(to_dev(a, dev))
            dn[j].copy_(to_dev(b, dev))
    return w, gu, dn


def ep_placement(cfg, world, rank, dev, transport, mode):
    """(owner rank per expert or None, this rank's experts, description).
    "balanced" (peer exchange, N > 1): the routes per expert of the layer's
    router over one calibration batch per rank (seeds no timed step uses),
    summed over the ranks, placed by the longest-processing-time rule; else
    contiguous ranges."""
    from lightreason_b200.expert_parallel import balanced_placement, expert_loads, placement_experts, shard

    if world == 1 or transport != "p2p" or mode == "contiguous":
        return None, list(shard(EXPERTS, world, rank)), "contiguous: rank r owns experts [r*E/N, (r+1)*E/N)"
    import torch.distributed as dist

    w = S.layer_weights(cfg["seed"], bias=cfg["bias"])
    x_cal = to_dev(S.hidden_states(900 + 17 * rank, cfg["tokens"], step=0), dev)
    loads = expert_loads(to_dev(w.router, dev), x_cal, bias=torch.from_numpy(w.bias).to(dev), top_k=TOP_K)
    dist.all_reduce(loads)
    owner = balanced_placement(loads.cpu().tolist(), world)
    return owner, placement_experts(owner, rank), ("balanced: routes per expert of the router over one "
                                                   "calibration batch per rank (not a timed batch), summed "
                                                   "over the ranks, longest-processing-time placement")


def build_ep(cfg, world, rank, dev, transport, placement_mode="balanced"):
    from lightreason_b200.expert_parallel import ExpertParallelLayer, PeerExchange, TorchExchange

    owner, mine, how = ep_placement(cfg, world, rank, dev, transport, placement_mode)
    w, gu, dn = ep_weights(cfg, mine, dev)
    d = lambda a: to_dev(a, dev)  # noqa: E731
    peer = None
    if transport == "p2p":
        peer = PeerExchange(world=world, rank=rank, tokens=cfg["tokens"], top_k=TOP_K, hidden=HIDDEN,
                            experts=EXPERTS, device=dev)
        exchange = peer
    else:
        exchange = TorchExchange()
    layer = ExpertParallelLayer(router=d(w.router), gate_up=gu, down=dn, shared_gate=d(w.sh_gate),
                                shared_up=d(w.sh_up), shared_down=d(w.sh_down), shared_gate_w=d(w.sh_gate_w),
                                bias=torch.from_numpy(w.bias).to(dev), rank=rank, world=world,
                                tokens=cfg["tokens"], exchange=exchange, placement=owner)
    layer.placement_how = how
    return w, mine, layer, peer


def bf16_ulp(x):
    x = np.abs(np.asarray(x, dtype=np.float32))
    return (2.0 ** (np.floor(np.log2(np.maximum(x, np.float32(2.0 ** -126)))) - 7)).astype(np.float32)


def ids_against_cpu_router(ids_gpu: np.ndarray, ids_cpu: np.ndarray, z_cpu: np.ndarray) -> dict:
    """Expert ids of the GPU layer against the torch CPU router's top-k: a
    token's selection may differ only where the experts swapped in or out lie
    within one BF16 ulp of the k-th largest z = logits + bias of the CPU
    router (a near tie decided by the FP32 summation order); such tokens are
    counted, anything else is a mismatch."""
    exact = excused = bad = 0
    for t in range(ids_gpu.shape[0]):
        g, c = set(ids_gpu[t].tolist()), set(ids_cpu[t].tolist())
        if g == c:
            exact += 1
            continue
        kth = np.sort(z_cpu[t])[::-1][TOP_K - 1]
        tol = bf16_ulp(kth)
        if all(abs(z_cpu[t][e] - kth) <= tol for e in g ^ c):
            excused += 1
        else:
            bad += 1
    return {"tokens": int(ids_gpu.shape[0]), "same_set": exact, "near_tie_excused": excused, "mismatched": bad}


def ep_parity(layer, w, out_host, x_dev, world, rank, dev, sample=64) -> dict:
    """The rank's expert-parallel output of its last timed step against the
    single-GPU layer with all 256 experts on this GPU (bit for bit), and the
    ids against the single-GPU layer (exactly) and the torch CPU router on a
    token sample (near ties counted)."""
    from lightreason_b200 import native

    el = layer.local_experts
    if world > 1:
        import torch.distributed as dist

        full_gu = torch.empty((EXPERTS, 2 * INNER, HIDDEN), dtype=torch.bfloat16, device=dev)
        full_dn = torch.empty((EXPERTS, HIDDEN, INNER), dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(full_gu, layer.gate_up[:el].contiguous())
        dist.all_gather_into_tensor(full_dn, layer.down[:el].contiguous())
        if layer.placement is not None:  # gathered in rank order: back to expert order
            from lightreason_b200.expert_parallel import placement_experts
            order = [e for r in range(world) for e in placement_experts(layer.placement, r)]
            pos = torch.tensor(np.argsort(order), dtype=torch.int64, device=dev)
            full_gu, full_dn = full_gu.index_select(0, pos), full_dn.index_select(0, pos)
    else:
        full_gu, full_dn = layer.gate_up[:EXPERTS], layer.down[:EXPERTS]
    sg, su = layer.gate_up[el, :INNER], layer.gate_up[el, INNER:]
    single = native.Layer(router=layer.router, gate_up=full_gu, down=full_dn, bias=layer.bias, shared_gate=sg,
                          shared_up=su, shared_down=layer.down[el], shared_gate_w=layer.shared_gate_w)
    tokens = x_dev.shape[0]
    idx = torch.empty((tokens, TOP_K), dtype=torch.int64, device=dev)
    want = single(x_dev, idx_out=idx)
    torch.cuda.synchronize()
    got_bits = out_host.view(torch.int16).numpy()
    want_bits = want.view(torch.int16).cpu().numpy()
    diff = int((got_bits != want_bits).sum())
    ids_ep = layer.idx[:tokens].cpu().numpy()
    ids_single = idx.cpu().numpy()
    x_bits = x_dev.view(torch.int16).cpu().numpy().view(np.uint16)[:sample]
    _, ids_cpu, z_cpu = cpu_reference_router(w, x_bits)
    vs_cpu = ids_against_cpu_router(np.sort(ids_ep[:sample], 1), np.sort(ids_cpu, 1), z_cpu)
    del single, full_gu, full_dn
    return {"bit_exact_vs_single_gpu": diff == 0, "values_differing": diff, "tokens": tokens,
            "ids_exact_vs_single_gpu": bool(np.array_equal(ids_ep, ids_single)),
            "ids_vs_torch_cpu_router": vs_cpu}


def cpu_reference_router(w, x_bits):
    """Router of the reference's torch path on the CPU (F.linear on BF16,
    softmax over logits + bias, top-k): (scores, ids, z)."""
    F = torch.nn.functional
    t_bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    with torch.no_grad():
        z = F.linear(t_bf(x_bits), t_bf(w.router)).float() + torch.from_numpy(w.bias)
        v, i = torch.topk(F.softmax(z, dim=-1), TOP_K, dim=-1)
    return v.numpy(), i.numpy(), z.numpy()


def run_ep(args, world, rank, local) -> dict:
    """one expert-parallel step per timed step.

    transport "p2p" (default, and always at N = 1): the NVLink peer-memory
    exchange, no host synchronisation, every timed step one CUDA-graph replay;
    at N = 1 the rank is its own only peer.  "nccl" (N > 1): the
    all_to_all_single exchange, eager steps (the split sizes are read on the
    host every step)."""
    from lightreason_b200 import native
    from lightreason_b200.expert_parallel import EP_STAGES

    cfg = CONFIGS[4]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    native.device_check(local)
    pk = peaks()
    tokens = cfg["tokens"]
    transport = args.transport if world > 1 else "p2p"
    t_setup = time.perf_counter()
    w, mine, layer, peer = build_ep(cfg, world, rank, dev, transport, args.placement)
    placement_how = layer.placement_how
    xs_np = [S.hidden_states(input_seed(cfg, rank), tokens, step=i) for i in range(POOL)]
    xs = [to_dev(a, dev) for a in xs_np]
    xs_host = [pinned(a) for a in xs_np]
    out = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
    out_host = torch.empty((tokens, HIDDEN), dtype=torch.bfloat16).pin_memory()
    xin = torch.empty_like(out)
    flush = l2_flusher(dev)
    log(f"[bench] ep setup {time.perf_counter() - t_setup:.1f}s, rank {rank}/{world}, {len(mine)} experts "
        f"({layer.placement_how.split(':')[0]} placement), transport {transport}")

    # the expert kernel's own events: two around the grouped kernel on the
    # peer exchange, the local layer's eight stage events on NCCL
    k_events, k_slots = (2, (0, 1)) if transport == "p2p" else (8, (4, 5))

    def dev_step(i, ev):
        layer(xs[i % POOL], out=out, stage_events=ev)

    def ep_step(i, ev):
        layer(xs[i % POOL], out=out, ep_events=ev)

    def e2e_step(i, ev):
        xin.copy_(xs_host[i % POOL], non_blocking=True)
        layer(xin, out=out)
        out_host.copy_(out, non_blocking=True)

    def eager(run_step, n_events=0, event_slots=()):
        """Eager steps (the NCCL exchange reads its split sizes on the host)."""
        for i in range(args.warmup):
            flush()
            run_step(i, None)
        torch.cuda.synchronize()
        barrier(world)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        rows = [[torch.cuda.Event(enable_timing=True) if j in event_slots else None for j in range(n_events)]
                for _ in range(args.steps)] if n_events else None
        for i in range(args.steps):
            flush()
            ev[i][0].record()
            run_step(args.warmup + i, rows[i] if rows else None)
            ev[i][1].record()
        torch.cuda.synchronize()
        barrier(world)
        return [a.elapsed_time(b) for a, b in ev], rows, None

    run = timed_steps if transport == "p2p" else eager
    sampler = ClockSampler(local)
    with sampler:
        for i in range(args.warmup):          # buffers and workspaces exist before capture
            dev_step(i, None)
        torch.cuda.synchronize()
        ms, _, _ = run(dev_step, args.steps, args.warmup, flush, world) if run is timed_steps else run(dev_step)
        if run is timed_steps:
            _, krows, _ = run(dev_step, args.steps, args.warmup, flush, world, n_events=k_events, event_slots=k_slots)
            _, erows, _ = run(ep_step, args.steps, args.warmup, flush, world, n_events=len(EP_STAGES) + 1,
                              event_slots=tuple(range(len(EP_STAGES) + 1)))
            e2e_ms, _, _ = run(e2e_step, args.steps, args.warmup, flush, world)
        else:
            _, krows, _ = run(dev_step, k_events, k_slots)
            erows = None
            e2e_ms, _, _ = run(e2e_step)
        out_last = out_host.clone()  # the serial loop's last timed step, for the parity check
        pipe_ms = pipelined_e2e(lambda x, o: layer(x, out=o), xs_host, (tokens, HIDDEN), dev, args.steps,
                                args.warmup, world, capture=transport == "p2p")
        if peer is not None:
            peer.check()
    clocks = sampler.summary()
    kern_ms = between(krows, *k_slots)
    total_ms = dist_max(sum(ms), world)
    e2e_total = dist_max(sum(e2e_ms), world)
    pipe_total = dist_max(pipe_ms, world)
    value = world * tokens * args.steps / (total_ms / 1e3)

    # this rank's work in the last timed step
    if transport == "p2p":
        st = layer.peer_stats()
        per_sender = st["rows_per_sender"]
        received_rows = st["rows_received"]
        u_local = st["local_experts_with_rows"]
        # the step's own routes (the selection's ids) whose owner is another rank
        ids = layer.idx[:tokens].cpu().numpy()
        owner = (np.asarray(layer.placement)[ids] if layer.placement is not None else ids // (EXPERTS // world))
        leaving = int(np.count_nonzero(owner != rank))
        from_peers = sum(per_sender) - per_sender[rank]
    else:
        m = layer.last_splits
        leaving = sum(m[rank][dd] for dd in range(world) if dd != rank)
        received = sum(m[s][rank] for s in range(world))
        from_peers = received - m[rank][rank]
        local_ids = layer.recv_meta[:received].cpu().numpy()
        received_rows = int(local_ids.size)
        u_local = len(set(local_ids.tolist()))
    rows = tokens + received_rows
    # grouped kernel: local experts' + the shared expert's weights, the
    # route-ordered rows in, activations out and back in, rows out; on the
    # peer exchange also its row gather (each row read from its sender, over
    # NVLink or locally, and written into the route-ordered buffer)
    gather_bytes = 2 * rows * HIDDEN * 2 if transport == "p2p" else 0
    kernel_bytes = ((u_local + 1) * EXPERT_BYTES + rows * HIDDEN * 2 + 2 * rows * INNER * 2 + rows * HIDDEN * 2
                    + gather_bytes)
    kernel_flops = rows * EXPERT_FLOPS_PER_ROW
    traffic, traffic_src = profiled_traffic(f"config4_world{world}_grouped")
    stages = None
    # rows crossing NVLink per step for this rank: its tokens' rows the owners
    # pull and the expert rows they store back (routes leaving), and the rows
    # it pulls from its senders and stores back to them (routes received)
    nvlink = {"rows_pulled_from_peers": from_peers, "rows_returned_to_peers": from_peers,
              "own_rows_pulled_by_peers": leaving, "own_rows_returned_by_peers": leaving,
              "bytes_in": (from_peers + leaving) * HIDDEN * 2, "bytes_out": (from_peers + leaving) * HIDDEN * 2}
    if erows is not None:
        st = stage_times(erows, EP_STAGES)
        stages = {k: round(1e3 * statistics.median(v), 2) for k, v in st.items()}
        stages["step_with_event_overhead"] = round(1e3 * statistics.median(between(erows, 0, len(EP_STAGES))), 2)
        stages["grouped_kernel"] = round(1e3 * statistics.median(kern_ms), 2)
        t_ms = statistics.median(st["experts"])
        if from_peers:
            nvlink["experts_stage_gbs_per_direction"] = round(2 * from_peers * HIDDEN * 2 / 2 / (t_ms / 1e3) / 1e9, 1)
    if peer is not None:
        peer.close()

    # parity of the last timed step (the e2e loop's, as the caller received it)
    last = (args.warmup + args.steps - 1) % POOL
    parity = ep_parity(layer, w, out_last, xs[last], world, rank, dev)
    ok = (parity["bit_exact_vs_single_gpu"] and parity["ids_exact_vs_single_gpu"]
          and parity["ids_vs_torch_cpu_router"]["mismatched"] == 0)
    all_ok = dist_all(ok, world)
    parity["all_ranks_ok"] = all_ok
    if not ok:
        log(f"[bench] rank {rank}: expert-parallel parity FAILED: {parity}")
    del layer
    torch.cuda.empty_cache()

    timing = ("each timed step one CUDA-graph replay of the whole rank step (no host synchronisation), CUDA "
              "events around it, max over ranks of the summed step times" if transport == "p2p" else
              "CUDA events around each whole step on the compute stream (includes the host read of the "
              "all-to-all split sizes), max over ranks of the summed step times")
    # p2p: router_tc + select/publish; plan, grouped; finish; combine.
    # NCCL: router x2, permute x3,
    # ep_dispatch, ep_unpack, the local layer in rows mode (permute x3,
    # grouped_plan, gather_tokens, grouped), combine
    launches = 6 if transport == "p2p" else 14
    res = {
        "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5), "us_per_step": round(1e3 * total_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations, Zipf(1.1) router bias)",
        "config": {"workload": cfg["workload"], "tokens_per_gpu": tokens, "hidden": HIDDEN, "inner": INNER,
                   "experts": EXPERTS, "experts_per_gpu": len(mine), "top_k": TOP_K, "shared_expert": True,
                   "parallelism": f"ep{world}", "transport": transport, "placement": placement_how,
                   "rank0_rows_received": received_rows,
                   "rank0_routes_leaving": leaving, "rank0_distinct_local_experts": u_local,
                   "grouped_kernel": grouped_mode(tokens + world * tokens * TOP_K),
                   "l2": "flushed between timed steps by reading a 256 MiB buffer, outside each step's event window",
                   "timing": timing},
        "roofline": roofline("swiglu_grouped_kernel (rank 0: local experts + shared expert; in-kernel row pull "
                             "and return over NVLink)", kernel_bytes,
                             kernel_flops, statistics.mean(kern_ms), pk, traffic=traffic,
                             traffic_source=traffic_src),
        "e2e": {"value": round(world * tokens * args.steps / (pipe_total / 1e3), 2), "unit": "tokens/s",
                "ms_per_step": round(pipe_total / args.steps, 4), "h2d_bytes_per_step": tokens * HIDDEN * 2,
                "d2h_bytes_per_step": tokens * HIDDEN * 2,
                "serial_ms_per_step": round(e2e_total / args.steps, 4),
                "serial_value": round(world * tokens * args.steps / (e2e_total / 1e3), 2),
                "path": ("ExpertParallelLayer.forward per rank over pinned host batches through "
                         "lightreason_b200.pipeline.HostStream: each step's x H2D and out D2H on side streams "
                         "overlapped with the neighbouring steps; the steps as one CUDA-graph replay (eager on "
                         "NCCL), no L2 flush between them (each rank's expert banks, streamed every step, exceed "
                         "L2); max over ranks.  serial_*: one step at a time, copies in line, L2 flushed between "
                         "steps")},
        "parity": parity,
        "ep_stages_us": stages, "nvlink_rank0": nvlink,
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }
    if not all_ok:
        res["parity_failed"] = True
    return res


# ------------------------------------------------------ N = 1 sub-records ---

def run_subconfigs(args, dev) -> dict:
    """configs[0..3] on this GPU, each as a sub-record with its own step time,
    roofline and CPU baseline (fewer CPU repeats than the main line)."""
    out = {}
    cpu = dict(with_cpu=not args.no_cpu_baseline, cpu_steps=min(args.steps, 6), cpu_warmup=1)
    for key, cfg in (("config0", CONFIGS[0]), ("config1", dict(CONFIGS[1], host_experts=True)),
                     ("config3", CONFIGS[3])):
        t = time.perf_counter()
        rec = run_layer(args, cfg, dev, **cpu)
        if key == "config1":
            e2e = rec.pop("e2e")
            cached = rec.pop("e2e_cached")
            out["config1_hbm"] = rec
            out["config1_e2e"] = dict(e2e, e2e_cached=cached, cpu_baseline=rec.get("cpu_baseline"),
                                      workload=CONFIGS[1]["workload"])
        else:
            out[key] = rec
        torch.cuda.empty_cache()
        log(f"[bench] {key} {time.perf_counter() - t:.1f}s")
    t = time.perf_counter()
    out["decode_widths"] = run_decode_widths(args, dev)
    torch.cuda.empty_cache()
    log(f"[bench] decode widths {time.perf_counter() - t:.1f}s")
    t = time.perf_counter()
    out["config2"] = run_stack(args, CONFIGS[2], dev, **cpu)
    torch.cuda.empty_cache()
    log(f"[bench] config2 {time.perf_counter() - t:.1f}s")
    return out


# --------------------------------------------------------- reference arm ---

def run_reference(args, cfg_index, world, rank):
    """Reference arm: the reference's CPU implementation of the main line's
    workload on the host cores, rank 0 only (the host is shared by the ranks):
    the same inputs, repeat count and median as the cpu_baseline leg."""
    if rank != 0:
        return None
    cfg = CONFIGS[cfg_index]
    layers = 1
    if cfg_index == 2:
        # one layer of the stack's shape (seeded on the host), times 40 layers
        layers = cfg["layers"]
        cfg = dict(CONFIGS[0], index=2, tokens=cfg["tokens"], bias=cfg["bias"], workload=cfg["workload"])
    w, gu, dn, xs = cpu_inputs(cfg)
    cb = time_cpu_reference(w, gu, dn, xs, args.steps, args.warmup)
    if layers > 1:
        stack_ms = cb["ms_per_step"] * layers
        cb = dict(cb, value=round(cfg["tokens"] / (stack_ms / 1e3), 2), ms_per_step=round(stack_ms, 3),
                  sample=cb["sample"] + f" (one layer; the {layers}-layer step is {layers} x the median)")
    return {
        "impl": "reference", "metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
        "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg["workload"], "tokens_per_step": cb["tokens_per_step"],
                   "note": "one host's CPU path; at N > 1 GPUs the host does not grow, so compare per GPU"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "spread")},
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------ profiling helpers ---

def run_profile(args, cfg_index):
    """--profile N: N eager steps of the config on one GPU, no CUDA graphs and
    no timing, for a profiler's launch list or kernel capture (config 4: the
    expert-parallel step at world 1)."""
    from lightreason_b200 import native

    dev = torch.device("cuda", 0)
    native.device_check(0)
    flush = l2_flusher(dev)
    cfg = CONFIGS[cfg_index]
    if cfg_index == 4:
        _, _, layer, peer = build_ep(cfg, 1, 0, dev, "p2p")
        xs = [to_dev(S.hidden_states(input_seed(cfg, 0), cfg["tokens"], step=i), dev) for i in range(2)]
        for i in range(args.profile):
            flush()
            layer(xs[i % 2])
        torch.cuda.synchronize()
        peer.check()
        peer.close()
    else:
        w = S.layer_weights(cfg.get("seed", 1), bias=cfg["bias"])
        gu, dn = w.stacked()
        d = lambda a: to_dev(a, dev)  # noqa: E731
        hbm = native.Layer(router=d(w.router), gate_up=d(gu), down=d(dn), bias=torch.from_numpy(w.bias).to(dev),
                           shared_gate=d(w.sh_gate), shared_up=d(w.sh_up), shared_down=d(w.sh_down),
                           shared_gate_w=d(w.sh_gate_w))
        xs = [d(S.hidden_states(1, cfg["tokens"], step=i)) for i in range(min(args.profile, 4))]
        for i in range(args.profile):
            flush()
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
    pk = peaks()
    hbm_peak = pk["hbm"]
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
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if pk["source"] == "measured" else
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


# ------------------------------------------------------------------ main ---

def single_gpu_line(args, cfg_index, dev) -> dict:
    """--config 0|1|2|3 as the main line on one GPU."""
    cfg = CONFIGS[cfg_index]
    if cfg_index == 2:
        rec = run_stack(args, cfg, dev, with_cpu=not args.no_cpu_baseline)
    else:
        if cfg_index == 1:
            cfg = dict(cfg, host_experts=True)
        if args.tokens:
            cfg = dict(cfg, tokens=args.tokens, workload=cfg["workload"] + f" (tokens overridden to {args.tokens})")
        rec = run_layer(args, cfg, dev, with_cpu=not args.no_cpu_baseline)
    tokens = cfg["tokens"]
    line = {"metric": "MoE-layer throughput (tokens/s) and us/step, fraction of HBM roofline",
            "value": rec.pop("value"), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": rec.pop("ms_per_step"), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": rec.pop("workload"), "tokens_per_step": tokens, "hidden": HIDDEN,
                       "inner": INNER, "experts": EXPERTS, "top_k": TOP_K, "parallelism": "single-gpu",
                       "l2": rec.pop("l2", "flushed between timed steps by reading a 256 MiB buffer")}}
    line.update(rec)
    return line


def main():
    # The one JSON line goes to the real stdout; anything libraries print there
    # (NCCL's version banner, for one) is sent to stderr instead.
    json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=4,
                    help="BASELINE config of the main line (default 4, the expert-parallel layer, at every N)")
    ap.add_argument("--tokens", type=int, default=None, help="override the tokens per step of configs 0, 1, 3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subconfigs", action="store_true",
                    help="at N = 1, skip the configs[0..3] sub-records of the default line")
    ap.add_argument("--transport", choices=("p2p", "nccl"), default="p2p",
                    help="expert-parallel exchange on N > 1 GPUs: NVLink peer memory (default) or NCCL all_to_all")
    ap.add_argument("--placement", choices=("balanced", "contiguous"), default="balanced",
                    help="expert placement of the peer exchange on N > 1 GPUs: balanced by the routes of a "
                         "calibration batch (default) or contiguous ranges")
    ap.add_argument("--encode", action="store_true",
                    help="time the device codec encoders on one layer's expert banks instead of the layer")
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="run N eager steps of the config on one GPU (for ncu) and print a short status line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        res = run_reference(args, args.config, world, rank)
        if res is not None:
            print(json.dumps(res), file=json_out, flush=True)
        return
    if args.profile:
        print(json.dumps(run_profile(args, args.config)), file=json_out, flush=True)
        return
    if args.encode:
        print(json.dumps(run_encode(args)), file=json_out, flush=True)
        return
    world, rank, local = dist_setup()
    failed = False
    try:
        if args.config == 4:
            res = run_ep(args, world, rank, local)
            failed = bool(res.get("parity_failed"))
            dev = torch.device("cuda", local)
            if world == 1 and not args.no_cpu_baseline:
                w, gu, dn, xs = cpu_inputs(CONFIGS[4])
                res["cpu_baseline"] = time_cpu_reference(w, gu, dn, xs, args.steps, args.warmup)
                del w, gu, dn
            if world == 1 and not args.no_subconfigs:
                res["configs"] = run_subconfigs(args, dev)
        else:
            if world > 1:
                raise SystemExit("configs 0-3 run on one GPU; use --config 4 with --gpus N > 1")
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
            from lightreason_b200 import native

            native.device_check(local)
            res = single_gpu_line(args, args.config, dev)
        if rank == 0:
            print(json.dumps(res), file=json_out, flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if failed:
        sys.exit(3)


if __name__ == "__main__":
    main()
