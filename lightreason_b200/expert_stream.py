"""B200 drop-in for edge35b/expert_stream.py: patch a model's
Qwen3_5MoeExperts forwards onto the sm_100a MoE kernels.

Same names and contracts as the reference (:29-526): MODES, TransferStats,
ExpertPool(device, capacity_bytes=..., non_blocking=...), the per-module
_Layer with its checks, and the patch_experts(model, mode=..., pool=...)
context manager that installs module.forward and restores it with `del` on
exit.  The forward keeps the eager contract of Qwen3_5MoeExperts.forward
(hidden[T,H] BF16, top_k_index[T,K] int64, top_k_weights[T,K] BF16 ->
[T,H] BF16; ascending-expert BF16 accumulation) and runs it as one chain of
device launches with no host synchronisation: the reference's host reads of
the routes (expert_stream.py:359, :207; fused_experts.py:47;
block_experts.py:103) are gone.

Modes.  The reference's transfer controls all compute the same eager
arithmetic and differ in where the expert rows live; on B200 they map onto
three residencies:
  "b200"         experts in HBM (module parameters copied to the pool device
                 once, or used in place when they already live there) -- also
                 what "fused", "batched", "scheduled", "grouped" and "seeded"
                 select;
  "b200-host"    experts stay in (pinned, mapped) host RAM and the union of
                 each call's selected experts is copied into HBM slots on the
                 device -- also "dense", "selected", "cached", "pipelined",
                 "cpu" and "hybrid";
  "b200-packed"  as b200-host with the rows kept in the lossless row codec
                 (bf16_expert_codec), 25% fewer bytes over the host link --
                 also "packed".
With capacity_bytes > 0 the host residencies keep up to capacity_bytes of
experts per layer in HBM slots across calls (a device-side LRU, the role of
the reference pool's byte-bounded row cache, expert_stream.py:132-174): only
the missing experts cross the host link.  Calls that route to more experts
than the cache holds take the uncached path.
"""

from __future__ import annotations

import threading
from contextlib import contextmanager
from dataclasses import asdict, dataclass

import numpy as np
import torch

from lightreason_b200 import native

REFERENCE_MODES = ("dense", "selected", "cached", "packed", "scheduled", "grouped", "pipelined", "fused",
                   "batched", "cpu", "seeded", "hybrid")
B200_MODES = ("b200", "b200-host", "b200-packed")
MODES = REFERENCE_MODES + B200_MODES
RESIDENCY = {
    **{m: "b200" for m in ("b200", "fused", "batched", "scheduled", "grouped", "seeded")},
    **{m: "b200-host" for m in ("b200-host", "dense", "selected", "cached", "pipelined", "cpu", "hybrid")},
    **{m: "b200-packed" for m in ("b200-packed", "packed")},
}


@dataclass
class TransferStats:
    layer_calls: int = 0
    b200_layer_calls: int = 0
    host_layer_calls: int = 0
    packed_layer_calls: int = 0
    tokens: int = 0
    resident_bytes: int = 0
    pinned_bytes: int = 0
    replayed_layer_calls: int = 0   # calls served by a captured graph (scheduled_graph.replay_experts)
    mixer_replays: int = 0          # mixer forwards served by a captured graph (packed_native.mixer_graphs)


class ExpertPool:
    """Per-device state shared by the patched layers: the device copies (HBM
    residency) or host mappings / packed banks (host residencies), and the
    workspaces.  Like the reference pool, it is used on one CUDA device,
    thread and stream (expert_stream.py:124-130)."""

    def __init__(self, device="cuda:0", *, capacity_bytes=0, non_blocking=True):
        if type(capacity_bytes) is not int or capacity_bytes < 0:
            raise ValueError("capacity_bytes must be a nonnegative integer")
        if type(non_blocking) is not bool:
            raise ValueError("non_blocking must be a boolean")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("Expert streaming requires a CUDA destination")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self._capacity_bytes = capacity_bytes
        self._non_blocking = non_blocking
        self._owner = None
        self._attached = False
        self._cache_layers = 1   # layers sharing capacity_bytes, set when a patch is installed
        self._layers = {}
        self.stats = TransferStats()

    def snapshot(self):
        return {**asdict(self.stats), "capacity_bytes": self._capacity_bytes, "layers": len(self._layers),
                "non_blocking": self._non_blocking}

    def reset_stats(self):
        self.stats = TransferStats(resident_bytes=self.stats.resident_bytes, pinned_bytes=self.stats.pinned_bytes)

    def clear(self):
        """Release device copies, host mappings and packed banks."""
        for layer in self._layers.values():
            layer.release()
        self._layers.clear()
        self.stats.resident_bytes = self.stats.pinned_bytes = 0

    def _check_context(self):
        if torch.cuda.is_current_stream_capturing():
            return  # a CUDA-graph capture records on its own side stream; the replay runs on the caller's
        owner = (threading.get_ident(), torch.cuda.current_stream(self.device).cuda_stream)
        if self._owner is None:
            self._owner = owner
        elif owner != self._owner:
            raise RuntimeError("Use the pool on its original CUDA thread and stream")

    def cache_slots(self, layer: "_Layer", routed: int) -> int:
        """Expert-cache slots for a host-resident layer (0: none), if a call
        routing to `routed` distinct experts at most fits in them.  The
        reference keeps one LRU of device rows under capacity_bytes for all
        layers (expert_stream.py:147-174); here each patched layer gets an even
        share of the budget as its own device-planned slot bank."""
        if layer.residency == "b200" or not self._capacity_bytes:
            return 0
        share = self._capacity_bytes // max(1, self._cache_layers)
        slots = min(share // layer.row_bytes, layer.module.num_experts, 1024)
        return slots if slots >= routed else 0

    def _native_layer(self, layer: "_Layer", top_k: int, owner=None, extra=None, cache: int = 0) -> native.Layer:
        """The native layer of one patched module, built on first use: the
        expert banks in the layer's residency plus `extra` device tensors
        (router and shared expert, for a whole-block patch), behind an
        expert cache of `cache` slots when nonzero."""
        key = (id(owner if owner is not None else layer.module), layer.residency, cache)
        cached = self._layers.get(key)
        if cached is not None:
            if cached.top_k != top_k:
                cached.set_top_k(top_k)
            return cached
        extra = {k: v() for k, v in (extra or {}).items()}
        gu, dn = layer.gate_up, layer.down
        if layer.residency == "b200":
            if gu.device != self.device:
                gu = gu.detach().to(self.device)
                dn = dn.detach().to(self.device)
                self.stats.resident_bytes += gu.numel() * 2 + dn.numel() * 2
            built = native.Layer(gate_up=gu.contiguous(), down=dn.contiguous(), top_k=top_k, **extra)
        elif layer.residency == "b200-host":
            shared = self._layers.get((key[0], layer.residency, 0))
            if shared is not None and shared._host_dev[0] is not None:
                host = dict(host_gate_up=shared.host_gate_up, host_down=shared.host_down)
            else:
                host = dict(host_gate_up=gu.detach().contiguous(), host_down=dn.detach().contiguous())
                self.stats.pinned_bytes += gu.numel() * 2 + dn.numel() * 2
            built = native.Layer(top_k=top_k, device=self.device, cache_slots=cache or None, **host, **extra)
        else:
            shared = self._layers.get((key[0], layer.residency, 0)) or next(
                (v for k, v in self._layers.items() if k[:2] == key[:2]), None)
            if shared is not None:
                banks = shared.host_packed
            else:
                bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
                banks = native.PackedHostBanks(bits(gu), bits(dn), self.device)
                self.stats.pinned_bytes += sum(b.numel() for b in banks.buffers)
            built = native.Layer(host_packed=banks, top_k=top_k, device=self.device, cache_slots=cache or None,
                                 **extra)
        self.stats.resident_bytes += sum(t.numel() * t.element_size() for t in extra.values())
        self._layers[key] = built
        return built


def _check_module(name, module):
    if module.num_experts <= 0 or module.hidden_dim <= 0 or module.intermediate_dim <= 0:
        raise ValueError(f"{name}: invalid expert dimensions")
    expected = (
        (module.num_experts, 2 * module.intermediate_dim, module.hidden_dim),
        (module.num_experts, module.hidden_dim, module.intermediate_dim),
    )
    for source, shape in zip((module.gate_up_proj, module.down_proj), expected):
        if source.dtype != torch.bfloat16 or source.requires_grad or not source.is_contiguous() or \
                tuple(source.shape) != shape:
            raise ValueError(f"{name}: expected frozen contiguous BF16 expert parameters")


class _Layer:
    """One patched Qwen3_5MoeExperts module (expert_stream.py:309-454)."""

    def __init__(self, name, module, pool, mode):
        self.name = name
        self.module = module
        self.pool = pool
        self.mode = mode
        self.residency = RESIDENCY[mode]
        self.gate_up = module.gate_up_proj
        self.down = module.down_proj
        self.act_fn = module.act_fn
        if "forward" in vars(module) or getattr(module, "_hf_hook", None) is not None:
            raise ValueError(f"{name}: expert forwards must have no existing offload hooks")
        _check_module(name, module)
        if self.residency != "b200" and self.gate_up.device.type != "cpu":
            raise ValueError(f"{name}: host residency needs CPU expert parameters")
        self.row_bytes = (self.gate_up.numel() + self.down.numel()) * 2 // module.num_experts

    def _check_sources(self):
        module = self.module
        if module.training:
            raise RuntimeError(f"{self.name}: use eval mode")
        if module.gate_up_proj is not self.gate_up or module.down_proj is not self.down or \
                self.gate_up.requires_grad or self.down.requires_grad:
            raise RuntimeError(f"{self.name}: original expert weights or activation changed")

    def forward(self, hidden_states, top_k_index, top_k_weights):
        pool = self.pool
        pool._check_context()
        self._check_sources()
        if torch.is_grad_enabled():
            raise RuntimeError("Use expert streaming under torch.no_grad() or torch.inference_mode()")
        if (hidden_states.ndim != 2 or hidden_states.device != pool.device or top_k_index.device != pool.device
                or top_k_weights.device != pool.device):
            raise ValueError(f"{self.name}: routed states and indices must be on the pool CUDA device")
        if (hidden_states.dtype != torch.bfloat16 or top_k_index.dtype != torch.long
                or top_k_weights.dtype != torch.bfloat16 or top_k_index.ndim != 2
                or top_k_index.shape != top_k_weights.shape or top_k_index.shape[0] != hidden_states.shape[0]
                or hidden_states.shape[1] != self.module.hidden_dim):
            raise ValueError(f"{self.name}: expected BF16 states [T, H], int64 expert ids and BF16 weights [T, K]")
        pool.stats.layer_calls += 1
        pool.stats.tokens += hidden_states.shape[0]
        counter = {"b200": "b200_layer_calls", "b200-host": "host_layer_calls", "b200-packed": "packed_layer_calls"}
        setattr(pool.stats, counter[self.residency], getattr(pool.stats, counter[self.residency]) + 1)
        return self.run(hidden_states, top_k_index, top_k_weights)

    def run(self, hidden_states, top_k_index, top_k_weights):
        """The device chain itself, shared by the per-path entry points."""
        if hidden_states.shape[0] == 0:
            return torch.zeros_like(hidden_states)
        routed = min(self.module.num_experts, top_k_index.numel())
        layer = self.pool._native_layer(self, top_k_index.shape[1], cache=self.pool.cache_slots(self, routed))
        return layer(hidden_states.contiguous(), route_in=top_k_index.contiguous(),
                     weights_in=top_k_weights.contiguous())


@contextmanager
def patch_experts(model, *, mode, pool):
    """Install one mode on every Qwen3_5MoeExperts module, then restore the
    model's expert forwards (expert_stream.py:457-526)."""
    if mode not in MODES:
        raise ValueError(f"Choose an expert transfer mode from {MODES}")
    if pool._attached:
        raise RuntimeError("The pool already has active expert forwards")
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeExperts

    layers = [_Layer(name, module, pool, mode)
              for name, module in model.named_modules() if type(module) is Qwen3_5MoeExperts]
    if not layers:
        raise ValueError("No Transformers Qwen3_5MoeExperts modules found")
    pool._check_context()
    if RESIDENCY[mode] != "b200":
        layouts = {(tuple(layer.gate_up.shape[1:]), tuple(layer.down.shape[1:])) for layer in layers}
        if len(layouts) != 1:
            raise ValueError("Host-resident expert layers must share one gate/down layout")
    pool._attached = True
    pool._cache_layers = len(layers)
    installed = []
    try:
        for layer in layers:
            layer.module.forward = layer.forward
            installed.append(layer)
        yield pool
    finally:
        for layer in reversed(installed):
            del layer.module.forward
        pool._attached = False
