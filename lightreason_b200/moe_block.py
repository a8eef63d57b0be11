"""Whole-block patch: Qwen3_5MoeSparseMoeBlock.forward on one device chain.

The 35B runner's MoE block (transformers modeling_qwen3_5_moe.py
Qwen3_5MoeSparseMoeBlock.forward, with the expert forward edge35b patches)
is router GEMV -> softmax -> top-8 -> renormalise -> BF16 weights -> eager
routed experts -> + sigmoid(shared gate) * shared expert.  patch_moe_blocks
runs all of it as moe_layer_forward: the router and the shared expert move to
the pool device once, the routed experts keep the residency of the chosen
mode (HBM, pinned host rows, or packed host rows), and no host read happens
inside the forward.  The router weights are rounded to BF16 before the
combine, the contract of the reference's expert forwards
(expert_stream.py:356, fused_experts.py:41-45).
"""

from __future__ import annotations

from contextlib import contextmanager

import torch

from lightreason_b200.expert_stream import MODES, _Layer


class _Block:
    def __init__(self, name, block, pool, mode):
        self.name = name
        self.block = block
        self.pool = pool
        self.experts = _Layer(f"{name}.experts", block.experts, pool, mode)
        gate = block.gate
        if gate.weight.dtype != torch.bfloat16 or tuple(gate.weight.shape) != (
                block.experts.num_experts, block.experts.hidden_dim):
            raise ValueError(f"{name}: expected a BF16 router [experts, hidden]")
        self.top_k = gate.top_k

    def _extra(self):
        dev = self.pool.device
        b = self.block
        t = lambda w: (lambda: w.detach().to(dev).contiguous())  # noqa: E731
        return {"router": t(b.gate.weight), "shared_gate": t(b.shared_expert.gate_proj.weight),
                "shared_up": t(b.shared_expert.up_proj.weight), "shared_down": t(b.shared_expert.down_proj.weight),
                "shared_gate_w": t(b.shared_expert_gate.weight.reshape(-1))}

    def forward(self, hidden_states):
        pool = self.pool
        pool._check_context()
        self.experts._check_sources()
        if torch.is_grad_enabled():
            raise RuntimeError("Use expert streaming under torch.no_grad() or torch.inference_mode()")
        if hidden_states.device != pool.device or hidden_states.dtype != torch.bfloat16:
            raise ValueError(f"{self.name}: hidden states must be BF16 on the pool CUDA device")
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1]).contiguous()
        pool.stats.layer_calls += 1
        pool.stats.tokens += x.shape[0]
        if x.shape[0] == 0:
            return torch.zeros_like(hidden_states)
        routed = min(self.block.experts.num_experts, x.shape[0] * self.top_k)
        layer = pool._native_layer(self.experts, self.top_k, owner=self.block, extra=self._extra(),
                                   cache=pool.cache_slots(self.experts, routed))
        return layer(x).reshape(shape)


@contextmanager
def patch_moe_blocks(model, *, mode="b200", pool):
    """Install the device chain on every Qwen3_5MoeSparseMoeBlock, then
    restore the blocks' forwards."""
    if mode not in MODES:
        raise ValueError(f"Choose an expert transfer mode from {MODES}")
    if pool._attached:
        raise RuntimeError("The pool already has active expert forwards")
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock

    blocks = [_Block(name, module, pool, mode)
              for name, module in model.named_modules() if type(module) is Qwen3_5MoeSparseMoeBlock]
    if not blocks:
        raise ValueError("No Transformers Qwen3_5MoeSparseMoeBlock modules found")
    pool._check_context()
    pool._attached = True
    pool._cache_layers = len(blocks)
    installed = []
    try:
        for b in blocks:
            if "forward" in vars(b.block):
                raise ValueError(f"{b.name}: block forward is already patched")
            b.block.forward = b.forward
            installed.append(b)
        yield pool
    finally:
        for b in reversed(installed):
            del b.block.forward
        pool._attached = False
