"""A small Transformers model holding Qwen3_5MoeSparseMoeBlock layers with the
35B layer widths (hidden 2048, expert inner 512, shared inner 512) and fewer
experts, filled with the seeded synthetic weights, for the drop-in API tests."""

from __future__ import annotations

import numpy as np
import torch

from lightreason_b200 import synthetic as S


def t_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class Stack(torch.nn.Module):
    def __init__(self, blocks):
        super().__init__()
        self.layers = torch.nn.ModuleList(blocks)


def make_model(*, experts: int = 32, layers: int = 2, seed: int = 40):
    """Returns (model, weights per layer as synthetic.LayerWeights)."""
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock

    config = Qwen3_5MoeTextConfig(hidden_size=S.HIDDEN, moe_intermediate_size=S.INNER, num_experts=experts,
                                  num_experts_per_tok=8, shared_expert_intermediate_size=S.INNER)
    config._experts_implementation = "eager"
    blocks, weights = [], []
    for layer in range(layers):
        with torch.device("meta"):
            block = Qwen3_5MoeSparseMoeBlock(config)
        block = block.to_empty(device="cpu").to(torch.bfloat16).eval().requires_grad_(False)
        w = S.layer_weights(seed, layer, bias="none", experts=experts)
        gu, dn = w.stacked()
        with torch.no_grad():
            block.gate.weight.copy_(t_bf16(w.router))
            block.experts.gate_up_proj.copy_(t_bf16(gu))
            block.experts.down_proj.copy_(t_bf16(dn))
            block.shared_expert.gate_proj.weight.copy_(t_bf16(w.sh_gate))
            block.shared_expert.up_proj.weight.copy_(t_bf16(w.sh_up))
            block.shared_expert.down_proj.weight.copy_(t_bf16(w.sh_down))
            block.shared_expert_gate.weight.copy_(t_bf16(w.sh_gate_w).reshape(1, -1))
        blocks.append(block)
        weights.append((w, gu, dn))
    return Stack(blocks).eval().requires_grad_(False), weights
