"""Single-token decode entry point, drop-in for edge35b/fused_experts.py
fused_forward (:40-71).

Same shape contract and errors as the reference: one BF16 token of the 35B
layout ([1, 2048], experts [E, 1024, 2048] / [E, 2048, 512]) with eight
distinct in-range routes and BF16 weights.  The reference checks the routes
on the host (indices.tolist()) before its Triton matvecs; here the check is
the same host read, and the compute is the layer's device chain (grouped
tcgen05 SwiGLU + in-kernel ordered BF16 combine), which produces the eager
result bit for bit.  torch_projections (the reference's "batched" variant)
selects the same arithmetic and is accepted for compatibility.
"""

from __future__ import annotations

import torch


def check_single_token(layer, hidden, indices, weights, message):
    """The 35B single-token shape checks shared by fused_forward and
    cpu_forward (fused_experts.py:41-45, cpu_route.py:24-27)."""
    if (tuple(hidden.shape) != (1, 2048) or tuple(indices.shape) != (1, 8) or tuple(weights.shape) != (1, 8)
            or hidden.dtype != torch.bfloat16 or weights.dtype != torch.bfloat16
            or not hidden.is_contiguous() or not weights.is_contiguous()
            or tuple(layer.gate_up.shape[1:]) != (1024, 2048) or tuple(layer.down.shape[1:]) != (2048, 512)):
        raise ValueError(message)


def check_distinct_routes(layer, indices):
    experts = indices[0].tolist()
    if len(set(experts)) != 8 or not all(0 <= e < layer.module.num_experts for e in experts):
        raise ValueError("Fused expert decode requires eight distinct valid routes")


def fused_forward(layer, hidden, indices, weights, *, torch_projections=False):
    check_single_token(layer, hidden, indices, weights, "Fused expert decode requires the single-token 35B route shape")
    check_distinct_routes(layer, indices)
    return layer.run(hidden, indices, weights)
