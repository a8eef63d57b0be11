"""Multi-position verifier entry point, drop-in for edge35b/block_experts.py
grouped_block (:89-137).

Same contract as the reference: 2-16 contiguous BF16 positions of width 2048
with eight routes each.  The reference groups the positions by expert on the
host (indices.tolist()) and runs two Triton projections plus an ordered
combine; here the grouping is the device permute and the projections are the
grouped tcgen05 kernel with its fused combine -- no host read of the routes.
"""

from __future__ import annotations


def grouped_block(layer, hidden, indices, weights):
    count, width = hidden.shape
    if not 2 <= count <= 16 or width != 2048 or tuple(indices.shape) != (count, 8):
        raise ValueError("Grouped expert verification needs 2–16 Qwen3.6 target positions")
    if not hidden.is_contiguous() or not weights.is_contiguous():
        raise ValueError("Grouped expert verification requires contiguous target activations")
    return layer.run(hidden, indices, weights)
