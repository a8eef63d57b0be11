"""Routed multi-token forward, drop-in for edge35b/pipeline.py routed_forward
(:79-111).

The reference walks the routed experts in groups of eight, copying each
group's rows over PCIe (optionally double-buffered by TransferPipeline) and
index_add-ing the weighted BF16 contributions in ascending expert order.  The
B200 layer chain does the same grouping on the device: the selected rows are
staged into HBM slots by one kernel while the grouped SwiGLU kernel consumes
them, and the combine keeps the eager ascending-expert BF16 order.  The
`pipeline` argument is accepted for compatibility; the overlap it provided is
built into the chain.
"""

from __future__ import annotations


def routed_forward(layer, hidden_states, top_k_index, top_k_weights, *, pipeline=None):
    """Preserve eager expert and per-expert token order, including BF16 adds."""
    return layer.run(hidden_states, top_k_index, top_k_weights)
