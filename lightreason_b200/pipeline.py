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

HostStream carries the same idea (copies on a side stream, ordered by per-item
events, overlapped with the computation) to the layer's activations: a run
over many host batches copies batch i + 1 in and batch i - 1 out while batch i
computes.
"""

from __future__ import annotations

import torch


def routed_forward(layer, hidden_states, top_k_index, top_k_weights, *, pipeline=None):
    """Preserve eager expert and per-expert token order, including BF16 adds."""
    return layer.run(hidden_states, top_k_index, top_k_weights)


class HostStream:
    """A step function over a sequence of host batches, with the transfers
    overlapped: batch i + 1 is copied host -> device on one side stream and
    batch i - 1 device -> host on another while `step` runs batch i on the
    current stream.  Device inputs and outputs are `depth`-buffered; fresh
    events order every copy against the steps that use its buffer, so `run`
    can also be captured in a CUDA graph (the side streams join the capture
    through the first event).  Host tensors should be pinned."""

    def __init__(self, shape_in, shape_out, *, dtype=torch.bfloat16, device=None, depth: int = 2):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.depth = depth
        self.x = [torch.empty(shape_in, dtype=dtype, device=self.device) for _ in range(depth)]
        self.out = [torch.empty(shape_out, dtype=dtype, device=self.device) for _ in range(depth)]
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)

    def run(self, step, host_in, host_out) -> None:
        """step(x_dev, out_dev) for every host_in[i] -> host_out[i] (equal
        lengths; entries may repeat, the copies into one host buffer stay in
        order).  Returns once everything is enqueued; the current stream
        waits for the last copy."""
        if len(host_in) != len(host_out):
            raise ValueError("host_in and host_out must have the same length")
        s = torch.cuda.current_stream(self.device)
        fork = torch.cuda.Event()
        fork.record(s)
        self.h2d.wait_event(fork)
        self.d2h.wait_event(fork)
        n, depth = len(host_in), self.depth
        done = [torch.cuda.Event() for _ in range(n)]
        drained = [torch.cuda.Event() for _ in range(n)]
        for i in range(n):
            b = i % depth
            loaded = torch.cuda.Event()
            with torch.cuda.stream(self.h2d):
                if i >= depth:
                    self.h2d.wait_event(done[i - depth])      # step i - depth has read x[b]
                self.x[b].copy_(host_in[i], non_blocking=True)
                loaded.record(self.h2d)
            s.wait_event(loaded)
            if i >= depth:
                s.wait_event(drained[i - depth])               # out[b] of step i - depth is copied out
            step(self.x[b], self.out[b])
            done[i].record(s)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done[i])
                host_out[i].copy_(self.out[b], non_blocking=True)
                drained[i].record(self.d2h)
        s.wait_stream(self.h2d)
        s.wait_stream(self.d2h)
