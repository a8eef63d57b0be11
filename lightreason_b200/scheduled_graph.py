"""CUDA-graph replay of the patched expert operator at decode widths.

Drop-in for edge35b/scheduled_graph.py `replay_experts` (:66-140).  The
reference stages the eight selected experts' rows with a Triton kernel and
replays one captured Scheduled forward, after reading the ids on the host.
Here the whole device chain of a patched layer (routing given, staging,
grouped products, combine) already runs without a host round trip, so a
graph per (layer, token width) replaces every launch of the call by one
graph launch: while the context is active, each patched
`Qwen3_5MoeExperts.forward` on `pool` with at most `max_tokens` tokens copies
its inputs into the graph's static buffers and replays it.  Other calls take
the ordinary path.

As in the reference, the returned tensor is the graph's static output: it is
valid until the next replay of the same layer at the same width.  Graphs
persist on the pool (`pool.replay_graphs`) across contexts; `pool.clear()`
releases the native layers they use, so clear the graphs first
(`release_graphs(pool)`).
"""

from __future__ import annotations

from contextlib import contextmanager

import torch

from lightreason_b200.expert_stream import _Layer


class _Replay:
    """One captured expert call: static inputs, the graph, its output."""

    def __init__(self, layer, run, hidden, indices, weights, memory):
        self.hidden = hidden.detach().clone()
        self.indices = indices.detach().clone()
        self.weights = weights.detach().clone()
        run(layer, self.hidden, self.indices, self.weights)  # builds the native layer and its workspace
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=memory):
            self.output = run(layer, self.hidden, self.indices, self.weights)

    def __call__(self, hidden, indices, weights):
        self.hidden.copy_(hidden)
        self.indices.copy_(indices)
        self.weights.copy_(weights)
        self.graph.replay()
        return self.output


def release_graphs(pool) -> None:
    """Drop the pool's captured expert graphs."""
    graphs = getattr(pool, "replay_graphs", None)
    if graphs:
        graphs.clear()


@contextmanager
def replay_experts(pool, *, max_tokens: int = 16):
    """Serve the patched expert forwards of `pool` from captured graphs."""
    if not 0 < max_tokens <= 64:
        raise ValueError("max_tokens must be in [1, 64]")
    if not hasattr(pool, "replay_graphs"):
        pool.replay_graphs = {}
        pool.replay_graph_memory = torch.cuda.graph_pool_handle()
    original = _Layer.run

    def run(layer, hidden, indices, weights):
        tokens = hidden.shape[0]
        # (inside a capture of the caller's own, the ordinary launches are recorded instead)
        if layer.pool is not pool or not 0 < tokens <= max_tokens or torch.cuda.is_current_stream_capturing():
            return original(layer, hidden, indices, weights)
        key = (id(layer.module), layer.residency, tokens, indices.shape[1])
        entry = pool.replay_graphs.get(key)
        if entry is None:
            entry = pool.replay_graphs[key] = _Replay(layer, original, hidden, indices, weights,
                                                      pool.replay_graph_memory)
        pool.stats.replayed_layer_calls += 1
        return entry(hidden, indices, weights)

    _Layer.run = run
    try:
        yield pool
    finally:
        _Layer.run = original
