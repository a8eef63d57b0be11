"""CUDA-graph replay of the single-token mixers around the MoE layers.

Drop-in for edge35b/packed_native.py `mixer_graphs` and `StaticMixerCache`
(:77-150): the step on either side of the MoE layer at decode.  Each Gated
DeltaNet mixer (`decoder_layer.linear_attn`) of the model, called with one
token and a cache that already holds its state, is captured once per layer
into a CUDA graph over static conv / recurrent state buffers; every later
such call copies the live request's state in, replays, and copies the next
state back out, so the captured addresses serve any request.  Other calls
(prefill, no cache, an attention mask) take the original forward, and so does
a mixer whose kernels cannot be captured (Transformers' pure-torch fallback,
used when the flash-linear-attention kernels are not installed, copies from
pageable host memory inside the step).

The rest of the reference's packed_native.py (the Ada Triton matvecs and the
CPU packed workers) is what the MoE layer of this package replaces.
"""

from __future__ import annotations

from contextlib import contextmanager
from types import SimpleNamespace

import torch


class StaticMixerCache:
    """The cache a captured mixer graph reads and writes: static state
    buffers of one layer, shaped like the live ones, with the methods the
    mixer's single-token path calls."""

    def __init__(self, layer_index: int, source):
        self.layers = {layer_index: SimpleNamespace(conv_states=torch.empty_like(source.conv_states),
                                                    recurrent_states=torch.empty_like(source.recurrent_states))}

    def has_previous_state(self, _index) -> bool:
        return True

    def update_recurrent_state(self, state, index):
        buf = self.layers[index].recurrent_states
        buf.copy_(state)  # the captured output must land in the static buffer
        return buf


class _MixerReplay:
    def __init__(self, forward, index, hidden_states, live, memory):
        self.index = index
        self.cache = StaticMixerCache(index, live)
        self.state = self.cache.layers[index]
        self.input = torch.empty_like(hidden_states)
        self._load(hidden_states, live)
        forward(self.input, cache_params=self.cache, attention_mask=None)  # warm-up outside the capture
        self._load(hidden_states, live)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=memory):
            self.output = forward(self.input, cache_params=self.cache, attention_mask=None)

    def _load(self, hidden_states, live):
        self.input.copy_(hidden_states)
        self.state.conv_states.copy_(live.conv_states)
        self.state.recurrent_states.copy_(live.recurrent_states)

    def __call__(self, hidden_states, live):
        self._load(hidden_states, live)
        self.graph.replay()
        live.conv_states.copy_(self.state.conv_states)
        live.recurrent_states.copy_(self.state.recurrent_states)
        return self.output


def _capturable(mixer) -> bool:
    """False for a mixer running Transformers' pure-torch recurrent fallback,
    whose step allocates on the host and copies to the device."""
    rule = getattr(mixer, "recurrent_gated_delta_rule", None)
    return not getattr(rule, "__name__", "").startswith("torch_")


@contextmanager
def mixer_graphs(model, pool):
    """Replay single-token Gated DeltaNet mixers of `model` (layers at
    `model.model.layers`) from per-layer CUDA graphs kept on `pool`."""
    if not hasattr(pool, "mixer_graphs"):
        pool.mixer_graphs = {}
        pool.mixer_graph_memory = torch.cuda.graph_pool_handle()
    graphs = pool.mixer_graphs
    installed = []

    def bind(mixer, forward, index):
        def replayed(hidden_states, cache_params=None, attention_mask=None):
            if (hidden_states.shape[:2] != (1, 1) or cache_params is None or attention_mask is not None
                    or not cache_params.has_previous_state(index) or torch.cuda.is_current_stream_capturing()):
                return forward(hidden_states, cache_params=cache_params, attention_mask=attention_mask)
            live = cache_params.layers[index]
            if index not in graphs and not _capturable(mixer):
                graphs[index] = None
            if index not in graphs:
                try:
                    graphs[index] = _MixerReplay(forward, index, hidden_states, live, pool.mixer_graph_memory)
                except RuntimeError:
                    # a step that cannot be captured keeps its ordinary forward
                    graphs[index] = None
            entry = graphs[index]
            if entry is None:
                return forward(hidden_states, cache_params=cache_params, attention_mask=attention_mask)
            if hasattr(pool, "stats"):
                pool.stats.mixer_replays += 1
            return entry(hidden_states, live)
        return replayed

    try:
        for index, layer in enumerate(model.model.layers):
            mixer = getattr(layer, "linear_attn", None)
            if mixer is None:
                continue
            installed.append((mixer, mixer.__dict__.get("forward")))
            mixer.forward = bind(mixer, mixer.forward, getattr(mixer, "layer_idx", index))
        yield pool
    finally:
        for mixer, previous in reversed(installed):
            if previous is None:
                del mixer.forward
            else:
                mixer.forward = previous
