"""CUDA-graph replay around the MoE layer on the GPU.

* scheduled_graph.replay_experts: patched expert forwards served from a graph
  per (layer, width) give the ordinary path's bits, on reuse with new inputs
  too, in the HBM and packed host residencies.
* Whole-stack capture: the patched blocks of a two-layer stack captured as
  one caller-owned CUDA graph and replayed on new tokens equal eager (the
  layer chain has no host round trip; the reference's Scheduled path reads
  the ids on the host and cannot be captured whole); three 35B-shaped layers
  at the configs[2] width captured as one graph match the oracle on every
  replay.
* packed_native.mixer_graphs: single-token mixers replayed from per-layer
  graphs keep outputs and the live cache state bit-identical to the mixer's
  own forward over several decode steps (a capturable stand-in with the
  Gated DeltaNet cache protocol), and Transformers' Gated DeltaNet itself
  gives its own forward's bits whether or not its kernels capture.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from lightreason_b200 import build, expert_stream, moe_block, native, packed_native, scheduled_graph
from lightreason_b200 import synthetic as S

pytestmark = pytest.mark.gpu
EXPERTS = 32


def bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def to_dev(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)


@pytest.fixture(scope="module")
def dev():
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    native.device_check(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def model():
    from tests.dropin_model import make_model

    return make_model(experts=EXPERTS, layers=2)


def routes(tokens: int, seed: int, dev):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.choice(EXPERTS, 8, replace=False) for _ in range(tokens)]).astype(np.int64)
    wts = S.f32_to_bf16_bits(rng.dirichlet(np.ones(8), size=tokens).astype(np.float32))
    return to_dev(S.hidden_states(seed, tokens), dev), torch.from_numpy(idx).to(dev), to_dev(wts, dev)


@pytest.mark.parametrize("mode", ["b200", "b200-packed"])
def test_replay_experts_equals_ordinary_path(dev, model, mode):
    net, _ = model
    cases = [routes(t, 700 + 10 * t + k, dev) for t in (1, 3) for k in range(2)]
    pool = expert_stream.ExpertPool(dev)
    with torch.no_grad(), expert_stream.patch_experts(net, mode=mode, pool=pool):
        want = [[bits(layer.experts(*args)) for layer in net.layers] for args in cases]
        with scheduled_graph.replay_experts(pool):
            got = [[bits(layer.experts(*args)) for layer in net.layers] for args in cases]
            assert pool.stats.replayed_layer_calls == 2 * len(cases)
            assert len(pool.replay_graphs) == 4          # 2 layers x widths 1 and 3
        assert expert_stream._Layer.run is not None
        again = [bits(layer.experts(*cases[0])) for layer in net.layers]
    for w, g in zip(want, got):
        for a, b in zip(w, g):
            assert np.array_equal(a, b)
    assert all(np.array_equal(a, b) for a, b in zip(want[0], again))
    scheduled_graph.release_graphs(pool)
    pool.clear()


def test_whole_stack_graph_equals_eager(dev, model):
    net, _ = model
    pool = expert_stream.ExpertPool(dev)
    blocks = [layer for layer in net.layers]
    tokens = 4
    with torch.no_grad(), moe_block.patch_moe_blocks(net, mode="b200", pool=pool):
        def step(x):
            for b in blocks:
                x = b(x[None])[0]   # the block takes [batch, seq, H]
            return x

        xs = [to_dev(S.hidden_states(900 + i, tokens), dev) for i in range(3)]
        want = [bits(step(x)) for x in xs]
        static = xs[0].clone()
        step(static)  # warm every native layer and workspace before the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = step(static)
        for x, w in zip(xs, want):
            static.copy_(x)
            g.replay()
            torch.cuda.synchronize()
            assert np.array_equal(bits(out), w)
        del g
    pool.clear()


def test_stack_graph_replay_matches_oracle(dev):
    """configs[2] in miniature: three layers at the 35B shapes (256 experts,
    Zipf(1.1) routing, each with its own weights) at the decode width B = 64,
    captured as one CUDA graph over static input buffers and replayed on two
    new batches; every layer's ids (tier 2) and outputs of every replay
    against the oracle."""
    from oracle import oracle as O
    from tests.helpers import assert_close, compare_ids

    tokens, n_layers = 64, 3
    ws, layers = [], []
    for li in range(n_layers):
        w = S.layer_weights(2000 + li, layer=li, bias="zipf")
        gu, dn = w.stacked()
        for e in range(256):
            w.gate_up[e], w.down[e] = gu[e], dn[e]
        layers.append(native.Layer(router=to_dev(w.router, dev), gate_up=to_dev(gu, dev), down=to_dev(dn, dev),
                                   bias=torch.from_numpy(w.bias).to(dev), shared_gate=to_dev(w.sh_gate, dev),
                                   shared_up=to_dev(w.sh_up, dev), shared_down=to_dev(w.sh_down, dev),
                                   shared_gate_w=to_dev(w.sh_gate_w, dev)))
        ws.append(w)
    static = [torch.zeros((tokens, 2048), dtype=torch.bfloat16, device=dev) for _ in layers]
    outs = [torch.empty_like(x) for x in static]
    idxs = [torch.empty((tokens, 8), dtype=torch.int64, device=dev) for _ in layers]
    lgs = [torch.empty((tokens, 256), dtype=torch.bfloat16, device=dev) for _ in layers]

    def step():
        for layer, x, o, i, lg in zip(layers, static, outs, idxs, lgs):
            layer(x, out=o, idx_out=i, logits_out=lg)

    step()  # workspaces exist before the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for rep in range(2):
        xs = [S.hidden_states(3000 + 10 * rep + li, tokens) for li in range(n_layers)]
        for x, b in zip(static, xs):
            x.copy_(to_dev(b, dev))
        g.replay()
        torch.cuda.synchronize()
        for li, (w, b) in enumerate(zip(ws, xs)):
            w_out, w_idx, _, w_lg = O.moe_layer(b, w.router, w.bias, w.gate_up, w.down, w.sh_gate, w.sh_up,
                                                w.sh_down, w.sh_gate_w)
            idx = idxs[li].cpu().numpy()
            assert_close(bits(lgs[li]), w_lg, what=f"replay {rep} layer {li} logits")
            compare_ids(idx, w_idx, S.bf16_bits_to_f32(w_lg) + w.bias, slack_ulps=1.0,
                        case=f"stack replay {rep} layer {li} T={tokens}")
            same = np.all(idx == w_idx, axis=1)
            assert same.mean() > 0.9
            assert_close(bits(outs[li])[same], w_out[same], what=f"replay {rep} layer {li} output")
    del g


class _LiveCache:
    """The part of the Transformers cache the single-token mixer path uses."""

    def __init__(self, index, conv, rec):
        self.layers = {index: SimpleNamespace(conv_states=conv, recurrent_states=rec)}

    def has_previous_state(self, _index):
        return True

    def update_recurrent_state(self, state, index):
        self.layers[index].recurrent_states = state
        return state


class _StandInMixer(torch.nn.Module):
    """A single-token mixer with the Gated DeltaNet cache protocol: the conv
    state is updated in place, the next recurrent state goes through
    cache_params.update_recurrent_state; all of it capturable."""

    def __init__(self, hidden, width, kernel, layer_idx, gen, dev):
        super().__init__()
        self.layer_idx = layer_idx
        rnd = lambda *s: (torch.randn(*s, generator=gen, device=dev) * 0.05).to(torch.bfloat16)  # noqa: E731
        self.w_in, self.w_out, self.w_conv = rnd(width, hidden), rnd(hidden, width), rnd(width, kernel)

    def forward(self, hidden_states, cache_params=None, attention_mask=None):
        state = cache_params.layers[self.layer_idx]
        v = hidden_states[:, 0] @ self.w_in.t()                             # [1, width]
        window = torch.cat([state.conv_states[:, :, 1:], v[:, :, None]], dim=-1)
        state.conv_states.copy_(window)
        c = (window * self.w_conv).sum(-1).float()                          # [1, width]
        rec = state.recurrent_states * 0.9 + c[:, :, None] * c[:, None, :]
        rec = cache_params.update_recurrent_state(rec, self.layer_idx)
        y = (rec @ c[:, :, None])[:, :, 0].to(torch.bfloat16)
        return (y @ self.w_out.t())[:, None]


def _run_mixers(model, caches, steps):
    outs = []
    for x in steps:
        for i, layer in enumerate(model.model.layers):
            x = layer.linear_attn(x, cache_params=caches[i])
        torch.cuda.synchronize()
        outs.append(x.clone())
    return outs


def _caches(states):
    return [_LiveCache(i, c.clone(), r.clone()) for i, (c, r) in enumerate(states)]


def test_mixer_graphs_replay_stand_in(dev):
    g = torch.Generator(device=dev).manual_seed(6)
    mixers = [_StandInMixer(256, 64, 4, i, g, dev) for i in range(3)]
    model = SimpleNamespace(model=SimpleNamespace(layers=[SimpleNamespace(linear_attn=m) for m in mixers]))
    states = [(torch.randn(1, 64, 4, generator=g, device=dev).to(torch.bfloat16),
               torch.randn(1, 64, 64, generator=g, device=dev)) for _ in mixers]
    steps = [torch.randn(1, 1, 256, generator=g, device=dev).to(torch.bfloat16) for _ in range(4)]
    eager, replay = _caches(states), _caches(states)
    pool = SimpleNamespace(stats=expert_stream.TransferStats())
    with torch.no_grad():
        want = _run_mixers(model, eager, steps)
        with packed_native.mixer_graphs(model, pool):
            got = _run_mixers(model, replay, steps)
        assert all("forward" not in vars(m) for m in mixers)
    assert pool.stats.mixer_replays == len(mixers) * len(steps)
    assert all(pool.mixer_graphs[i] is not None for i in range(len(mixers)))
    for w, o in zip(want, got):
        assert torch.equal(w, o)
    for a, b in zip(eager, replay):
        i = next(iter(a.layers))
        assert torch.equal(a.layers[i].conv_states, b.layers[i].conv_states)
        assert torch.equal(a.layers[i].recurrent_states, b.layers[i].recurrent_states)
    # with the pure-torch fallback kernels (no flash-linear-attention here)
    # the mixers are not captured and keep their own forward
    fallback = not packed_native._capturable(mixers[0])
    assert (pool.stats.mixer_replays == 0) == fallback


def test_mixer_graphs_gated_deltanet(dev):
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeGatedDeltaNet

    cfg = Qwen3_5MoeTextConfig(hidden_size=256, linear_num_value_heads=4, linear_num_key_heads=2,
                               linear_key_head_dim=32, linear_value_head_dim=32, linear_conv_kernel_dim=4)
    torch.manual_seed(5)
    mixers = [Qwen3_5MoeGatedDeltaNet(cfg, layer_idx=i).to(dev, torch.bfloat16).eval() for i in range(2)]
    model = SimpleNamespace(model=SimpleNamespace(layers=[SimpleNamespace(linear_attn=m) for m in mixers]))
    conv_dim, kernel = mixers[0].conv1d.weight.shape[0], mixers[0].conv_kernel_size
    rec_shape = (1, mixers[0].num_v_heads, mixers[0].head_k_dim, mixers[0].head_v_dim)
    g = torch.Generator(device=dev).manual_seed(6)
    states = [(torch.randn(1, conv_dim, kernel, generator=g, device=dev).to(torch.bfloat16),
               torch.randn(rec_shape, generator=g, device=dev)) for _ in mixers]
    steps = [torch.randn(1, 1, 256, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
    eager, replay = _caches(states), _caches(states)
    pool = SimpleNamespace(stats=expert_stream.TransferStats())
    with torch.no_grad():
        want = _run_mixers(model, eager, steps)
        with packed_native.mixer_graphs(model, pool):
            got = _run_mixers(model, replay, steps)
    for w, o in zip(want, got):
        assert torch.equal(w, o)
    for a, b in zip(eager, replay):
        i = next(iter(a.layers))
        assert torch.equal(a.layers[i].conv_states, b.layers[i].conv_states)
        assert torch.equal(a.layers[i].recurrent_states, b.layers[i].recurrent_states)
    # with the pure-torch fallback kernels (no flash-linear-attention here)
    # the mixers are not captured and keep their own forward
    fallback = not packed_native._capturable(mixers[0])
    assert (pool.stats.mixer_replays == 0) == fallback
