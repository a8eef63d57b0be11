"""The drop-in API mirror on the GPU: patched Qwen3_5MoeExperts forwards in
every residency, the per-path entry points, the whole-block patch and the
resident tile arena, against the oracle and against each other.

Residencies run the same kernels on the same rows, so their outputs are
compared bit for bit; against the oracle the tolerance is helpers.assert_close
(max-abs 2e-2, rel-L2 1e-2).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from lightreason_b200 import block_experts, build, cpu_route, expert_stream, fused_experts, moe_block, native
from lightreason_b200 import gpu_resident_experts as gre
from lightreason_b200 import pipeline
from lightreason_b200 import synthetic as S
from oracle import oracle as O
from tests.helpers import assert_close

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
    x = S.hidden_states(seed, tokens)
    return x, idx, wts, (to_dev(x, dev), torch.from_numpy(idx).to(dev), to_dev(wts, dev))


def oracle_experts(weights, x, idx, wts):
    _, gu, dn = weights
    offsets, ptok, _, rpos = O.permute(idx, EXPERTS)
    return O.combine(O.experts_by_route(x, gu, dn, offsets, ptok, EXPERTS), rpos, wts)


@pytest.mark.parametrize("tokens", [1, 12])
def test_patched_experts_every_residency(dev, model, tokens):
    net, weights = model
    x, idx, wts, args = routes(tokens, 500 + tokens, dev)
    outs = {}
    for mode in ("b200", "b200-host", "b200-packed", "fused", "cached", "packed"):
        pool = expert_stream.ExpertPool(dev)
        with torch.no_grad(), expert_stream.patch_experts(net, mode=mode, pool=pool):
            outs[mode] = [bits(layer.experts(*args)) for layer in net.layers]
        assert all("forward" not in vars(layer.experts) for layer in net.layers)
        assert pool.stats.layer_calls == 2 and pool.stats.tokens == 2 * tokens
        pool.clear()
    for mode, got in outs.items():
        for a, b in zip(got, outs["b200"]):
            assert np.array_equal(a, b), mode
    for layer, w in enumerate(weights):
        assert_close(outs["b200"][layer], oracle_experts(w, x, idx, wts), what=f"patched layer {layer}")


def test_capacity_bytes_caches_experts(dev, model):
    """ExpertPool(capacity_bytes=...) on the host residencies: a device expert
    cache per layer; repeated calls hit it and stay bit-identical to HBM."""
    net, _ = model
    want = {}
    pool = expert_stream.ExpertPool(dev)
    with torch.no_grad(), expert_stream.patch_experts(net, mode="b200", pool=pool):
        for seed in (800, 801, 800):
            want[seed] = bits(net.layers[0].experts(*routes(3, seed, dev)[3]))
    pool.clear()
    for mode in ("cached", "b200-packed"):
        # 24 of the 32 experts per layer: the budget is shared by the 2 layers
        pool = expert_stream.ExpertPool(dev, capacity_bytes=2 * 24 * 6291456)
        with torch.no_grad(), expert_stream.patch_experts(net, mode=mode, pool=pool):
            for seed in (800, 801, 800):
                got = bits(net.layers[0].experts(*routes(3, seed, dev)[3]))
                assert np.array_equal(got, want[seed]), (mode, seed)
        layer = next(v for k, v in pool._layers.items() if k[2])
        assert layer.cache_slots == 24
        st = layer.cache_stats()
        assert st["calls"] == 3 and st["misses"] < st["uses"], st
        pool.clear()


def test_per_path_entry_points_are_the_patched_forward(dev, model):
    net, _ = model
    pool = expert_stream.ExpertPool(dev)
    layer = expert_stream._Layer("layers.0.experts", net.layers[0].experts, pool, "b200")
    with torch.no_grad():
        _, _, _, one = routes(1, 601, dev)
        want = bits(layer.forward(*one))
        assert np.array_equal(bits(fused_experts.fused_forward(layer, *one)), want)
        assert np.array_equal(bits(fused_experts.fused_forward(layer, *one, torch_projections=True)), want)
        assert np.array_equal(bits(cpu_route.cpu_forward(layer, *one)), want)
        _, _, _, many = routes(9, 602, dev)
        want = bits(layer.forward(*many))
        assert np.array_equal(bits(block_experts.grouped_block(layer, *many)), want)
        assert np.array_equal(bits(pipeline.routed_forward(layer, *many)), want)


def test_pool_refuses_other_streams(dev, model):
    net, _ = model
    pool = expert_stream.ExpertPool(dev)
    _, _, _, args = routes(2, 603, dev)
    with torch.no_grad(), expert_stream.patch_experts(net, mode="b200", pool=pool):
        net.layers[0].experts(*args)
        with torch.cuda.stream(torch.cuda.Stream(dev)), pytest.raises(RuntimeError, match="original CUDA thread"):
            net.layers[0].experts(*args)
    with pytest.raises(RuntimeError, match="torch.no_grad"), expert_stream.patch_experts(net, mode="b200", pool=pool):
        net.layers[0].experts(*args)


@pytest.mark.parametrize("tokens", [1, 16, 80])
def test_patched_moe_block(dev, model, tokens):
    """Whole SparseMoeBlock: router, top-8, experts and gated shared expert on
    one chain; bit-identical to moe_layer_forward called directly, and within
    tolerance of the oracle given the device's own routes."""
    net, weights = model
    w, gu, dn = weights[0]
    x = S.hidden_states(700 + tokens, tokens)
    xd = to_dev(x, dev)
    outs = {}
    for mode in ("b200", "b200-packed"):
        pool = expert_stream.ExpertPool(dev)
        with torch.no_grad(), moe_block.patch_moe_blocks(net, mode=mode, pool=pool):
            outs[mode] = bits(net.layers[0](xd.reshape(1, tokens, -1)).reshape(tokens, -1))
        assert "forward" not in vars(net.layers[0])
        pool.clear()
    assert np.array_equal(outs["b200"], outs["b200-packed"])
    d = lambda a: to_dev(a, dev)  # noqa: E731
    direct = native.Layer(router=d(w.router), gate_up=d(gu), down=d(dn), shared_gate=d(w.sh_gate),
                          shared_up=d(w.sh_up), shared_down=d(w.sh_down), shared_gate_w=d(w.sh_gate_w))
    idx = torch.empty((tokens, 8), dtype=torch.int64, device=dev)
    sc = torch.empty((tokens, 8), dtype=torch.bfloat16, device=dev)
    out = bits(direct(xd, idx_out=idx, scores_out=sc))
    assert np.array_equal(out, outs["b200"])
    idx, sc = idx.cpu().numpy(), bits(sc)
    offsets, ptok, _, rpos = O.permute(idx, EXPERTS)
    y = O.experts_by_route(x, gu, dn, offsets, ptok, EXPERTS)
    sh, sig = O.shared_expert(x, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)
    assert_close(out, O.combine(y, rpos, sc, sh, sig), what="patched block")


def test_resident_arena_layouts_audit(dev, model):
    _, weights = model
    _, gu, dn = weights[1]
    t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    arena = gre.ResidentArena([t(gu), t(dn)], experts=[0, 5, 31], device=dev)
    for mode in ("raw", "packed", "raw"):
        arena.select(mode)
        assert arena.audit() == 3 * (gu[0].size + dn[0].size)
    assert arena.used["packed"] < arena.used["raw"]


def test_device_rows_descriptors(dev, model):
    _, weights = model
    _, gu, _ = weights[0]
    raw = to_dev(gu[:4], dev)
    desc, owners, total = gre.device_rows([gu[e] for e in range(4)], raw)
    assert desc.shape == (4, 3) and total < raw.numel() * 2
    out = torch.empty_like(raw[0])
    dests = torch.tensor([out.data_ptr()], device=dev, dtype=torch.int64)
    sizes = torch.tensor([out.numel() * 2], device=dev, dtype=torch.int64)
    one = torch.ones(1, device=dev, dtype=torch.int64)
    from lightreason_b200.native_bf16_gather import NativeBf16Gather

    for e in range(4):
        src = torch.tensor([e], device=dev, dtype=torch.int32)
        zero = torch.zeros(1, device=dev, dtype=torch.int32)
        NativeBf16Gather().copy(desc.reshape(1, 4, 3), dests, sizes, src, zero, one, max_copies=1, experts=4,
                                geometry=gre.GEOMETRY)
        assert np.array_equal(bits(out), gu[e])
