"""Parity of the CUDA layer path against the CPU oracle (GPU only).

Ids and per-expert token orders are compared bit-exactly (tier 1: selection on
the oracle's own logits; tier 2: end-to-end, where only a near tie may move),
outputs within max-abs 2e-2 / rel-L2 1e-2 (helpers.assert_close).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from lightreason_b200 import build, native
from lightreason_b200 import synthetic as S
from oracle import oracle as O
from tests.helpers import assert_close, compare_ids, golden_layers, load_golden

pytestmark = pytest.mark.gpu


def to_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def dev():
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    native.device_check(0)
    return torch.device("cuda", 0)


class Case:
    def __init__(self, seed: int, bias: str, dev, *, host_resident: bool = False):
        self.w = S.layer_weights(seed, bias=bias)
        self.gu, self.dn = self.w.stacked()
        for e in range(256):
            self.w.gate_up[e], self.w.down[e] = self.gu[e], self.dn[e]
        self.seed = seed
        d = lambda a: to_dev(a, dev)  # noqa: E731
        self.router, self.sh = d(self.w.router), [d(self.w.sh_gate), d(self.w.sh_up), d(self.w.sh_down),
                                                  d(self.w.sh_gate_w)]
        self.bias = torch.from_numpy(self.w.bias).to(dev) if self.w.bias is not None else None
        self.gu_dev, self.dn_dev = d(self.gu), d(self.dn)
        self.layer = native.Layer(router=self.router, gate_up=self.gu_dev, down=self.dn_dev, bias=self.bias,
                                  shared_gate=self.sh[0], shared_up=self.sh[1], shared_down=self.sh[2],
                                  shared_gate_w=self.sh[3])
        self.dev = dev

    def packed_layer(self):
        banks = native.PackedHostBanks(self.gu, self.dn, self.dev)
        return native.Layer(router=self.router, bias=self.bias, shared_gate=self.sh[0], shared_up=self.sh[1],
                            shared_down=self.sh[2], shared_gate_w=self.sh[3], host_packed=banks)

    def host_layer(self):
        hg = torch.from_numpy(self.gu.view(np.int16)).view(torch.bfloat16).pin_memory()
        hd = torch.from_numpy(self.dn.view(np.int16)).view(torch.bfloat16).pin_memory()
        return native.Layer(router=self.router, bias=self.bias, shared_gate=self.sh[0], shared_up=self.sh[1],
                            shared_down=self.sh[2], shared_gate_w=self.sh[3], host_gate_up=hg, host_down=hd)

    def run(self, x_bits, layer=None):
        x = to_dev(x_bits, self.dev)
        tokens = x.shape[0]
        idx = torch.empty((tokens, 8), dtype=torch.int64, device=self.dev)
        sc = torch.empty((tokens, 8), dtype=torch.bfloat16, device=self.dev)
        lg = torch.empty((tokens, 256), dtype=torch.bfloat16, device=self.dev)
        out = (layer or self.layer)(x, idx_out=idx, scores_out=sc, logits_out=lg)
        torch.cuda.synchronize()
        return bits(out), idx.cpu().numpy(), bits(sc), bits(lg)

    def oracle(self, x_bits):
        w = self.w
        return O.moe_layer(x_bits, w.router, w.bias, w.gate_up, w.down, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)


@pytest.fixture(scope="module")
def case13(dev):
    return Case(13, "normal", dev)


@pytest.fixture(scope="module")
def case14(dev):
    return Case(14, "zipf", dev)


def test_router_select_tier1_exact(dev, case13):
    x = S.hidden_states(101, 64)
    logits = O.linear_bf16(x, case13.w.router)
    want_idx, want_f32, want_bf16 = O.router_select(logits, case13.w.bias)
    idx, sf, sb = native.router_select(to_dev(logits, dev), case13.bias)
    assert np.array_equal(idx.cpu().numpy(), want_idx)
    np.testing.assert_allclose(sf.cpu().numpy(), want_f32, rtol=2e-6, atol=1e-7)
    assert_close(bits(sb), want_bf16, max_abs=1e-2, rel_l2=1e-3, what="scores")


def test_router_select_exact_ties_take_lower_ids(dev):
    logits = np.full((3, 256), 0x3F80, dtype=np.uint16)       # all equal
    logits[1, [5, 9, 200]] = 0x4000                          # three winners, then ties
    logits[2, ::2] = 0x4000                                  # every even id ties on top
    idx, _, sb = native.router_select(to_dev(logits, dev), None)
    got = idx.cpu().numpy()
    want, _, want_sb = O.router_select(logits, None)
    assert np.array_equal(got, want)
    assert got[0].tolist() == list(range(8))
    assert got[1].tolist() == [5, 9, 200, 0, 1, 2, 3, 4]
    assert got[2].tolist() == [0, 2, 4, 6, 8, 10, 12, 14]


@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("tokens,experts,top_k", [(1, 256, 8), (16, 256, 8), (333, 256, 8), (4096, 256, 8),
                                                   (50, 1024, 4), (7, 64, 8), (8192, 256, 8), (3000, 1024, 1),
                                                   (2000, 16, 2)])
def test_permute_bit_exact(dev, tokens, experts, top_k, wide):
    rng = np.random.default_rng(tokens * 7 + experts)
    p = rng.zipf(1.1, size=experts * 4).astype(np.float64)
    p = p[:experts] / p[:experts].sum()
    idx = np.stack([rng.choice(experts, size=top_k, replace=False, p=p) for _ in range(tokens)]).astype(np.int64)
    want = O.permute(idx, experts)
    off, ptok, pslot, rpos, active, n_active, bad = native.permute(torch.from_numpy(idx).to(dev), experts, wide=wide)
    torch.cuda.synchronize()
    assert np.array_equal(off.cpu().numpy(), want[0])
    assert np.array_equal(ptok.cpu().numpy(), want[1])
    assert np.array_equal(pslot.cpu().numpy(), want[2])
    assert np.array_equal(rpos.cpu().numpy(), want[3])
    n = int(n_active.item())
    assert active[:n].cpu().numpy().tolist() == sorted(set(idx.reshape(-1).tolist()))
    assert int(bad.item()) == 0


@pytest.mark.parametrize("wide", [False, True])
def test_permute_drops_out_of_range_ids_at_width(dev, wide):
    """Dropped ids at 4096 routes (the wide path's size): the valid routes keep
    the eager order (ascending expert, slot-major, token) and no position."""
    experts, tokens, top_k = 64, 1024, 4
    rng = np.random.default_rng(5)
    idx = rng.integers(0, experts, size=(tokens, top_k)).astype(np.int64)
    idx[3, 1], idx[100, 0], idx[777, 3], idx[1023, 0] = -1, experts, 1000, -5
    r_t, r_k = np.tile(np.arange(tokens), top_k), np.repeat(np.arange(top_k), tokens)
    e = idx[r_t, r_k]
    valid = (e >= 0) & (e < experts)
    order = np.argsort(np.where(valid, e, experts), kind="stable")[:int(valid.sum())]
    want_pos = np.full((tokens, top_k), -1, dtype=np.int32)
    want_pos[r_t[order], r_k[order]] = np.arange(order.size)
    want_off = np.concatenate(([0], np.cumsum(np.bincount(e[valid], minlength=experts))))
    off, ptok, pslot, rpos, active, n_active, bad = native.permute(torch.from_numpy(idx).to(dev), experts, wide=wide)
    torch.cuda.synchronize()
    assert int(bad.item()) == 4
    assert np.array_equal(off.cpu().numpy(), want_off)
    assert np.array_equal(ptok.cpu().numpy()[:order.size], r_t[order])
    assert np.array_equal(pslot.cpu().numpy()[:order.size], r_k[order])
    assert np.array_equal(rpos.cpu().numpy(), want_pos)


def test_permute_drops_out_of_range_ids(dev):
    idx = np.array([[3, 1], [-1, 3], [7, 300]], dtype=np.int64)
    off, ptok, pslot, rpos, active, n_active, bad = native.permute(torch.from_numpy(idx).to(dev), 8)
    torch.cuda.synchronize()
    assert int(bad.item()) == 2
    r = rpos.cpu().numpy()
    assert r[1, 0] == -1 and r[2, 1] == -1
    assert off.cpu().numpy().tolist() == [0, 0, 1, 1, 3, 3, 3, 3, 4]
    # expert 3: (slot 0, token 0) then (slot 1, token 1)
    assert ptok.cpu().numpy()[1:3].tolist() == [0, 1] and pslot.cpu().numpy()[1:3].tolist() == [0, 1]
    assert active[:int(n_active.item())].cpu().numpy().tolist() == [1, 3, 7]


@pytest.mark.parametrize("tokens", [1, 2, 3, 8, 16, 64])
def test_layer_matches_oracle(dev, case13, tokens):
    x = S.hidden_states(200 + tokens, tokens)
    out, idx, sc, lg = case13.run(x)
    w_out, w_idx, w_sc, w_lg = case13.oracle(x)
    z = S.bf16_bits_to_f32(w_lg) + case13.w.bias
    compare_ids(idx, w_idx, z, slack_ulps=1.0, case=f"layer T={tokens}")
    same = np.all(idx == w_idx, axis=1)
    assert same.mean() > 0.9
    assert_close(lg, w_lg, what="logits")
    assert_close(sc[same], w_sc[same], what="scores")
    assert_close(out[same], w_out[same], what="layer output")


@pytest.mark.parametrize("top_k", [4, 16])
@pytest.mark.parametrize("tokens", [1, 2, 16, 100])
def test_layer_other_top_k_matches_oracle(dev, case13, top_k, tokens):
    """top_k other than 8 through every width class: the fused decode kernel,
    which also routes (T <= 2; top_k 16 at T = 2 fills its 32-route plan), the
    grouped kernel with its own combine (16), the general
    routing with the standalone combine (100)."""
    c = case13
    layer = native.Layer(router=c.router, gate_up=c.gu_dev, down=c.dn_dev, bias=c.bias, shared_gate=c.sh[0],
                         shared_up=c.sh[1], shared_down=c.sh[2], shared_gate_w=c.sh[3], top_k=top_k)
    x_bits = S.hidden_states(400 + tokens + top_k, tokens)
    x = to_dev(x_bits, dev)
    idx = torch.empty((tokens, top_k), dtype=torch.int64, device=dev)
    lg = torch.empty((tokens, 256), dtype=torch.bfloat16, device=dev)
    out = bits(layer(x, idx_out=idx, logits_out=lg))
    w = c.w
    w_out, w_idx, _, w_lg = O.moe_layer(x_bits, w.router, w.bias, w.gate_up, w.down, w.sh_gate, w.sh_up, w.sh_down,
                                        w.sh_gate_w, top_k=top_k)
    idx = idx.cpu().numpy()
    compare_ids(idx, w_idx, S.bf16_bits_to_f32(w_lg) + w.bias, slack_ulps=1.0,
                case=f"layer T={tokens} top_k={top_k}")
    same = np.all(idx == w_idx, axis=1)
    assert same.mean() > 0.9
    assert_close(out[same], w_out[same], what=f"layer output, top_k {top_k}")


@pytest.mark.parametrize("tokens", [1, 16, 100])
def test_shared_expert_matches_oracle(dev, case13, tokens):
    """moe_shared_expert (the shared MLP and its sigmoid gate on their own)."""
    c, w = case13, case13.w
    x_bits = S.hidden_states(500 + tokens, tokens)
    out, sig = native.shared_expert(to_dev(x_bits, dev), c.sh[0], c.sh[1], c.sh[2], gate_w=c.sh[3])
    torch.cuda.synchronize()
    w_out, w_sig = O.shared_expert(x_bits, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)
    assert_close(bits(out), w_out, what="shared expert")
    assert_close(bits(sig), w_sig, what="shared gate")


@pytest.mark.parametrize("tokens,top_k", [(1, 8), (37, 8), (200, 16)])
def test_combine_matches_oracle(dev, tokens, top_k):
    """moe_combine on random route rows with the gated shared rows:
    bit-identical to the oracle's ordered BF16 combine."""
    rng = np.random.default_rng(tokens * 31 + top_k)
    idx = np.stack([rng.choice(256, top_k, replace=False) for _ in range(tokens)]).astype(np.int64)
    _, _, _, rpos = O.permute(idx, 256)
    rows = int(rpos.max()) + 1
    y = S.f32_to_bf16_bits(rng.standard_normal((rows, 2048)).astype(np.float32))
    sc = S.f32_to_bf16_bits(rng.random((tokens, top_k)).astype(np.float32))
    sh = S.f32_to_bf16_bits(rng.standard_normal((tokens, 2048)).astype(np.float32))
    sg = S.f32_to_bf16_bits(rng.random(tokens).astype(np.float32))
    got = native.combine(to_dev(y, dev), torch.from_numpy(np.ascontiguousarray(rpos, dtype=np.int32)).to(dev),
                         to_dev(sc, dev), shared_rows=to_dev(sh, dev), sig=to_dev(sg, dev))
    torch.cuda.synchronize()
    assert np.array_equal(bits(got), O.combine(y, rpos, sc, sh, sg))


@pytest.mark.parametrize("name", golden_layers())
def test_layer_matches_transformers_golden(dev, name):
    g = load_golden(name)
    case = Case(int(g["seed"]), str(g["bias_kind"]), dev)
    x = S.hidden_states(int(g["seed"]), int(g["tokens"]))
    out, idx, sc, lg = case.run(x)
    z = S.bf16_bits_to_f32(g["logits"]) + case.w.bias
    compare_ids(idx, g["idx"], z, slack_ulps=1.0, case=f"golden {name}")
    same = np.all(idx == g["idx"], axis=1)
    assert_close(out[same], g["out"][same], what="layer output vs transformers eager")


def test_host_resident_experts_match_hbm_resident(dev, case13):
    x = S.hidden_states(300, 16)
    hbm = case13.run(x)
    host = case13.run(x, layer=case13.host_layer())
    for a, b in zip(hbm, host):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("tokens", [1, 2, 16])
def test_packed_host_experts_match_hbm_resident(dev, case13, tokens):
    """Experts kept in pinned host RAM in the lossless row codec decode on their
    way into HBM: the layer output is bit-identical to the HBM-resident one."""
    x = S.hidden_states(310 + tokens, tokens)
    hbm = case13.run(x)
    packed = case13.run(x, layer=case13.packed_layer())
    for a, b in zip(hbm, packed):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("packed,slots,tokens", [(True, 128, 16), (False, 128, 16), (True, 200, 4), (True, 64, 8),
                                                  (True, 16, 2)])
def test_expert_cache_matches_hbm_resident(dev, case13, packed, slots, tokens):
    """The expert cache over host banks: over a run of calls (hits, misses and
    evictions; slots == min(E, T*top_k) evicts on nearly every call) every
    output is bit-identical to the HBM-resident layer, and the counters add up."""
    kw = dict(router=case13.router, bias=case13.bias, shared_gate=case13.sh[0], shared_up=case13.sh[1],
              shared_down=case13.sh[2], shared_gate_w=case13.sh[3], cache_slots=slots)
    if packed:
        cached = native.Layer(host_packed=native.PackedHostBanks(case13.gu, case13.dn, dev), **kw)
    else:
        hg = torch.from_numpy(case13.gu.view(np.int16)).view(torch.bfloat16).pin_memory()
        hd = torch.from_numpy(case13.dn.view(np.int16)).view(torch.bfloat16).pin_memory()
        cached = native.Layer(host_gate_up=hg, host_down=hd, **kw)
    uses = 0
    for call in range(6):
        x = S.hidden_states(400 + call % 4, tokens)  # repeats: calls 4 and 5 reuse the inputs of 0 and 1
        want = case13.run(x)
        got = case13.run(x, layer=cached)
        for a, b in zip(want, got):
            assert np.array_equal(a, b), call
        uses += len(set(got[1].reshape(-1).tolist()))
    st = cached.cache_stats()
    assert st["calls"] == 6 and st["uses"] == uses and 0 < st["misses"] <= uses
    if slots >= 128:
        assert st["misses"] < uses
    cache = cached.cache.cpu().numpy()
    slot_of, expert_of = cache[:256], cache[256:256 + slots]
    held = expert_of[expert_of >= 0]
    assert len(set(held.tolist())) == held.size                      # an expert holds at most one slot
    assert all(slot_of[e] == s for s, e in enumerate(expert_of) if e >= 0)
    assert (slot_of >= 0).sum() == held.size
    cached.release()


def test_route_in_is_the_experts_forward(dev, case13):
    """Qwen3_5MoeExperts.forward semantics: given ids and BF16 weights, no router
    and no shared expert (edge35b _Layer.forward)."""
    tokens = 12
    rng = np.random.default_rng(4)
    idx = np.stack([rng.choice(256, 8, replace=False) for _ in range(tokens)]).astype(np.int64)
    wts = S.f32_to_bf16_bits(rng.dirichlet(np.ones(8), size=tokens).astype(np.float32))
    x = S.hidden_states(301, tokens)
    out = case13.layer(to_dev(x, dev), route_in=torch.from_numpy(idx).to(dev), weights_in=to_dev(wts, dev))
    offsets, ptok, _, rpos = O.permute(idx, 256)
    y = O.experts_by_route(x, case13.w.gate_up, case13.w.down, offsets, ptok, 256)
    want = O.combine(y, rpos, wts)
    assert_close(bits(out), want, what="experts forward")


def test_empty_batch(dev, case13):
    """An empty batch (T = 0), as the eager module takes it: the whole block
    (router and shared expert), the experts forward with given routes, the
    permute (zero offsets, no active expert) and the combine return empty
    results of the right shapes without error, and the next call of the same
    layer still matches the oracle."""
    x = torch.empty((0, 2048), dtype=torch.bfloat16, device=dev)
    assert tuple(case13.layer(x).shape) == (0, 2048)
    idx = torch.empty((0, 8), dtype=torch.int64, device=dev)
    wts = torch.empty((0, 8), dtype=torch.bfloat16, device=dev)
    assert tuple(case13.layer(x, route_in=idx, weights_in=wts).shape) == (0, 2048)
    for wide in (False, True):
        offsets, _, _, rpos, _, n_active, bad = native.permute(idx, 256, wide=wide)
        torch.cuda.synchronize()
        assert offsets.cpu().numpy().tolist() == [0] * 257 and int(n_active.item()) == 0 and int(bad.item()) == 0
        assert tuple(rpos.shape) == (0, 8)
    y = torch.empty((0, 2048), dtype=torch.bfloat16, device=dev)
    assert tuple(native.combine(y, rpos, wts).shape) == (0, 2048)
    torch.cuda.synchronize()
    xb = S.hidden_states(990, 3)
    out, idx3, _, _ = case13.run(xb)
    w_out, w_idx, _, w_lg = case13.oracle(xb)
    compare_ids(idx3, w_idx, S.bf16_bits_to_f32(w_lg) + case13.w.bias, slack_ulps=1.0, case="after an empty batch")
    same = np.all(idx3 == w_idx, axis=1)
    assert_close(out[same], w_out[same], what="layer after an empty batch")


def oracle_with_routes(w, x_bits, idx, scores):
    """The oracle's expert path, combine and shared expert for given routes
    (ids and BF16 scores), for tokens whose selection the GPU decided through
    a near tie."""
    offsets, ptok, _, rpos = O.permute(np.ascontiguousarray(idx, dtype=np.int64), 256)
    y = O.experts_by_route(x_bits, w.gate_up, w.down, offsets, ptok, 256)
    sh, sig = O.shared_expert(x_bits, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)
    return O.combine(y, rpos, np.ascontiguousarray(scores), sh, sig)


@pytest.mark.parametrize("tokens", [4096, 8192])
def test_layer_prefill_full_width_matches_oracle(dev, case14, tokens):
    """configs[3] (T = 4096, Zipf(1.1) routing) and twice that, every token:
    logits, ids (tier 2, near ties counted), scores and outputs against the
    oracle; the tokens whose selection moved through a near tie are checked
    too -- their ids must be the oracle's selection on the GPU's own logits
    (tier 1), and their outputs the oracle's for the GPU's routes."""
    x = S.hidden_states(400 + tokens, tokens)
    out, idx, sc, lg = case14.run(x)
    w_out, w_idx, w_sc, w_lg = case14.oracle(x)
    assert_close(lg, w_lg, what="prefill logits")
    z = S.bf16_bits_to_f32(w_lg) + case14.w.bias
    excused = compare_ids(idx, w_idx, z, slack_ulps=1.0, case=f"prefill T={tokens}")
    assert excused <= tokens // 50, f"{excused} near-tie tokens of {tokens}"
    same = np.all(idx == w_idx, axis=1)
    assert_close(sc[same], w_sc[same], what="prefill scores")
    assert_close(out[same], w_out[same], what="prefill output")
    moved = np.flatnonzero(~same)
    if moved.size:
        own_idx, _, own_sc = O.router_select(lg[moved], case14.w.bias)
        assert np.array_equal(own_idx, idx[moved])
        assert_close(sc[moved], own_sc, what="near-tie tokens' scores")
        want = oracle_with_routes(case14.w, np.ascontiguousarray(x[moved]), idx[moved], sc[moved])
        assert_close(out[moved], want, what="near-tie tokens' outputs")


def test_graph_capture_replays_with_new_routes(dev, case13):
    tokens = 16
    x1, x2 = S.hidden_states(500, tokens), S.hidden_states(501, tokens)
    want2 = case13.run(x2)[0]
    xs = to_dev(x1, dev)
    out = torch.empty_like(xs)
    case13.layer(xs, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        case13.layer(xs, out=out)
    xs.copy_(to_dev(x2, dev))
    graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(bits(out), want2)


def test_expert_rows_against_cpu_experts(dev, case13):
    """moe_expert_rows / moe_expert_block_rows vs edge35b/cpu_experts.c (built
    from the reference) or, where that was not built, the oracle restatement."""
    rng = np.random.default_rng(8)
    experts = rng.choice(256, 8, replace=False)
    x = S.hidden_states(600, 4)
    gu = [case13.gu_dev[e] for e in experts]
    dn = [case13.dn_dev[e] for e in experts]
    got1 = bits(native.expert_block_rows(gu, dn, to_dev(x[:1], dev)))
    tok = rng.integers(0, 4, size=8).tolist()
    got4 = bits(native.expert_block_rows(gu, dn, to_dev(x, dev), token_ids=tok))
    off = np.arange(9, dtype=np.int32)
    table_g = {i: case13.gu[e] for i, e in enumerate(experts)}
    table_d = {i: case13.dn[e] for i, e in enumerate(experts)}
    want1 = O.experts_by_route(x[:1], table_g, table_d, off, np.zeros(8, np.int32), 8)
    want4 = O.experts_by_route(x, table_g, table_d, off, np.array(tok, np.int32), 8)
    if O.ref_experts_lib() is not None:
        assert np.array_equal(want4, O.ref_expert_block_rows(x, [case13.gu[e] for e in experts],
                                                             [case13.dn[e] for e in experts], tok))
    assert_close(got1, want1, what="expert_rows")
    assert_close(got4, want4, what="expert_block_rows")


def test_layer_on_two_devices_in_one_process():
    """One process drives the layer on device 0 and then on device 1: kernel
    attributes (the shared-memory opt-ins) are per device, so every width
    class must launch on the second device too, with the same bits."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    build.build()
    w = S.layer_weights(17, experts=64)
    gu, dn = w.stacked()
    got = {}
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            native.device_check(d)
            layer = native.Layer(router=to_dev(w.router, dev), gate_up=to_dev(gu, dev), down=to_dev(dn, dev),
                                 bias=torch.from_numpy(w.bias).to(dev), shared_gate=to_dev(w.sh_gate, dev),
                                 shared_up=to_dev(w.sh_up, dev), shared_down=to_dev(w.sh_down, dev),
                                 shared_gate_w=to_dev(w.sh_gate_w, dev))
            for tokens in (1, 16, 100):
                got[d, tokens] = bits(layer(to_dev(S.hidden_states(70 + tokens, tokens), dev)))
            torch.cuda.synchronize(dev)
    for tokens in (1, 16, 100):
        assert np.array_equal(got[0, tokens], got[1, tokens]), tokens


@pytest.mark.parametrize("tokens", [700, 4096])
def test_grouped_kernel_layouts_agree(dev, case14, tokens, monkeypatch):
    """At 128-token tiles the grouped kernel runs tokens-as-M (the token tile
    the M = 128 operand, the item's 256 weight rows one N = 256 operand); the
    swapped layout (LRB_GROUPED_SWAP=1) and the CTA-pair kernel
    (LRB_GROUPED_PAIRS=1, tcgen05.mma cta_group::2) compute the same products.
    At a width with many partial token tiles (700 tokens, ~22 rows per
    expert) and at configs[3] (4096) all three must agree bit for bit: every
    output element is the same FP32 K-sum rounded at the same points."""
    x = S.hidden_states(900 + tokens, tokens)
    monkeypatch.delenv("LRB_GROUPED_SWAP", raising=False)
    monkeypatch.delenv("LRB_GROUPED_PAIRS", raising=False)
    assert native.lib().moe_grouped_paired(tokens, S.INNER, S.HIDDEN) == 0
    tokm = case14.run(x)
    monkeypatch.setenv("LRB_GROUPED_SWAP", "1")
    swapped = case14.run(x)
    monkeypatch.delenv("LRB_GROUPED_SWAP")
    monkeypatch.setenv("LRB_GROUPED_PAIRS", "1")
    assert native.lib().moe_grouped_paired(tokens, S.INNER, S.HIDDEN) == 1, "pairs not selectable at this width"
    paired = case14.run(x)
    for other, name in ((swapped, "swapped"), (paired, "paired")):
        for a, b, what in zip(tokm, other, ("output", "ids", "scores", "logits")):
            assert np.array_equal(a, b), f"tokens-as-M vs {name} {what} differ at T={tokens}"


def test_host_stream_overlapped_transfers_equal_per_batch_calls(dev, case13):
    """pipeline.HostStream runs the layer over host batches with each batch's
    copies on side streams overlapped with its neighbours' compute, eagerly
    and as one captured CUDA graph; every output equals the layer's own call
    on that batch, bit for bit, and nothing is left unwritten."""
    from lightreason_b200.pipeline import HostStream

    tokens, n = 64, 5
    xs = [S.hidden_states(1300 + i, tokens) for i in range(n)]
    want = [bits(case13.layer(to_dev(x, dev))) for x in xs]
    host_in = [torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16).pin_memory()
               for x in xs]
    hs = HostStream((tokens, 2048), (tokens, 2048), device=dev)
    for captured in (False, True):
        host_out = [torch.full((tokens, 2048), float("nan"), dtype=torch.bfloat16).pin_memory() for _ in range(n)]
        if captured:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                hs.run(lambda x, o: case13.layer(x, out=o), host_in, host_out)
            for o in host_out:
                o.fill_(float("nan"))
            g.replay()
        else:
            hs.run(lambda x, o: case13.layer(x, out=o), host_in, host_out)
        torch.cuda.synchronize()
        for i in range(n):
            assert np.array_equal(host_out[i].view(torch.int16).numpy().view(np.uint16), want[i]), (captured, i)
