"""Pin the CPU oracle before trusting it (CPU only).

* expert rows: bit-identical to edge35b/cpu_experts.c built from the
  reference sources (oracle/_ref, present where the reference tree was mounted
  at build time);
* whole layer: against the transformers eager Qwen3_5MoeSparseMoeBlock golden
  fixtures (tests/golden/make_golden.py);
* codecs: against the reference's own test vectors (codec_vectors.npz).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from lightreason_b200 import synthetic as S
from oracle import oracle as O
from tests.helpers import assert_close, compare_ids, golden_layers, load_golden


def _digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


needs_ref = pytest.mark.skipif(O.ref_experts_lib() is None,
                               reason="oracle/_ref not built (needs the reference tree at build time)")


@needs_ref
@pytest.mark.parametrize("tokens,pairs", [(1, 8), (16, 24)])
def test_expert_rows_bit_identical_to_cpu_experts_c(tokens, pairs):
    w = S.layer_weights(3)
    rng = np.random.default_rng(5)
    experts = rng.choice(256, size=min(pairs, 12), replace=False)
    w.ensure(experts)
    x = S.hidden_states(3, tokens)
    pair_expert = np.sort(rng.choice(experts, size=pairs))
    token_ids = rng.integers(0, tokens, size=pairs).astype(np.int32)
    want = O.ref_expert_block_rows(x, [w.gate_up[e] for e in pair_expert], [w.down[e] for e in pair_expert],
                                   token_ids)
    # The oracle computes per route position; lay the pairs out as one expert
    # group each (offsets over a virtual expert axis of `pairs` entries).
    offsets = np.arange(pairs + 1, dtype=np.int32)
    gu = {i: w.gate_up[e] for i, e in enumerate(pair_expert)}
    dn = {i: w.down[e] for i, e in enumerate(pair_expert)}
    got = O.experts_by_route(x, gu, dn, offsets, token_ids, pairs)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("name", golden_layers())
def test_layer_matches_transformers_eager(name):
    g = load_golden(name)
    tokens, seed, bias_kind = int(g["tokens"]), int(g["seed"]), str(g["bias_kind"])
    x = S.hidden_states(seed, tokens)
    assert _digest(x) == str(g["x_sha256"]), "synthetic activations drifted from the fixture"
    w = S.layer_weights(seed, bias=bias_kind)
    routed = sorted(set(g["idx"].reshape(-1).tolist()))
    w.ensure(routed)
    assert _digest(*[a for e in routed for a in (w.gate_up[e], w.down[e])]) == str(g["routed_sha256"])
    out, idx, scores, logits = O.moe_layer(x, w.router, w.bias, w.gate_up, w.down, w.sh_gate, w.sh_up, w.sh_down,
                                           w.sh_gate_w)
    z_ref = S.bf16_bits_to_f32(g["logits"]) + w.bias
    # FP32 summation order differs from torch's CPU GEMM: logits may move by
    # one BF16 ulp, so ids get the tier-2 slack of one ulp.
    compare_ids(idx, g["idx"], z_ref, slack_ulps=1.0)
    same = np.all(idx == g["idx"], axis=1)
    assert_close(logits, g["logits"], max_abs=2e-2, rel_l2=1e-2, what="logits")
    assert_close(scores[same], g["scores"][same], what="scores")
    assert_close(out[same], g["out"][same], what="layer output")


@pytest.fixture(scope="module")
def codec():
    return load_golden("codec_vectors.npz")


def test_row_codec_every_bf16_pattern(codec):
    values = np.arange(65536, dtype=np.uint16)
    base, escapes = O.exponent_window(values)
    assert (base, escapes) == (int(codec["all_base"]), int(codec["all_escapes"]))
    packed = O.row_pack(values, base, escapes)
    assert _digest(packed) == str(codec["all_packed_sha256"])
    assert np.array_equal(O.row_restore(packed, values.size, base, escapes), values)


def test_row_codec_mixed_bank_vectors(codec):
    for n in (64, 32):
        bits = codec[f"mixed{n}_bits"]
        for e in (2, 3):
            base, escapes = O.exponent_window(bits[e])
            assert [base, escapes] == codec[f"mixed{n}_e{e}_meta"].tolist()
            packed = O.row_pack(bits[e], base, escapes)
            assert np.array_equal(packed, codec[f"mixed{n}_e{e}_packed"])
            assert np.array_equal(O.row_restore(packed, n, base, escapes), bits[e])


def test_tile_codec_vectors(codec):
    raw = codec["tiles7091_bits"]
    packed, bases, encoded = O.tile_pack(raw)
    assert encoded == int(codec["tiles7091_encoded"]) == 24
    assert np.array_equal(bases, codec["tiles7091_bases"])
    enc = bases != 255
    ref = codec["tiles7091_packed"].reshape(32, 384)
    assert np.array_equal(packed.reshape(32, 384)[enc], ref[enc])
    data, headers, n_enc, n_raw = O.compact_encode(raw)
    assert (n_enc, n_raw) == tuple(codec["tiles7091_counts"].tolist()) == (24, 8)
    assert np.array_equal(data, codec["tiles7091_data"])
    assert np.array_equal(headers, codec["tiles7091_headers"])


def test_gather_emulation_restores_mixed_bank(codec):
    """Host emulation of the descriptor copies on the seed-76 bank: raw rows,
    packed rows with escapes, sentinel-filled untouched slots, count 0 and 3."""
    for copies in (0, 3):
        keep, dests, descs, banks = [], [], [], []
        for n in (64, 32):
            bits = np.ascontiguousarray(codec[f"mixed{n}_bits"])
            out = np.full((5, n), 0x5A5A, dtype=np.uint16)
            table = []
            for e in range(4):
                if e < 2:
                    row = np.ascontiguousarray(bits[e])
                    keep.append(row)
                    table.append((row.ctypes.data, -1, 0))
                else:
                    p = np.ascontiguousarray(codec[f"mixed{n}_e{e}_packed"])
                    keep.append(p)
                    b, esc = codec[f"mixed{n}_e{e}_meta"].tolist()
                    table.append((p.ctypes.data, b, esc))
            banks.append(bits)
            dests.append(out)
            descs.append(table)
        src = np.array([2, 0, 3, -1], dtype=np.int32)
        dst = np.array([4, 1, 2, -1], dtype=np.int32)
        O.gather_rows(np.array(descs, dtype=np.int64), np.array([d.ctypes.data for d in dests], dtype=np.int64),
                      np.array([64 * 2, 32 * 2], dtype=np.int64), src, dst, copies, 4, 0)
        for bits, out in zip(banks, dests):
            expected = np.full(out.shape, 0x5A5A, dtype=np.uint16)
            for e, slot in zip(src[:copies], dst[:copies]):
                expected[slot] = bits[e]
            assert np.array_equal(out, expected)


def test_permute_order_is_eager_dispatch_order():
    rng = np.random.default_rng(9)
    tokens, k, experts = 37, 8, 64
    idx = np.stack([rng.choice(experts, size=k, replace=False) for _ in range(tokens)]).astype(np.int64)
    offsets, ptok, pslot, rpos = O.permute(idx, experts)
    # eager: for each expert ascending, torch.where(one_hot mask[e]) over (slot, token)
    order = [(s, t) for e in range(experts) for s in range(k) for t in range(tokens) if idx[t, s] == e]
    assert [(int(s), int(t)) for s, t in zip(pslot, ptok)] == order
    assert np.array_equal(np.diff(offsets), np.bincount(idx.reshape(-1), minlength=experts))
    for t in range(tokens):
        for s in range(k):
            assert ptok[rpos[t, s]] == t and pslot[rpos[t, s]] == s
