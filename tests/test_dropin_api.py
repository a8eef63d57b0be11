"""Host-side checks of the drop-in API mirror (no GPU): the tile encoder of
gpu_resident_experts against the reference's vectors, mode names, and the
reference's argument and shape errors for the patch and per-path entries."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from lightreason_b200 import block_experts, cpu_route, expert_stream, fused_experts, moe_block
from lightreason_b200 import gpu_resident_experts as gre
from tests.helpers import load_golden


def test_resident_tile_encoder_matches_reference_vectors():
    """gpu_resident_experts.encode / pack_tiles (edge35b/gpu_resident_experts.py:22-42,
    cpu_bf16_reads.h:16-52) against the vectors its tests pinned."""
    z = load_golden("codec_vectors.npz")
    packed, bases, encoded = gre.pack_tiles(z["tiles7091_bits"])
    assert np.array_equal(packed.reshape(-1), z["tiles7091_packed"])
    assert np.array_equal(bases, z["tiles7091_bases"])
    assert encoded == int(z["tiles7091_encoded"])
    data, headers, enc, raw = gre.encode(z["tiles7091_bits"])
    assert np.array_equal(data, z["tiles7091_data"]) and np.array_equal(headers, z["tiles7091_headers"])
    assert (enc, raw) == tuple(z["tiles7091_counts"])


def test_resident_encoder_keeps_rows_that_do_not_pack_raw():
    rng = np.random.default_rng(3)
    wide = rng.integers(0, 1 << 16, size=4 * 256, dtype=np.uint16)   # every tile spans > 7 exponents
    data, headers, enc, raw = gre.encode(wide)
    assert headers is None and enc == 0 and raw == 4 and np.array_equal(data.view(np.uint16), wide)


def test_modes_cover_the_reference_modes():
    assert set(expert_stream.REFERENCE_MODES) <= set(expert_stream.MODES)
    assert set(expert_stream.RESIDENCY) == set(expert_stream.MODES)
    assert set(expert_stream.RESIDENCY.values()) == set(expert_stream.B200_MODES)


def test_pool_argument_errors():
    with pytest.raises(ValueError, match="capacity_bytes"):
        expert_stream.ExpertPool("cuda:0", capacity_bytes=-1)
    with pytest.raises(ValueError, match="non_blocking"):
        expert_stream.ExpertPool("cuda:0", non_blocking=1)
    with pytest.raises(ValueError, match="CUDA destination"):
        expert_stream.ExpertPool("cpu")


@pytest.fixture(scope="module")
def model():
    from tests.dropin_model import make_model

    return make_model(experts=8, layers=1)[0]


def test_patch_rejects_unknown_mode_and_modelless(model):
    pool = expert_stream.ExpertPool("cuda:0")
    with pytest.raises(ValueError, match="transfer mode"):
        with expert_stream.patch_experts(model, mode="bogus", pool=pool):
            pass
    with pytest.raises(ValueError, match="Qwen3_5MoeExperts"):
        with expert_stream.patch_experts(torch.nn.Linear(2, 2), mode="b200", pool=pool):
            pass
    with pytest.raises(ValueError, match="Qwen3_5MoeSparseMoeBlock"):
        with moe_block.patch_moe_blocks(torch.nn.Linear(2, 2), mode="b200", pool=pool):
            pass


def test_layer_rejects_hooked_or_unfrozen_experts(model):
    pool = expert_stream.ExpertPool("cuda:0")
    experts = model.layers[0].experts
    experts.forward = experts.forward
    try:
        with pytest.raises(ValueError, match="offload hooks"):
            expert_stream._Layer("e", experts, pool, "b200")
    finally:
        del experts.forward
    experts.gate_up_proj.requires_grad_(True)
    try:
        with pytest.raises(ValueError, match="frozen contiguous BF16"):
            expert_stream._Layer("e", experts, pool, "b200")
    finally:
        experts.gate_up_proj.requires_grad_(False)


def test_per_path_shape_errors(model):
    pool = expert_stream.ExpertPool("cuda:0")
    layer = expert_stream._Layer("e", model.layers[0].experts, pool, "fused")
    h1 = torch.zeros((1, 2048), dtype=torch.bfloat16)
    i1 = torch.zeros((1, 8), dtype=torch.long)
    w1 = torch.zeros((1, 8), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="single-token 35B route shape"):
        fused_experts.fused_forward(layer, h1[:, :1024], i1, w1)
    with pytest.raises(ValueError, match="single-token 35B route shape"):
        fused_experts.fused_forward(layer, h1, i1, w1.float())
    with pytest.raises(ValueError, match="eight distinct valid routes"):
        fused_experts.fused_forward(layer, h1, i1, w1)                 # eight copies of expert 0
    with pytest.raises(ValueError, match="eight distinct valid routes"):
        fused_experts.fused_forward(layer, h1, torch.arange(1, 9).reshape(1, 8), w1)   # 8 is out of range
    with pytest.raises(ValueError, match="AVX2 kernel"):
        cpu_route.cpu_forward(layer, torch.zeros((2, 2048), dtype=torch.bfloat16), i1, w1)
    with pytest.raises(ValueError, match="2–16"):
        block_experts.grouped_block(layer, h1, i1, w1)
    with pytest.raises(ValueError, match="contiguous"):
        h2 = torch.zeros((2048, 2), dtype=torch.bfloat16).t()
        block_experts.grouped_block(layer, h2, torch.zeros((2, 8), dtype=torch.long), w1.expand(2, 8))


def test_prefix_table_counts_raw_tiles():
    """native.prefix_table: per 32 tiles, (raw tiles before << 32) | raw bitmask,
    the table stage_bf16_primary / gather_bf16_compact_tail index
    (edge35b/packed_primary_cache.py:80-86 builds the same words)."""
    from lightreason_b200 import native

    bases = np.full((2, 96), 7, dtype=np.uint8)
    bases[0, [0, 31, 32, 95]] = 255
    bases[1, 40:72] = 255
    got = native.prefix_table(bases).numpy().view(np.uint64)
    assert got.shape == (2, 3)
    assert got[0, 0] == (0 << 32) | (1 | (1 << 31))
    assert got[0, 1] == (2 << 32) | 1
    assert got[0, 2] == (3 << 32) | (1 << 31)
    assert got[1, 0] == 0
    assert got[1, 1] == (0 << 32) | (0xFFFFFFFF & ~0xFF)
    assert got[1, 2] == (24 << 32) | 0xFF
