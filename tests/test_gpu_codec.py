"""Device encoders of the two lossless codecs against the reference's bytes.

* Row codec (moe_rowcodec_plan / moe_rowcodec_pack): the reference's own
  vectors (tests/golden/codec_vectors.npz, made by edge35b/bf16_expert_codec.py
  from its tests test_freetoken_packed_transfer.py:15-26 and :127-149), then
  whole banks against the host encoder bf16_expert_codec.pack_bank and the C
  oracle's or_row_pack: several chunks per row, lengths that are multiples of
  8 but not of 32, ties between windows, the 1% raw rule at its edge, and
  exponents 0 and 255.
* Tile codec (moe_tilecodec_pack): the reference's pack_cpu_read_tiles output
  on the seed-7091 words of test_gpu_resident_experts.py:13-23, then large
  random tile arrays against the host encoder gpu_resident_experts.pack_tiles.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from lightreason_b200 import bf16_expert_codec as codec
from lightreason_b200 import build, native
from lightreason_b200 import gpu_resident_experts as gre
from oracle import oracle as O
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    native.device_check(0)
    return torch.device("cuda", 0)


def to_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).to(dev)


def device_pack(bits: np.ndarray, dev):
    packed, plan = native.rowcodec_pack(to_dev(bits, dev))
    return packed.cpu().numpy(), plan


def test_row_codec_reference_vectors(dev):
    z = load_golden("codec_vectors.npz")
    values = np.arange(65536, dtype=np.uint16)
    common = np.full(values.shape, 0x3F80, dtype=np.uint16)
    # plan_bank of [common, every bit pattern, common]
    packed, plan = device_pack(np.stack([common, values, common]), dev)
    want = [None if none else tuple(int(v) for v in row) for none, row in zip(z["plan_none"], z["plan_rows"])]
    assert plan == want
    assert packed.size == int(z["plan_size"])
    # every bit pattern packed although the 1% rule keeps it raw: 61440 escapes
    meta = torch.tensor([[0, int(z["all_base"]), int(z["all_escapes"])]], dtype=torch.int64, device=dev)
    packed, plan = native.rowcodec_pack(to_dev(values[None], dev), meta=meta)
    assert plan == [(0, int(z["all_base"]), int(z["all_escapes"]))]
    assert hashlib.sha256(packed.cpu().numpy()[:codec.row_bytes(65536, int(z["all_escapes"]))]).hexdigest() == \
        str(z["all_packed_sha256"])
    # mixed raw/packed banks of 64- and 32-value rows: the planner agrees with
    # plan_bank (3 escapes in 64 values exceed 1%), and rows 2 and 3 packed as
    # the reference packs them (pack_verified_row, which has no 1% rule)
    for n in (64, 32):
        bits = z[f"mixed{n}_bits"]
        _, plan = device_pack(bits, dev)
        assert plan == codec.plan_bank(bits)[0]
        metas = [z[f"mixed{n}_e{e}_meta"].tolist() for e in (2, 3)]
        second = (codec.row_bytes(n, metas[0][1]) + 15) & ~15
        meta = torch.tensor([[-1, 0, 0], [-1, 0, 0], [0, *metas[0]], [second, *metas[1]]], dtype=torch.int64,
                            device=dev)
        packed, _ = native.rowcodec_pack(to_dev(bits, dev), meta=meta)
        packed = packed.cpu().numpy()
        for e, off in ((2, 0), (3, second)):
            want = z[f"mixed{n}_e{e}_packed"]
            assert np.array_equal(packed[off:off + want.size], want), (n, e)


def crafted_bank(rng: np.random.Generator, n: int) -> np.ndarray:
    """Rows that reach every branch of the planner and the packer."""
    rows = []
    # weight-like values: exponents around 120, a few escapes spread through the row
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    rows.append((w.view(np.uint32) >> 16).astype(np.uint16))
    w = rows[-1].copy()
    hit = rng.choice(n, size=n // 200, replace=False)
    w[hit] = rng.integers(0, 2 ** 16, hit.size, dtype=np.uint16)
    rows.append(w)
    # two equally full windows: the first wins
    w = np.where(np.arange(n) % 2 == 0, 0x3F80, 0x3F80 + (40 << 7)).astype(np.uint16)
    rows.append(w)
    # exponents 0 and 255 (zeros, subnormals, inf, NaN) inside and outside the window
    w = rows[0].copy()
    w[:8] = [0x0000, 0x8000, 0x0001, 0x7F80, 0xFF80, 0x7FC0, 0xFFFF, 0x007F]
    rows.append(w)
    # the 1% rule at its edge: escapes == n/100 packs, one more stays raw
    limit = n // 100
    for extra in (0, 1):
        w = np.full(n, 0x3F80, dtype=np.uint16)
        pos = np.linspace(0, n - 1, limit + extra).astype(np.int64)
        w[pos] = 0x0001
        rows.append(w)
    # a row whose window sits at the top of the exponent range
    rows.append((0x7F00 | rng.integers(0, 2 ** 7, n)).astype(np.uint16) ^ np.uint16(0x8000) * (np.arange(n) % 3 == 0))
    return np.stack(rows)


@pytest.mark.parametrize("n", [8 * 1001, 8192 * 3 + 64, 100_000])
def test_row_codec_matches_host_encoder(dev, n):
    bank = crafted_bank(np.random.default_rng(n), n)
    packed, plan = device_pack(bank, dev)
    want_packed, want_plan = codec.pack_bank(bank)
    assert plan == want_plan
    assert np.array_equal(packed, want_packed)
    for row, p in zip(bank, plan):
        if p is not None:
            off, base, escapes = p
            assert (base, escapes) == O.exponent_window(row)
            size = codec.row_bytes(n, escapes)
            assert np.array_equal(packed[off:off + size], O.row_pack(row, base, escapes))


def test_row_codec_expert_bank(dev):
    """16 experts of the 35B gate_up bank shape (1024 x 2048 values each)."""
    from lightreason_b200 import synthetic as S

    w = S.layer_weights(23, bias="zipf")
    gu, _ = w.stacked()
    bank = np.ascontiguousarray(gu[:16])
    packed, plan = device_pack(bank, dev)
    want_packed, want_plan = codec.pack_bank(bank)
    assert plan == want_plan
    assert np.array_equal(packed, want_packed)


def test_tile_codec_reference_vectors(dev):
    z = load_golden("codec_vectors.npz")
    packed, bases, encoded = native.tilecodec_pack(to_dev(z["tiles7091_bits"], dev))
    assert encoded == int(z["tiles7091_encoded"]) == 24
    assert np.array_equal(bases.cpu().numpy(), z["tiles7091_bases"])
    assert np.array_equal(packed.cpu().numpy().reshape(-1), z["tiles7091_packed"])


@pytest.mark.parametrize("tiles", [1, 7, 4097, 100_003])
def test_tile_codec_matches_host_encoder(dev, tiles):
    rng = np.random.default_rng(tiles)
    words = rng.integers(0, 2 ** 16, (tiles, 256), dtype=np.uint16)
    # most tiles in an 8-exponent span (encodable), others wide; signs random
    span = rng.integers(1, 12, tiles)[:, None]
    exps = (110 + rng.integers(0, 2 ** 16, (tiles, 256)) % span).astype(np.uint16)
    words = (words & 0x80FF) | (exps << 8) & 0x7F00
    packed, bases, encoded = native.tilecodec_pack(to_dev(words, dev))
    want_packed, want_bases, want_encoded = gre.pack_tiles(words)
    assert encoded == want_encoded
    assert np.array_equal(bases.cpu().numpy(), want_bases)
    assert np.array_equal(packed.cpu().numpy(), want_packed)
    if tiles <= 4097:
        o_packed, o_bases, o_encoded = O.tile_pack(words)
        assert o_encoded == encoded and np.array_equal(o_packed, packed.cpu().numpy().reshape(-1))


def test_packed_host_banks_encoders_agree(dev):
    """PackedHostBanks from the device encoder and from the host encoder hold
    the same bytes and the same descriptor bases and escape counts."""
    from lightreason_b200 import synthetic as S

    w = S.layer_weights(29, bias="zipf")
    gu, dn = w.stacked()
    gu, dn = np.ascontiguousarray(gu[:8]), np.ascontiguousarray(dn[:8])
    a = native.PackedHostBanks(gu, dn, dev, encoder="device")
    b = native.PackedHostBanks(gu, dn, dev, encoder="host")
    for x, y in zip(a.buffers, b.buffers):
        assert torch.equal(x, y)
    da, db = a.descriptors.cpu(), b.descriptors.cpu()
    assert torch.equal(da[..., 1:], db[..., 1:])
