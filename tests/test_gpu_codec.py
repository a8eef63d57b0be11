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


def _compact_on_device(rows_bits: np.ndarray, dev, shrinks=None):
    """moe_tilecodec_pack + moe_tilecodec_compact of rows [n_rows, n]; each row
    at a 256-byte-aligned offset with its headers after it.  Returns (arena
    bytes, data offsets, header offsets, written sizes)."""
    rows = to_dev(rows_bits, dev).reshape(rows_bits.shape)
    n_rows, n = rows_bits.shape
    tiles = n // 256
    packed, bases, _ = native.tilecodec_pack(rows.reshape(-1))
    cap = (512 * tiles + 4 * tiles + 512 + 255) // 256 * 256
    data_off = np.arange(n_rows, dtype=np.int64) * cap
    if shrinks is not None:
        data_off = np.where(shrinks, data_off, -1)
    header_off = np.arange(n_rows, dtype=np.int64) * cap + 512 * tiles + 256
    arena = torch.full((n_rows * cap,), 0xA5, dtype=torch.uint8, device=dev)
    sizes = native.tilecodec_compact(rows, packed, bases, arena, torch.from_numpy(data_off).to(dev),
                                     torch.from_numpy(header_off).to(dev))
    return arena.cpu().numpy(), data_off, header_off, sizes.cpu().numpy()


def test_tile_compact_rows_reference_vectors(dev):
    """Device compact-row assembly on the seed-7091 row (24 encoded + 8 raw
    tiles) gives the reference encode()'s data and headers byte for byte."""
    z = load_golden("codec_vectors.npz")
    bits = z["tiles7091_bits"].reshape(1, -1)
    arena, doff, hoff, sizes = _compact_on_device(bits, dev)
    data, headers = z["tiles7091_data"], z["tiles7091_headers"]
    assert sizes[0] == data.size
    assert np.array_equal(arena[doff[0]:doff[0] + data.size], data)
    assert np.array_equal(arena[hoff[0]:hoff[0] + headers.size], headers)
    assert np.all(arena[doff[0] + data.size:hoff[0]] == 0xA5)   # nothing written past the row


@pytest.mark.parametrize("tiles", [1, 33, 1024, 1025, 8192])
def test_tile_compact_rows_match_host_encoder(dev, tiles):
    """Rows across the kernel's 1024-tile chunk boundary, with raw tiles at
    random places and a skipped row, against the host encode()."""
    rng = np.random.default_rng(tiles + 5)
    n_rows = 3
    words = rng.integers(0, 2 ** 16, (n_rows, tiles * 256), dtype=np.uint16)
    span = np.repeat(rng.choice([4, 8, 13], size=(n_rows, tiles), p=[0.6, 0.25, 0.15]), 256, axis=1)
    exps = (100 + rng.integers(0, 2 ** 16, words.shape) % span).astype(np.uint16)
    words = (words & 0x80FF) | ((exps << 8) & 0x7F00)
    shrinks = np.array([True, False, True])
    arena, doff, hoff, sizes = _compact_on_device(words, dev, shrinks)
    assert sizes[1] == 0
    for r in (0, 2):
        packed, bases, _ = gre.pack_tiles(words[r])
        starts, headers, data_bytes = gre.compact_layout(bases)
        assert sizes[r] == data_bytes
        # the host encoder returns the row raw when it does not shrink; lay it
        # out compactly here anyway to compare every tile
        want = np.empty(data_bytes, dtype=np.uint8)
        for t in range(tiles):
            src = words[r].view(np.uint8)[t * 512:(t + 1) * 512] if bases[t] == 255 else packed[t]
            want[starts[t]:starts[t] + src.size] = src
        assert np.array_equal(arena[doff[r]:doff[r] + data_bytes], want), f"row {r} data"
        assert np.array_equal(arena[hoff[r]:hoff[r] + 4 * tiles], headers.view(np.uint8)), f"row {r} headers"
        data, hdr, _, _ = gre.encode(words[r])
        if hdr is not None:
            assert np.array_equal(data, want) and np.array_equal(hdr, headers.view(np.uint8))


def test_tile_compact_refuses_rows_outside_the_arena(dev):
    """A row whose data would run past the arena is reported (-1) and left
    unwritten; the call itself succeeds."""
    bits = load_golden("codec_vectors.npz")["tiles7091_bits"].reshape(1, -1)
    rows = to_dev(bits, dev).reshape(bits.shape)
    packed, bases, _ = native.tilecodec_pack(rows.reshape(-1))
    arena = torch.full((4096,), 0x5A, dtype=torch.uint8, device=dev)
    off = torch.zeros(1, dtype=torch.int64, device=dev)
    sizes = native.tilecodec_compact(rows, packed, bases, arena, off, off)
    torch.cuda.synchronize()
    assert int(sizes.item()) == -1
    assert bool((arena == 0x5A).all())
