"""Bit-exact parity of the descriptor-driven expert gathers (GPU only).

Mirrors the reference's tests of the same kernels: sentinel-filled slots,
device-side counts of 0 and partial plans under CUDA-graph replay, mixed raw /
packed / compact sources, mapped pinned host sources and the production row
sizes (edge35b/test_gpu_resident_experts.py:12-53,
edge35b/test_freetoken_packed_transfer.py:31-87,127-192).  Expected bytes come
from the oracle's host emulation (oracle.gather_rows) and the reference's own
vectors (tests/golden/codec_vectors.npz).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from lightreason_b200 import build, native
from lightreason_b200.native_bf16_gather import CPU_TILE_GEOMETRIES, NATIVE_GEOMETRIES, NativeBf16Gather
from oracle import oracle as O
from tests.helpers import load_golden

pytestmark = pytest.mark.gpu
SENTINEL = 0x5A5A


@pytest.fixture(scope="module")
def dev():
    build.build()
    native.device_check(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def codec():
    return load_golden("codec_vectors.npz")


def i64(values, dev):
    return torch.tensor(values, dtype=torch.int64, device=dev)


def i32(values, dev):
    return torch.tensor(values, dtype=torch.int32, device=dev)


def place(array: np.ndarray, dev, where: str, keep: list) -> int:
    """Address of a copy of `array` in device memory or mapped pinned host memory."""
    t = torch.from_numpy(np.ascontiguousarray(array).view(np.uint8).copy())
    t = t.to(dev) if where == "device" else t.pin_memory()
    keep.append(t)
    return t.data_ptr()


@pytest.mark.parametrize("where", ["device", "host"])
@pytest.mark.parametrize("geometry", NATIVE_GEOMETRIES + ((3, 64, "default"), (1, 1024, "l2")))
def test_row_codec_mixed_bank_graph_replay(dev, codec, where, geometry):
    keep, outs, descs, banks = [], [], [], []
    for n in (64, 32):
        bits = codec[f"mixed{n}_bits"]
        out = torch.full((5, n), SENTINEL, dtype=torch.int16, device=dev)
        table = []
        for e in range(4):
            if e < 2:
                table.append((place(bits[e], dev, "device" if e == 0 else where, keep), -1, 0))
            else:
                b, esc = codec[f"mixed{n}_e{e}_meta"].tolist()
                table.append((place(codec[f"mixed{n}_e{e}_packed"], dev, where, keep), b, esc))
        banks.append(bits)
        outs.append(out)
        descs.append(table)
    src, dst = i32([2, 0, 3, -1], dev), i32([4, 1, 2, -1], dev)
    count = i64([0], dev)
    args = (i64(descs, dev), i64([o.data_ptr() for o in outs], dev), i64([128, 64], dev), src, dst, count)
    gather = NativeBf16Gather()
    gather.copy(*args, max_copies=4, experts=4, geometry=geometry)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gather.copy(*args, max_copies=4, experts=4, geometry=geometry)
    for copies in (0, 3, 1):
        count.fill_(copies)
        for o in outs:
            o.fill_(SENTINEL)
        graph.replay()
        torch.cuda.synchronize()
        for bits, out in zip(banks, outs):
            expected = np.full(out.shape, SENTINEL, dtype=np.uint16)
            for e, slot in zip([2, 0, 3][:copies], [4, 1, 2][:copies]):
                expected[slot] = bits[e]
            assert np.array_equal(out.cpu().numpy().view(np.uint16), expected)


def test_resident_tiles_descriptor_switch(dev, codec):
    """test_gpu_resident_experts.py:14-53 on this kernel: compact packed row
    (24 encoded + 8 inline raw tiles) and a raw row, descriptors flipped and
    count 2, 0, 1 under graph replay, untouched slots keep the sentinel."""
    original = codec["tiles7091_bits"]
    data = torch.from_numpy(codec["tiles7091_data"]).to(dev)
    meta = torch.from_numpy(codec["tiles7091_headers"]).to(dev)
    other = torch.from_numpy((original.view(np.int16) ^ 31).copy()).to(dev)
    descriptors = i64([[[data.data_ptr(), meta.data_ptr(), -1], [0, 0, other.data_ptr()]]], dev)
    output = torch.full((4, 32, 256), -123, dtype=torch.int16, device=dev)
    args = (descriptors, i64([output.data_ptr()], dev), i64([original.size * 2], dev), i32([0, 1], dev),
            i32([1, 3], dev), i64([2], dev))
    gather = NativeBf16Gather()
    gather.copy(*args, max_copies=2, experts=2, geometry=(4, 256, "resident"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gather.copy(*args, max_copies=2, experts=2, geometry=(4, 256, "resident"))
    references = [torch.from_numpy(original.view(np.int16).copy()), other.cpu()]
    for n in (2, 0, 1):
        descriptors.copy_(descriptors.flip(1))
        references.reverse()
        output.fill_(-123)
        args[5].fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        expected = torch.full_like(output.cpu(), -123)
        for slot, ref in zip((1, 3)[:n], references[:n]):
            expected[slot] = ref
        assert torch.equal(output.cpu(), expected)


def _random_bank(rng, rows, elements, raw_every=3):
    """BF16 rows whose 256-value tiles mostly fit the tile codec, some raw."""
    bits = rng.integers(0, 2 ** 16, (rows, elements), dtype=np.uint16)
    narrow = (bits & 0x80FF) | ((118 + (bits >> 8) % 6).astype(np.uint16) << 8 & 0x7F00)
    tiles = narrow.reshape(rows, -1, 256)
    tiles[:, ::raw_every] = bits.reshape(rows, -1, 256)[:, ::raw_every]
    return tiles.reshape(rows, elements)


@pytest.mark.parametrize("geometry", CPU_TILE_GEOMETRIES + ((5, 96, "cpu-tiles"), (4, 256, "resident")))
def test_tile_codec_production_rows_from_pinned_host(dev, geometry):
    rng = np.random.default_rng(841)
    sizes = (1024 * 2048, 2048 * 512)
    keep, outs, descs, banks = [], [], [], []
    compact = geometry[2] == "resident"
    for n in sizes:
        bits = _random_bank(rng, 4, n)
        banks.append(bits)
        table = []
        for e in range(4):
            if e == 1:
                table.append((0, 0, place(bits[e], dev, "host", keep)))          # raw row
            elif compact and e == 3:
                data, headers, _, _ = O.compact_encode(bits[e])
                table.append((place(data, dev, "host", keep), place(headers, dev, "device", keep), -1))
            else:
                packed, bases, _ = O.tile_pack(bits[e])
                table.append((place(packed, dev, "host", keep), place(bases, dev, "device", keep),
                              place(bits[e], dev, "host", keep)))
        descs.append(table)
        outs.append(torch.full((6, n), SENTINEL, dtype=torch.int16, device=dev))
    src, dst = [3, 0, 1, 2], [4, 1, 5, 0]
    gather = NativeBf16Gather()
    gather.copy(i64(descs, dev), i64([o.data_ptr() for o in outs], dev), i64([n * 2 for n in sizes], dev),
                i32(src, dev), i32(dst, dev), i64([4], dev), max_copies=4, experts=4, geometry=geometry)
    torch.cuda.synchronize()
    for bits, out in zip(banks, outs):
        expected = np.full(out.shape, SENTINEL, dtype=np.uint16)
        for e, slot in zip(src, dst):
            expected[slot] = bits[e]
        assert np.array_equal(out.cpu().numpy().view(np.uint16), expected)


def test_row_codec_production_rows_with_escapes(dev):
    """4 MiB / 2 MiB rows through the row codec with a few hundred escapes,
    against the oracle's decode; sources in mapped pinned memory."""
    rng = np.random.default_rng(12)
    keep, descs, outs, banks = [], [], [], []
    for n in (1024 * 2048, 2048 * 512):
        vals = (rng.standard_normal((3, n)).astype(np.float32) * 0.02)
        from lightreason_b200.synthetic import f32_to_bf16_bits
        bits = f32_to_bf16_bits(vals)
        table = []
        for e in range(3):
            base, esc = O.exponent_window(bits[e])
            packed = O.row_pack(bits[e], base, esc)
            table.append((place(packed, dev, "host", keep), base, esc))
        descs.append(table)
        banks.append(bits)
        outs.append(torch.full((3, n), SENTINEL, dtype=torch.int16, device=dev))
    gather = NativeBf16Gather()
    for geometry in ((8, 256, "default"), (16, 128, "l2"), (7, 512, "default")):
        for o in outs:
            o.fill_(SENTINEL)
        gather.copy(i64(descs, dev), i64([o.data_ptr() for o in outs], dev), i64([b.shape[1] * 2 for b in banks], dev),
                    i32([0, 1, 2], dev), i32([2, 0, 1], dev), i64([3], dev), max_copies=3, experts=3,
                    geometry=geometry)
        torch.cuda.synchronize()
        for bits, out in zip(banks, outs):
            got = out.cpu().numpy().view(np.uint16)
            assert np.array_equal(got[2], bits[0]) and np.array_equal(got[0], bits[1])
            assert np.array_equal(got[1], bits[2])
