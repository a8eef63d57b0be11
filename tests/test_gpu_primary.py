"""Packed primary cache (moe_stage_primary, moe_gather_compact_tail) against the
oracle codecs.

Both kernels are lossless: every row they stage must equal the expert's BF16
bits, and every slot or tail entry they refill must hold the compact tile
bytes of oracle.compact_encode (the gpu_resident_experts.encode restatement
pinned to the reference's seed-7091 vectors).  The plans cover each source a
row can take (packed-slot hit, miss from the host source, from a compact
replica, from a raw replica; raw slots; uncached rows; raw rows without
bases; rows whose every tile is raw).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from lightreason_b200 import build, native
from lightreason_b200.native_bf16_gather import NativeBf16Gather
from oracle import oracle as O

pytestmark = pytest.mark.gpu

EXPERTS = 8
ROW_BYTES = (32768, 16384)        # bank 0: 64 tiles, bank 1: 32 tiles


@pytest.fixture(scope="module")
def dev():
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    native.device_check(0)
    return torch.device("cuda", 0)


def expert_rows(bank: int) -> np.ndarray:
    """[E, values] uint16: N(0, 0.02) BF16 rows with some wide tiles; expert 7
    has only raw tiles."""
    rng = np.random.default_rng(70 + bank)
    values = ROW_BYTES[bank] // 2
    rows = (rng.standard_normal((EXPERTS, values)).astype(np.float32) * 0.02)
    bits = (rows.view(np.uint32) >> 16).astype(np.uint16)
    for e in range(EXPERTS):
        for t in rng.choice(values // 256, 3, replace=False):   # three raw tiles per row
            bits[e, t * 256 + 7] = 0x7F00 | (e & 0x7F)
            bits[e, t * 256 + 9] = 0x0001
    bits[7] = rng.integers(0, 1 << 16, size=values, dtype=np.uint16)
    return bits


class Banks:
    def __init__(self, dev):
        self.dev = dev
        self.rows = [expert_rows(b) for b in range(2)]
        self.keep = []
        self.packed_host, self.bases_host, self.raw_host = [], [], []
        self.compact = []     # per bank, per expert: (data bytes, headers bytes or None)
        self.bases = []
        for b in range(2):
            packed, bases = [], []
            for e in range(EXPERTS):
                p, s, _ = O.tile_pack(self.rows[b][e])
                packed.append(p)
                bases.append(s)
            self.bases.append(np.stack(bases))
            self.packed_host.append([self.pin(p) for p in packed])
            self.bases_host.append([self.pin(s) for s in bases])
            self.raw_host.append([self.pin(self.rows[b][e].view(np.uint8)) for e in range(EXPERTS)])
            self.compact.append([O.compact_encode(self.rows[b][e])[:2] for e in range(EXPERTS)])
        self.prefix = [native.prefix_table(self.bases[b]).to(dev) for b in range(2)]
        self.prefix_ptrs = torch.tensor([p.data_ptr() for p in self.prefix], dtype=torch.int64, device=dev)

    def pin(self, a: np.ndarray) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).copy()).pin_memory()
        self.keep.append(t)
        return t

    def dev_bytes(self, a: np.ndarray) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).copy()).to(self.dev)
        self.keep.append(t)
        return t

    def source_table(self, *, raw_only=(), compact=()):
        """Tile-codec host descriptors; experts in raw_only have no bases, experts
        in compact point at a device compact replica (raw == -1)."""
        table = np.zeros((2, EXPERTS, 3), dtype=np.int64)
        for b in range(2):
            for e in range(EXPERTS):
                if e in compact:
                    data, headers = self.compact[b][e]
                    table[b, e] = (self.dev_bytes(data).data_ptr(), self.dev_bytes(headers).data_ptr(), -1)
                elif e in raw_only:
                    table[b, e] = (0, 0, self.raw_host[b][e].data_ptr())
                else:
                    table[b, e] = (self.packed_host[b][e].data_ptr(), self.bases_host[b][e].data_ptr(),
                                   self.raw_host[b][e].data_ptr())
        return table

    def slot_stride(self) -> list[int]:
        return [max((d.size + 127) // 128 * 128 for d, _ in self.compact[b]) for b in range(2)]


def as_rows(buf: torch.Tensor, b: int) -> np.ndarray:
    return buf.cpu().numpy().reshape(-1, ROW_BYTES[b]).view(np.uint16)


@pytest.fixture(scope="module")
def banks(dev):
    return Banks(dev)


def test_stage_primary_miss_then_hit(dev, banks):
    gather = NativeBf16Gather()
    packed_slots, raw_slots, max_rows = 5, 2, 12
    sources = banks.source_table(raw_only=(6,))
    miss = sources.copy()
    for b in range(2):
        data, headers = banks.compact[b][2]
        miss[b, 2] = (banks.dev_bytes(data).data_ptr(), banks.dev_bytes(headers).data_ptr(), -1)   # compact replica
        miss[b, 3] = (0, 0, banks.dev_bytes(banks.rows[b][3].view(np.uint8)).data_ptr())           # raw replica
    stride = banks.slot_stride()
    packed = [torch.zeros(packed_slots * stride[b], dtype=torch.uint8, device=dev) for b in range(2)]
    raw_slot = [torch.zeros(raw_slots * ROW_BYTES[b], dtype=torch.uint8, device=dev) for b in range(2)]
    work = [torch.zeros((max_rows + 1) * ROW_BYTES[b], dtype=torch.uint8, device=dev) for b in range(2)]
    layouts = torch.tensor([(packed[b].data_ptr(), raw_slot[b].data_ptr(), work[b].data_ptr(), stride[b], ROW_BYTES[b])
                            for b in range(2)], dtype=torch.int64, device=dev)
    # (expert, slot, miss): the row kinds listed in the module docstring
    rows = [(0, 0, 1), (1, 1, 1), (2, 2, 1), (3, 3, 1), (4, packed_slots, 1), (5, -1, 1), (6, -1, 1), (7, 4, 1),
            (2, packed_slots + 1, 1)]
    plan = torch.full((3, max_rows), 0, dtype=torch.int32)
    plan[:, :len(rows)] = torch.tensor(rows, dtype=torch.int32).t()
    count = torch.tensor([len(rows)], dtype=torch.int32, device=dev)
    src_t, miss_t = torch.from_numpy(sources).to(dev), torch.from_numpy(miss).to(dev)
    gather.stage_primary(src_t, miss_t, layouts, banks.prefix_ptrs, plan.to(dev), count, experts=EXPERTS,
                         packed_slots=packed_slots)
    torch.cuda.synchronize()
    for b in range(2):
        w = as_rows(work[b], b)
        rs = as_rows(raw_slot[b], b)
        for r, (e, slot, _) in enumerate(rows):
            got = rs[slot - packed_slots] if slot >= packed_slots else w[r + 1]
            assert np.array_equal(got, banks.rows[b][e]), (b, r)
            if 0 <= slot < packed_slots:
                data = banks.compact[b][e][0]
                if banks.compact[b][e][1] is None:          # kept raw by the encoder: every tile raw
                    data = banks.rows[b][e].view(np.uint8)
                cached = packed[b].cpu().numpy()[slot * stride[b]: slot * stride[b] + data.size]
                assert np.array_equal(cached, data), (b, r, "slot refill")
    # hits: the packed slots decode back to the rows; a raw-slot hit is skipped
    for w in work:
        w.fill_(0xAB)
    hits = [(0, 0, 0), (1, 1, 0), (2, 2, 0), (3, 3, 0), (7, 4, 0), (4, packed_slots, 0)]
    plan = torch.zeros((3, max_rows), dtype=torch.int32)
    plan[:, :len(hits)] = torch.tensor(hits, dtype=torch.int32).t()
    count.fill_(len(hits))
    gather.stage_primary(src_t, miss_t, layouts, banks.prefix_ptrs, plan.to(dev), count, experts=EXPERTS,
                         packed_slots=packed_slots)
    torch.cuda.synchronize()
    for b in range(2):
        w = as_rows(work[b], b)
        for r, (e, slot, _) in enumerate(hits):
            if slot >= packed_slots:
                assert (w[r + 1] == 0xABAB).all(), "a raw-slot hit writes nothing"
            else:
                assert np.array_equal(w[r + 1], banks.rows[b][e]), (b, r, "hit")


def test_compact_tail_fill_then_resident(dev, banks):
    gather = NativeBf16Gather()
    max_rows = 8
    sources = torch.from_numpy(banks.source_table(raw_only=(6,), compact=(5,))).to(dev)
    resident = torch.from_numpy(banks.source_table()).to(dev)
    stride = banks.slot_stride()
    storage = [torch.zeros(4 * stride[b], dtype=torch.uint8, device=dev) for b in range(2)]
    tail = torch.tensor([(storage[b].data_ptr(), stride[b]) for b in range(2)], dtype=torch.int64, device=dev)
    dest = [torch.zeros(max_rows * ROW_BYTES[b], dtype=torch.uint8, device=dev) for b in range(2)]
    destinations = torch.tensor([d.data_ptr() for d in dest], dtype=torch.int64, device=dev)
    sizes = torch.tensor(ROW_BYTES, dtype=torch.int64, device=dev)
    # (expert, dest row, tail entry, resident)
    rows = [(0, 3, 0, 0), (1, 0, -1, 0), (6, 1, -1, 0), (5, 2, -1, 0), (7, 4, 1, 0)]

    def run(rows):
        src = torch.zeros(max_rows, dtype=torch.int32)
        dst = torch.zeros(max_rows, dtype=torch.int32)
        entries = torch.zeros((2, max_rows), dtype=torch.int32)
        for r, (e, d, entry, res) in enumerate(rows):
            src[r], dst[r], entries[0, r], entries[1, r] = e, d, entry, res
        gather.copy_compact_tail(sources, destinations, sizes, banks.prefix_ptrs, tail, src.to(dev), dst.to(dev),
                                 torch.tensor([len(rows)], dtype=torch.int64, device=dev), entries.to(dev), resident,
                                 EXPERTS)
        torch.cuda.synchronize()

    run(rows)
    for b in range(2):
        out = as_rows(dest[b], b)
        for e, d, entry, _ in rows:
            assert np.array_equal(out[d], banks.rows[b][e]), (b, e)
            if entry >= 0:
                data = banks.compact[b][e][0] if banks.compact[b][e][1] is not None else banks.rows[b][e].view(np.uint8)
                got = storage[b].cpu().numpy()[entry * stride[b]: entry * stride[b] + data.size]
                assert np.array_equal(got, data), (b, e, "tail entry")
    for d in dest:
        d.zero_()
    run([(0, 5, 0, 1), (7, 6, 1, 1)])              # resident rows decode from their entries
    for b in range(2):
        out = as_rows(dest[b], b)
        assert np.array_equal(out[5], banks.rows[b][0]) and np.array_equal(out[6], banks.rows[b][7])
