"""Compact GPU replicas of expert rows in the 256-value tile codec.

Drop-in for the reference's edge35b/gpu_resident_experts.py encode /
device_rows (:22-59) and its resident arena (:62-209).  The reference builds
the arena from FreeToken cache objects; FreeToken is not part of this
project, so ResidentArena takes plain expert banks instead and keeps the same
two interchangeable layouts ("raw" and "packed"), the same descriptor
convention for NativeBf16Gather (`(packed, headers, -1)` for a compact row,
`(0, 0, raw)` for a raw one) and the same bit audit.

Tile codec (cpu_bf16_reads.h:16-52): a tile of 256 BF16 values keeps each low
byte and replaces each high byte by a 4-bit code -- 3-bit offset from the
tile's smallest 7-bit high-byte exponent, bit 3 the sign -- so a tile packs
into 384 bytes when its exponents span at most 7; other tiles stay raw (512
bytes, base 255).  A compact row stores the tiles back to back with raw
fallbacks inline and one uint32 header per tile: (raw tiles before it << 8) |
base.
"""

from __future__ import annotations

import numpy as np
import torch

TILE_VALUES = 256
RAW_TILE_BYTES = 2 * TILE_VALUES
PACKED_TILE_BYTES = 3 * TILE_VALUES // 2
RAW_TILE = 255
GEOMETRY = (4, 256, "resident")


def pack_tiles(raw_bits: np.ndarray):
    """Tile-encode a flat BF16 array (length a multiple of 256).  Returns
    (packed [tiles, 384] uint8, bases [tiles] uint8 with 255 = raw, encoded)."""
    w = np.ascontiguousarray(raw_bits).view(np.uint16).reshape(-1, TILE_VALUES)
    high = (w >> 8).astype(np.uint8)
    exp = high & 0x7F
    low_e, high_e = exp.min(axis=1), exp.max(axis=1)
    ok = (high_e.astype(np.int16) - low_e.astype(np.int16)) <= 7
    bases = np.where(ok, low_e, RAW_TILE).astype(np.uint8)
    code = ((exp - low_e[:, None]) & 7) | ((high >> 4) & 8)
    packed = np.zeros((w.shape[0], PACKED_TILE_BYTES), dtype=np.uint8)
    packed[:, :TILE_VALUES] = (w & 0xFF).astype(np.uint8)
    packed[:, TILE_VALUES:] = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    packed[~ok] = 0
    # the reference encoder audits every tile it packs
    dec_high = ((bases[:, None].astype(np.uint16) + (code & 7)) | ((code & 8).astype(np.uint16) << 4)) & 0xFF
    if not np.array_equal((packed[:, :TILE_VALUES] | (dec_high << 8))[ok], w[ok]):
        raise RuntimeError("Packed expert tile failed its BF16 bit audit")
    return packed, bases, int(ok.sum())


def encode(source):
    """Compact row of a BF16 tensor or uint16 array: (data, headers|None,
    encoded tiles, raw tiles).  Keeps the raw bytes when packing does not save
    space (edge35b/gpu_resident_experts.py:22-42 semantics)."""
    if isinstance(source, torch.Tensor):
        source = source.detach().cpu().contiguous().view(torch.int16).numpy()
    raw = np.ascontiguousarray(source).view(np.uint8).reshape(-1, RAW_TILE_BYTES)
    packed, bases, encoded = pack_tiles(raw.view(np.uint16))
    compressed = bases != RAW_TILE
    raw_before = np.cumsum(~compressed, dtype=np.uint32) - (~compressed)
    headers = (raw_before << 8) | bases
    lengths = np.where(compressed, PACKED_TILE_BYTES, RAW_TILE_BYTES)
    if int(lengths.sum()) + headers.nbytes >= raw.nbytes:
        return raw.reshape(-1).copy(), None, 0, len(raw)
    tiles = np.empty_like(raw)
    tiles[compressed, :PACKED_TILE_BYTES] = packed[compressed]
    tiles[~compressed] = raw[~compressed]
    data = tiles[np.arange(RAW_TILE_BYTES) < lengths[:, None]]
    return data, headers.view(np.uint8), encoded, len(raw) - encoded


def device_rows(weights, raw: torch.Tensor):
    """Descriptors [n, 3] (device int64) for independently owned compact device
    rows of `weights` (sequence of BF16 rows); rows that do not pack point at
    the matching row of `raw`.  Returns (descriptors, owners, bytes)."""
    rows, owners, total = [], [], 0
    for i, source in enumerate(weights):
        data, meta, _, _ = encode(source)
        if meta is None:
            rows.append((0, 0, raw[i].data_ptr()))
            total += raw[i].numel() * raw[i].element_size()
        else:
            d = torch.from_numpy(data).to(raw.device)
            h = torch.from_numpy(meta).to(raw.device)
            owners.extend((d, h))
            rows.append((d.data_ptr(), h.data_ptr(), -1))
            total += data.size + meta.size
    return torch.tensor(rows, dtype=torch.int64, device=raw.device), owners, total


class ResidentArena:
    """One device arena holding experts of one or more banks in two audited,
    interchangeable layouts ("raw" BF16 rows or "packed" compact rows), with
    per-layout descriptor tables for NativeBf16Gather.copy.

    banks: list of [E, ...] BF16 tensors (CPU); experts: the expert ids to
    hold.  descriptors(mode) -> int64 [banks, E, 3] on the device.
    """

    def __init__(self, banks, experts, device, capacity_bytes: int | None = None):
        from lightreason_b200.native_bf16_gather import NativeBf16Gather

        self.banks = [b.detach().cpu().contiguous() for b in banks]
        self.experts = list(experts)
        self.device = torch.device(device)
        self.native = NativeBf16Gather()
        n_exp = self.banks[0].shape[0]
        encoded = {}
        packed_total = 0
        for e in self.experts:
            for b, bank in enumerate(self.banks):
                data, headers, _, _ = encode(bank[e])
                encoded[e, b] = (data, headers)
                packed_total += (data.size + (headers.size if headers is not None else 0) + 127) // 128 * 128
        raw_total = sum(bank[0].numel() * 2 for bank in self.banks) * len(self.experts)
        self.capacity = capacity_bytes or max(raw_total, packed_total)
        self.buffer = torch.empty(self.capacity, dtype=torch.uint8, device=self.device)
        self.used = {"raw": raw_total, "packed": packed_total}
        self._host = {}
        self.tables = {}
        for mode in ("raw", "packed"):
            host = torch.zeros(self.capacity, dtype=torch.uint8)
            table = torch.zeros((len(self.banks), n_exp, 3), dtype=torch.int64)
            off = 0
            for e in self.experts:
                for b, bank in enumerate(self.banks):
                    if mode == "raw":
                        row = bank[e].view(torch.uint8).reshape(-1)
                        host[off:off + row.numel()] = row
                        table[b, e] = torch.tensor((0, 0, self.buffer.data_ptr() + off))
                        off += (row.numel() + 127) // 128 * 128
                    else:
                        data, headers = encoded[e, b]
                        host[off:off + data.size] = torch.from_numpy(data)
                        if headers is None:
                            table[b, e] = torch.tensor((0, 0, self.buffer.data_ptr() + off))
                            off += (data.size + 127) // 128 * 128
                        else:
                            meta = (off + data.size + 127) // 128 * 128
                            host[meta:meta + headers.size] = torch.from_numpy(headers)
                            table[b, e] = torch.tensor((self.buffer.data_ptr() + off, self.buffer.data_ptr() + meta,
                                                        -1))
                            off = (meta + headers.size + 127) // 128 * 128
            self._host[mode] = host
            self.tables[mode] = table.to(self.device)
        self.mode = None

    def select(self, mode: str) -> None:
        if mode not in self._host:
            raise ValueError(f"unknown arena layout {mode!r}")
        self.buffer.copy_(self._host[mode].to(self.device, non_blocking=False))
        self.mode = mode

    def descriptors(self, mode: str | None = None) -> torch.Tensor:
        return self.tables[mode or self.mode]

    def audit(self) -> int:
        """Reconstruct every held projection through the gather kernel and
        compare the bits with the source rows; returns the values checked."""
        if self.mode is None:
            raise RuntimeError("select a layout first")
        dev = self.device
        outputs = [torch.empty_like(bank[0], device=dev) for bank in self.banks]
        dests = torch.tensor([t.data_ptr() for t in outputs], device=dev, dtype=torch.int64)
        sizes = torch.tensor([t.numel() * 2 for t in outputs], device=dev, dtype=torch.int64)
        zero = torch.zeros(1, device=dev, dtype=torch.int32)
        count = torch.ones(1, device=dev, dtype=torch.int64)
        table = self.descriptors()
        values = 0
        for e in self.experts:
            desc = table[:, e:e + 1].contiguous()
            self.native.copy(desc, dests, sizes, zero, zero, count, max_copies=1, experts=1, geometry=GEOMETRY)
            for b, out in enumerate(outputs):
                if not torch.equal(out.view(torch.int16).cpu(), self.banks[b][e].view(torch.int16)):
                    raise RuntimeError(f"GPU {self.mode} weight audit failed at expert {e}, bank {b}")
                values += out.numel()
        return values
