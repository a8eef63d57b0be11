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


def _flat_bits(source) -> np.ndarray:
    if isinstance(source, torch.Tensor):
        source = source.detach().cpu().contiguous().view(torch.int16).numpy()
    return np.ascontiguousarray(source).view(np.uint16).reshape(-1)


def compact_layout(bases: np.ndarray):
    """Byte layout of a compact row from its tile bases: (tile start offsets,
    headers uint32, data bytes).  Tile t starts at 384 t + 128 p(t), p(t) =
    raw tiles before t, since every tile takes its 384 packed bytes and a raw
    tile 128 more; its header is (p(t) << 8) | base."""
    is_raw = (np.asarray(bases) == RAW_TILE).astype(np.int64)
    prior = np.zeros_like(is_raw)
    np.cumsum(is_raw[:-1], out=prior[1:])
    starts = PACKED_TILE_BYTES * np.arange(is_raw.size) + (RAW_TILE_BYTES - PACKED_TILE_BYTES) * prior
    headers = ((prior << 8) | np.asarray(bases, dtype=np.int64)).astype("<u4")
    return starts, headers, PACKED_TILE_BYTES * is_raw.size + (RAW_TILE_BYTES - PACKED_TILE_BYTES) * int(is_raw.sum())


def encode(source):
    """Compact row of a BF16 tensor or uint16 array: (data, headers|None,
    encoded tiles, raw tiles), the result edge35b/gpu_resident_experts.py:22-42
    returns.  A row whose compact bytes plus headers would not be smaller than
    its raw bytes is returned raw (headers None)."""
    bits = _flat_bits(source)
    packed, bases, encoded = pack_tiles(bits)
    tiles = bases.size
    starts, headers, data_bytes = compact_layout(bases)
    if data_bytes + headers.nbytes >= bits.nbytes:
        return bits.view(np.uint8).copy(), None, 0, tiles
    data = np.empty(data_bytes, dtype=np.uint8)
    sources = (packed, bits.view(np.uint8).reshape(tiles, RAW_TILE_BYTES))
    for raw_tile, width in ((False, PACKED_TILE_BYTES), (True, RAW_TILE_BYTES)):
        sel = (bases == RAW_TILE) == raw_tile
        data[starts[sel, None] + np.arange(width)] = sources[raw_tile][sel, :width]
    return data, headers.view(np.uint8), encoded, tiles - encoded


def _device_bits(source, device) -> torch.Tensor:
    if isinstance(source, torch.Tensor):
        return source.detach().reshape(-1).view(torch.int16).to(device)
    return torch.from_numpy(_flat_bits(source).view(np.int16)).to(device)


def device_rows(weights, raw: torch.Tensor):
    """Descriptors [n, 3] (device int64) of compact device copies of `weights`
    (a sequence of equally sized BF16 rows: tensors or uint16 arrays), built on
    the device: moe_tilecodec_pack then moe_tilecodec_compact into one arena,
    each row's data and headers 128-byte aligned.  A row that does not shrink
    points at the matching row of `raw` instead (`(0, 0, raw ptr)`), a compact
    one is `(data ptr, headers ptr, -1)` (edge35b/gpu_resident_experts.py:45-59
    descriptors).  Returns (descriptors, owners, bytes of the device rows)."""
    from lightreason_b200 import native

    device = raw.device
    rows = torch.stack([_device_bits(w, device) for w in weights])
    n_rows, n = rows.shape
    tiles = n // TILE_VALUES
    packed, bases, _ = native.tilecodec_pack(rows.reshape(-1))
    raw_tiles = (bases.view(n_rows, tiles) == RAW_TILE).sum(dim=1).cpu().numpy().astype(np.int64)
    data_bytes = PACKED_TILE_BYTES * tiles + (RAW_TILE_BYTES - PACKED_TILE_BYTES) * raw_tiles
    header_bytes = 4 * tiles
    shrinks = data_bytes + header_bytes < RAW_TILE_BYTES * tiles
    align = lambda v: (v + 127) // 128 * 128  # noqa: E731
    span = np.where(shrinks, align(data_bytes) + align(header_bytes), 0)
    first = np.concatenate(([0], np.cumsum(span)[:-1]))
    data_off = np.where(shrinks, first, -1)
    header_off = np.where(shrinks, first + align(data_bytes), 0)
    arena = torch.empty(max(int(span.sum()), 128), dtype=torch.uint8, device=device)
    written = native.tilecodec_compact(rows, packed, bases, arena, torch.from_numpy(data_off).to(device),
                                       torch.from_numpy(header_off).to(device))
    if not torch.equal(written.cpu(), torch.from_numpy(np.where(shrinks, data_bytes, 0))):
        raise RuntimeError("Compact expert rows did not fit their arena layout")
    base = arena.data_ptr()
    table = [(base + int(d), base + int(h), -1) if keep else (0, 0, raw[i].data_ptr())
             for i, (keep, d, h) in enumerate(zip(shrinks, data_off, header_off))]
    total = int(np.where(shrinks, data_bytes + header_bytes, RAW_TILE_BYTES * tiles).sum())
    return torch.tensor(table, dtype=torch.int64, device=device), [arena], total


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
