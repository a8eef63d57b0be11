"""Lossless BF16 row codec for host-resident expert banks (host-side encoder).

Same format, function names and semantics as edge35b/bf16_expert_codec.py
(:26-84), the layout the reference streams over PCIe and that
bf16_gather_ada.cu gather<> decodes; the B200 decoder is the row-codec path of
moe_gather_rows and of moe_layer_forward's packed host banks.

A row of n BF16 values packs into 3n/2 + 6*escapes bytes:
  bytes [0, n)         sign (bit 7) and 7-bit fraction of every value,
  bytes [n, 3n/2)      exponent - base as a 4-bit nibble (even values in the low
                       nibble), for a 16-exponent window starting at `base`,
  then escapes int32 indices (ascending) and escapes uint16 raw values of the
  values whose exponent falls outside the window.
`base` is the window start holding the most values (first maximum wins).
plan_bank keeps a row raw when its escapes exceed 1% of its values and aligns
packed rows to 16 bytes.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

WINDOW = 16
ALIGN = 16


def _flat_bits(bits) -> np.ndarray:
    a = np.asarray(bits)
    if a.dtype != np.uint16:
        a = a.view(np.uint16)
    return a.reshape(-1)


def exponent_window(bits):
    """(base, escapes) of the 16-exponent window holding the most values."""
    bits = _flat_bits(bits)
    if bits.size % 8 or not 0 < bits.size < 2 ** 31:
        raise ValueError("Expected a flat BF16 bit array whose length is a positive multiple of 8")
    counts = np.bincount((bits >> 7) & 0xFF, minlength=256).astype(np.int64)
    running = np.concatenate(([0], np.cumsum(counts)))
    inside = running[WINDOW:] - running[:-WINDOW]          # inside[b] = values with exponent in [b, b+16)
    base = int(np.argmax(inside))
    return base, int(bits.size - inside[base])


def row_bytes(n: int, escapes: int) -> int:
    return 3 * n // 2 + 6 * escapes


def pack_row(bits, base: int, escapes: int, output: np.ndarray) -> None:
    """Write one row's packed bytes into `output` (exactly row_bytes long)."""
    bits = _flat_bits(bits)
    n = bits.size
    delta = ((bits >> 7) & 0xFF).astype(np.int32) - base
    # a delta outside [0, 16) has bits above the low nibble (negative ones too)
    escaped = np.flatnonzero(delta & ~0xF)
    if escaped.size != escapes or output.size != row_bytes(n, escapes):
        raise ValueError("BF16 row disagrees with its packed layout")
    sign_fraction = ((bits >> 8) & 0x80 | bits & 0x7F).astype(np.uint8)
    pairs = (delta & 0xF).astype(np.uint8).reshape(-1, 2)
    nibbles = pairs[:, 0] | (pairs[:, 1] << 4)
    output[:] = np.concatenate((sign_fraction, nibbles, escaped.astype("<i4").view(np.uint8),
                                bits[escaped].astype("<u2").view(np.uint8)))


def restore_row(packed: np.ndarray, n: int, base: int, escapes: int) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    sign_fraction = packed[:n].astype(np.uint16)
    nibbles = packed[n:3 * n // 2]
    exponent = np.empty(n, dtype=np.uint16)
    exponent[0::2] = nibbles & 0xF
    exponent[1::2] = nibbles >> 4
    bits = ((sign_fraction & 0x80) << 8) | (sign_fraction & 0x7F) | ((exponent + base) << 7).astype(np.uint16)
    tail = packed[3 * n // 2:]
    where = tail[:4 * escapes].view("<i4")
    bits[where] = tail[4 * escapes:6 * escapes].view("<u2")
    return bits


def pack_verified_row(row, output, base: int, escapes: int) -> None:
    """pack_row, then decode the bytes again and require the original bits (the
    reference's audit; no 1% rule here)."""
    pack_row(row, base, escapes, output)
    bits = _flat_bits(row)
    if not np.array_equal(restore_row(output, bits.size, base, escapes), bits):
        raise RuntimeError("Packed expert did not round-trip to the original BF16 bits")


def _bank_rows(bits) -> np.ndarray:
    a = np.asarray(bits)
    if a.dtype != np.uint16:
        a = a.view(np.uint16)
    return a.reshape(a.shape[0], -1)


def _bank_windows(rows: np.ndarray, *, check=None, threads: int = 1):
    """(bases, escapes) int64 arrays for every row of a bank [E, n]: exponent
    histograms per row (check() runs before each row's), then the 16-exponent
    window sums of all rows at once from the cumulative histograms."""
    if rows.shape[1] % 8 or not 0 < rows.shape[1] < 2 ** 31:
        raise ValueError("Expected a flat BF16 bit array whose length is a positive multiple of 8")

    def hist(row):
        if check is not None:
            check()
        return np.bincount((row >> 7) & 0xFF, minlength=256)

    if threads > 1 and len(rows) > 1:
        with ThreadPoolExecutor(threads) as pool:
            hists = np.stack(list(pool.map(hist, rows)))
    else:
        hists = np.stack([hist(r) for r in rows]) if len(rows) else np.zeros((0, 256), np.int64)
    cum = np.zeros((len(rows), 257), dtype=np.int64)
    np.cumsum(hists, axis=1, out=cum[:, 1:])
    inside = cum[:, WINDOW:] - cum[:, :-WINDOW]             # [E, 241]
    bases = inside.argmax(axis=1)                            # first maximum wins
    escapes = rows.shape[1] - np.take_along_axis(inside, bases[:, None], axis=1)[:, 0]
    return bases.astype(np.int64), escapes.astype(np.int64)


def _layout(n: int, bases: np.ndarray, escapes: np.ndarray):
    """Plan rows from the windows: a row with escapes above 1% of n stays raw
    (None); packed rows follow each other at 16-byte-aligned offsets."""
    packed = escapes * 100 <= n
    span = np.where(packed, (row_bytes(n, 0) + 6 * escapes + ALIGN - 1) // ALIGN * ALIGN, 0)
    offsets = np.zeros(len(span), dtype=np.int64)
    np.cumsum(span[:-1], out=offsets[1:])
    rows = [(int(o), int(b), int(e)) if p else None for o, b, e, p in zip(offsets, bases, escapes, packed)]
    return rows, int(span.sum())


def plan_bank(bits, *, check=None):
    """Rows of a bank [E, ...]: (offset, base, escapes), or None for a row kept
    raw (escapes above 1% of its values); offsets aligned to 16 bytes.
    check() (e.g. a cancellation hook) runs once per row."""
    rows = _bank_rows(bits)
    return _layout(rows.shape[1], *_bank_windows(rows, check=check))


def pack_bank(bank: np.ndarray, *, threads: int = 0):
    """Pack a whole bank [E, ...] (uint16 BF16 bits).  Returns (packed uint8
    buffer, plan rows as in plan_bank).  Every packed row is verified."""
    rows = _bank_rows(np.ascontiguousarray(bank))
    workers = threads or min(32, os.cpu_count() or 1)
    plan, size = _layout(rows.shape[1], *_bank_windows(rows, threads=workers))
    out = np.zeros(max(size, ALIGN), dtype=np.uint8)
    todo = [(e, p) for e, p in enumerate(plan) if p is not None]

    def fill(item):
        e, (off, base, escapes) = item
        pack_verified_row(rows[e], out[off:off + row_bytes(rows.shape[1], escapes)], base, escapes)

    with ThreadPoolExecutor(workers) as pool:
        list(pool.map(fill, todo))
    return out, plan
