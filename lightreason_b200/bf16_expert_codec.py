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
    bits = _flat_bits(bits)
    n = bits.size
    exponent = ((bits >> 7) & 0xFF).astype(np.int32) - base
    outside = np.flatnonzero((exponent < 0) | (exponent >= WINDOW))
    if outside.size != escapes or output.size != row_bytes(n, escapes):
        raise ValueError("BF16 row disagrees with its packed layout")
    nib = (exponent & 0xF).astype(np.uint8)
    output[:n] = ((bits >> 8) & 0x80).astype(np.uint8) | (bits & 0x7F).astype(np.uint8)
    output[n:3 * n // 2] = nib[0::2] | (nib[1::2] << 4)
    tail = output[3 * n // 2:]
    tail[:4 * escapes].view("<i4")[:] = outside.astype(np.int32)
    tail[4 * escapes:].view("<u2")[:] = bits[outside]


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
    pack_row(row, base, escapes, output)
    if not np.array_equal(_flat_bits(row), restore_row(output, _flat_bits(row).size, base, escapes)):
        raise RuntimeError("Packed expert did not round-trip to the original BF16 bits")


def plan_bank(bits, *, check=None):
    """Rows of a bank [E, ...]: (offset, base, escapes), or None for a row kept
    raw (escapes above 1% of its values); offsets aligned to 16 bytes."""
    rows, size = [], 0
    for row in np.asarray(bits).reshape(len(bits), -1):
        if check is not None:
            check()
        base, escapes = exponent_window(row)
        if escapes * 100 > row.size:
            rows.append(None)
            continue
        rows.append((size, base, escapes))
        size = (size + row_bytes(row.size, escapes) + ALIGN - 1) & ~(ALIGN - 1)
    return rows, size


def pack_bank(bank: np.ndarray, *, threads: int = 0):
    """Pack a whole bank [E, ...] (uint16 BF16 bits).  Returns (packed uint8
    buffer, plan rows as in plan_bank).  Every packed row is verified."""
    bank = np.ascontiguousarray(bank)
    flat = bank.reshape(bank.shape[0], -1).view(np.uint16)
    with ThreadPoolExecutor(threads or min(32, os.cpu_count() or 1)) as pool:
        windows = list(pool.map(exponent_window, flat))
    rows, size = [], 0
    for (base, escapes), row in zip(windows, flat):
        if escapes * 100 > row.size:
            rows.append(None)
            continue
        rows.append((size, base, escapes))
        size = (size + row_bytes(row.size, escapes) + ALIGN - 1) & ~(ALIGN - 1)
    out = np.zeros(max(size, ALIGN), dtype=np.uint8)

    def fill(e):
        if rows[e] is not None:
            off, base, escapes = rows[e]
            pack_verified_row(flat[e], out[off:off + row_bytes(flat.shape[1], escapes)], base, escapes)

    with ThreadPoolExecutor(threads or min(32, os.cpu_count() or 1)) as pool:
        list(pool.map(fill, range(len(rows))))
    return out, rows
