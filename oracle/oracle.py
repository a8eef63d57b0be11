"""numpy-level wrapper around the CPU checker in oracle/moe_oracle.c.

TEST INFRASTRUCTURE ONLY.  The product package (lightreason_b200) never imports
this module; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs do, as the checker of the CUDA path.

Arrays of BF16 values are passed as uint16 bit patterns.  Each function names
the reference code it restates through the C function it wraps.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libmoe_oracle.so"
REF_EXPERTS = HERE / "_ref" / "libcpu_experts.so"
REF_TILES = HERE / "_ref" / "libref_tiles.so"

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64


def build() -> None:
    """Compile the checker (and the reference's CPU code when its tree is mounted)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    # the reference checkout: REFERENCE_ROOT, else a sibling of this repository
    root = os.environ.get("REFERENCE_ROOT", str(HERE.parent.parent / "reference"))
    if Path(root, "edge35b", "cpu_experts.c").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REFERENCE_ROOT={root}"], check=True)


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    if not LIB.exists():
        build()
    so = ctypes.CDLL(str(LIB))
    sigs = {
        "or_linear_bf16": [_p, _p, _i, _i, _i, _p],
        "or_router_select": [_p, _p, _i, _i, _i, _p, _p, _p],
        "or_permute": [_p, _i, _i, _i, _p, _p, _p, _p],
        "or_experts": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
        "or_shared_expert": [_p, _p, _p, _p, _p, _i, _i, _i, _p, _p],
        "or_combine": [_p, _p, _p, _i, _i, _i, _p, _p, _p],
        "or_exponent_window": [_p, _i64, _p, _p],
        "or_row_pack": [_p, _i64, ctypes.c_int32, _i64, _p],
        "or_row_restore": [_p, _i64, ctypes.c_int32, _i64, _p],
        "or_tile_pack": [_p, _p, _p, _i64],
        "or_compact_encode": [_p, _i64, _p, _p, _p, _p],
        "or_gather_rows": [_p, _p, _p, _p, _p, _i64, _i, _i, _i],
        "or_moe_layer": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p],
    }
    for name, args in sigs.items():
        fn = getattr(so, name)
        fn.argtypes = args
        fn.restype = _i64 if name in ("or_row_bytes", "or_tile_pack") else _i
    so.or_row_bytes.argtypes = [_i64, _i64]
    so.or_row_bytes.restype = _i64
    return so


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    if not a.flags.c_contiguous:
        raise ValueError("oracle arrays must be C-contiguous")
    return a.ctypes.data


def _check(rc: int) -> None:
    if rc != 0:
        raise ValueError(f"oracle rejected its arguments (status {rc})")


def _u16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a).view(np.uint16) if np.asarray(a).dtype != np.uint16 else a)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = ((x.view(np.uint32)[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ------------------------------------------------------------------ layer ---

def linear_bf16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """F.linear on BF16 with FP32 accumulation (or_linear_bf16)."""
    x, w = _u16(x), _u16(w)
    tokens, width = x.shape
    rows = w.shape[0]
    out = np.empty((tokens, rows), dtype=np.uint16)
    _check(lib().or_linear_bf16(_ptr(x), _ptr(w), tokens, rows, width, _ptr(out)))
    return out


def router_select(logits: np.ndarray, bias: np.ndarray | None, top_k: int = 8):
    """TF:762-770 selection on given BF16 logits (+FP32 bias): ids, f32 and bf16 scores."""
    logits = _u16(logits)
    tokens, experts = logits.shape
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    idx = np.empty((tokens, top_k), dtype=np.int64)
    sf = np.empty((tokens, top_k), dtype=np.float32)
    sb = np.empty((tokens, top_k), dtype=np.uint16)
    _check(lib().or_router_select(_ptr(logits), _ptr(bias), tokens, experts, top_k, _ptr(idx), _ptr(sf), _ptr(sb)))
    return idx, sf, sb


def permute(idx: np.ndarray, experts: int):
    """TF:730-744 eager order: offsets, perm_token, perm_slot, route_pos."""
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    tokens, top_k = idx.shape
    offsets = np.empty(experts + 1, dtype=np.int32)
    ptok = np.empty(tokens * top_k, dtype=np.int32)
    pslot = np.empty(tokens * top_k, dtype=np.int32)
    rpos = np.empty(tokens * top_k, dtype=np.int32)
    _check(lib().or_permute(_ptr(idx), tokens, top_k, experts, _ptr(offsets), _ptr(ptok), _ptr(pslot), _ptr(rpos)))
    return offsets, ptok, pslot, rpos.reshape(tokens, top_k)


def experts_by_route(x: np.ndarray, gate_up: dict | np.ndarray, down: dict | np.ndarray,
                     offsets: np.ndarray, perm_token: np.ndarray, experts: int) -> np.ndarray:
    """BF16 down projection of every route position (cpu_experts.c arithmetic).

    gate_up/down: arrays [E, 2I, H] / [E, H, I] of uint16, or dicts {expert: array}
    holding only the experts that are routed.
    """
    x = _u16(x)
    tokens, hidden = x.shape

    def table(src):
        keep, ptrs = [], (ctypes.c_void_p * experts)()
        for e in range(experts):
            if offsets[e + 1] == offsets[e]:
                continue
            a = _u16(src[e])
            keep.append(a)
            ptrs[e] = a.ctypes.data
        return ptrs, keep

    gptrs, gkeep = table(gate_up)
    dptrs, dkeep = table(down)
    any_e = next(iter(gkeep)) if gkeep else None
    inner = (any_e.shape[0] // 2) if any_e is not None else 512
    routes = int(offsets[experts])
    y = np.empty((max(routes, 1), hidden), dtype=np.uint16)
    _check(lib().or_experts(_ptr(x), ctypes.cast(gptrs, _p), ctypes.cast(dptrs, _p), _ptr(offsets),
                            _ptr(np.ascontiguousarray(perm_token, dtype=np.int32)), experts, hidden, inner,
                            tokens, _ptr(y)))
    return y[:routes]


def shared_expert(x, gate_w, up_w, down_w, sgate_w):
    """TF:698-711 shared MLP and the sigmoid of TF:779 shared_expert_gate."""
    x = _u16(x)
    tokens, hidden = x.shape
    gate_w, up_w, down_w, sgate_w = (_u16(a) for a in (gate_w, up_w, down_w, sgate_w))
    inner = gate_w.shape[0]
    out = np.empty((tokens, hidden), dtype=np.uint16)
    sig = np.empty(tokens, dtype=np.uint16)
    _check(lib().or_shared_expert(_ptr(x), _ptr(gate_w), _ptr(up_w), _ptr(down_w), _ptr(sgate_w.reshape(-1)),
                                  tokens, hidden, inner, _ptr(out), _ptr(sig)))
    return out, sig


def combine(y, route_pos, scores_bf16, shared_out=None, sig=None):
    """Ordered BF16 combine of TF:749-750 and TF:788-790."""
    y = _u16(y)
    route_pos = np.ascontiguousarray(route_pos, dtype=np.int32)
    scores_bf16 = _u16(scores_bf16)
    tokens, top_k = route_pos.shape
    hidden = y.shape[1]
    out = np.empty((tokens, hidden), dtype=np.uint16)
    _check(lib().or_combine(_ptr(y), _ptr(route_pos), _ptr(scores_bf16), tokens, top_k, hidden,
                            _ptr(None if shared_out is None else _u16(shared_out)),
                            _ptr(None if sig is None else _u16(sig)), _ptr(out)))
    return out


def moe_layer(x, router_w, bias, gate_up, down, sh_gate, sh_up, sh_down, sh_gate_w, top_k=8):
    """Whole Qwen3_5MoeSparseMoeBlock.forward (TF:781-792) with BF16 router scores.

    gate_up/down may be dicts holding only the routed experts; the router
    decides which are needed, so this routes first and then checks the dict.
    Returns (out, idx, scores_bf16, logits).
    """
    x = _u16(x)
    router_w = _u16(router_w)
    experts = router_w.shape[0]
    logits = linear_bf16(x, router_w)
    idx, _, scores = router_select(logits, bias, top_k)
    offsets, ptok, _, rpos = permute(idx, experts)
    y = experts_by_route(x, gate_up, down, offsets, ptok, experts)
    sh, sig = shared_expert(x, sh_gate, sh_up, sh_down, sh_gate_w)
    out = combine(y, rpos, scores, sh, sig)
    return out, idx, scores, logits


# ----------------------------------------------------------------- codecs ---

def exponent_window(bits: np.ndarray):
    bits = _u16(bits).reshape(-1)
    base, esc = ctypes.c_int32(), ctypes.c_int64()
    lib().or_exponent_window(_ptr(bits), bits.size, ctypes.byref(base), ctypes.byref(esc))
    return base.value, esc.value


def row_bytes(n: int, escapes: int) -> int:
    return int(lib().or_row_bytes(n, escapes))


def row_pack(bits: np.ndarray, base: int, escapes: int) -> np.ndarray:
    bits = _u16(bits).reshape(-1)
    out = np.zeros(row_bytes(bits.size, escapes), dtype=np.uint8)
    _check(lib().or_row_pack(_ptr(bits), bits.size, base, escapes, _ptr(out)))
    return out


def row_restore(packed: np.ndarray, n: int, base: int, escapes: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().or_row_restore(_ptr(np.ascontiguousarray(packed, dtype=np.uint8)), n, base, escapes, _ptr(out))
    return out


def tile_pack(raw: np.ndarray):
    raw = _u16(raw).reshape(-1)
    tiles = raw.size // 256
    packed = np.zeros(tiles * 384, dtype=np.uint8)
    bases = np.zeros(tiles, dtype=np.uint8)
    encoded = lib().or_tile_pack(_ptr(raw), _ptr(packed), _ptr(bases), tiles)
    return packed, bases, int(encoded)


def compact_encode(raw: np.ndarray):
    """gpu_resident_experts.encode restated: (data, headers|None, encoded, fallback)."""
    raw = _u16(raw).reshape(-1)
    tiles = raw.size // 256
    data = np.zeros(tiles * 512, dtype=np.uint8)
    headers = np.zeros(tiles, dtype=np.uint32)
    size, enc = ctypes.c_int64(), ctypes.c_int64()
    kept_raw = lib().or_compact_encode(_ptr(raw), tiles, _ptr(data), _ptr(headers), ctypes.byref(size),
                                       ctypes.byref(enc))
    if kept_raw:
        return raw.view(np.uint8).copy(), None, 0, tiles
    return data[:size.value].copy(), headers.view(np.uint8).copy(), enc.value, tiles - enc.value


def gather_rows(descriptors, destinations, sizes, src_ids, dst_ids, count, experts, mode):
    """Host emulation of the bf16_gather_ada.cu copies (pointers are host addresses)."""
    descriptors = np.ascontiguousarray(descriptors, dtype=np.int64)
    banks = descriptors.shape[0]
    _check(lib().or_gather_rows(_ptr(descriptors), _ptr(np.ascontiguousarray(destinations, dtype=np.int64)),
                                _ptr(np.ascontiguousarray(sizes, dtype=np.int64)),
                                _ptr(np.ascontiguousarray(src_ids, dtype=np.int32)),
                                _ptr(np.ascontiguousarray(dst_ids, dtype=np.int32)), int(count), experts, banks,
                                mode))


# -------------------------------------------------- the reference's own C ---

@lru_cache(maxsize=1)
def ref_experts_lib() -> ctypes.CDLL | None:
    """edge35b/cpu_experts.c compiled from the reference sources, if built."""
    if not REF_EXPERTS.exists():
        return None
    so = ctypes.CDLL(str(REF_EXPERTS))
    so.expert_rows.argtypes = [_p, _p, _p, _p, _i, _i]
    so.expert_rows.restype = None
    so.expert_block_rows.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i]
    so.expert_block_rows.restype = None
    return so


@lru_cache(maxsize=1)
def ref_tiles_lib() -> ctypes.CDLL | None:
    if not REF_TILES.exists():
        return None
    so = ctypes.CDLL(str(REF_TILES))
    so.ref_pack_cpu_read_tiles.argtypes = [_p, _p, _p, ctypes.c_size_t]
    so.ref_pack_cpu_read_tiles.restype = ctypes.c_size_t
    return so


def ref_expert_block_rows(x, gate_up_rows, down_rows, token_ids, threads=8):
    """Call the reference's expert_block_rows (cpu_experts.c:74-105) on host arrays."""
    so = ref_experts_lib()
    if so is None:
        raise RuntimeError("oracle/_ref/libcpu_experts.so is not built")
    x = _u16(x)
    pairs = len(gate_up_rows)
    gp = (ctypes.c_void_p * pairs)(*[_u16(a).ctypes.data for a in gate_up_rows])
    dp = (ctypes.c_void_p * pairs)(*[_u16(a).ctypes.data for a in down_rows])
    tid = np.ascontiguousarray(token_ids, dtype=np.int32)
    out = np.empty((pairs, x.shape[1]), dtype=np.uint16)
    so.expert_block_rows(ctypes.cast(gp, _p), ctypes.cast(dp, _p), _ptr(x), _ptr(tid), _ptr(out), x.shape[0], pairs,
                         threads)
    return out
