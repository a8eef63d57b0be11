"""ctypes binding of libmoe_b200.so and thin torch wrappers around its C ABI.

This is the only route from Python to the device code.  There is no fallback:
if the library is missing or the GPU is not sm_100, every call raises.
Status codes map to exceptions the way the reference's APIs raise them:
argument errors -> ValueError (edge35b/fused_experts.py:41-50), CUDA failures
-> RuntimeError (edge35b/native_bf16_gather.py:25-29).
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libmoe_b200.so"

MOE_OK, MOE_EINVAL, MOE_ECUDA, MOE_EARCH = 0, 1, 2, 3
CODEC_ROW, CODEC_TILES, CODEC_RESIDENT, CODEC_ROW_L2 = 0, 1, 2, 3

_p = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t


class LayerWeights(ctypes.Structure):
    """moe_layer_weights of include/moe_b200.h."""

    _fields_ = [("router", _p), ("router_bias", _p), ("gate_up", _p), ("down", _p),
                ("gate_up_stride", ctypes.c_int64), ("down_stride", ctypes.c_int64),
                ("shared_gate", _p), ("shared_up", _p), ("shared_down", _p), ("shared_gate_w", _p),
                ("experts", _i), ("hidden", _i), ("inner", _i), ("shared_inner", _i), ("top_k", _i)]


class EpP2P(ctypes.Structure):
    """moe_ep_p2p: the peer-memory exchange of one expert-parallel rank."""
    _fields_ = [("peers", _p), ("off_flags_publish", ctypes.c_int64), ("off_flags_return", ctypes.c_int64),
                ("off_count", ctypes.c_int64), ("off_meta", ctypes.c_int64), ("off_tokens", ctypes.c_int64),
                ("off_ret", ctypes.c_int64), ("world", _i), ("rank", _i), ("capacity", _i), ("hidden", _i),
                ("top_k", _i), ("experts", _i), ("local_experts", _i), ("own_rows", _i), ("step", _p),
                ("sync", _p), ("error", _p), ("placement", _p)]


class LayerIO(ctypes.Structure):
    """moe_layer_io of include/moe_b200.h."""

    _fields_ = [("route_in", _p), ("weights_in", _p), ("idx_out", _p), ("scores_out", _p), ("logits_out", _p),
                ("host_gate_up", _p), ("host_down", _p), ("gate_up_slots", _p), ("down_slots", _p),
                ("max_slots", _i), ("host_descriptors", _p), ("stage_events", ctypes.POINTER(_p)),
                ("num_stage_events", _i), ("status", _p), ("rows_mode", _i), ("expert_cache", _p)]


_SIGNATURES = {
    "moe_version": ([], _i),
    "moe_last_error": ([], ctypes.c_char_p),
    "moe_device_check": ([_i], _i),
    "moe_host_register": ([_p, _sz, ctypes.POINTER(ctypes.c_uint64)], _i),
    "moe_host_unregister": ([_p], _i),
    "moe_router_topk": ([_p, _p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p], _i),
    "moe_router_workspace_bytes": ([_i, _i], _sz),
    "moe_router_topk_ws": ([_p, _p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _sz, _p], _i),
    "moe_router_select": ([_p, _p, _i, _i, _i, _p, _p, _p, _p], _i),
    "moe_permute": ([_p, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p], _i),
    "moe_permute_hist_ints": ([_i, _i, _i], _i),
    "moe_permute_wide": ([_p, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p], _i),
    "moe_expert_rows": ([_p, _p, _p, _p, _i, _p, _sz, _p], _i),
    "moe_expert_block_rows": ([_p, _p, _p, _p, _p, _i, _i, _p, _sz, _p], _i),
    "moe_expert_block_rows_noalloc": ([_p, _p, _p, _p, _p, _i, _i, _p], _i),
    "moe_layer_workspace_bytes": ([_i, _i, _i, _i, _i, _i], _sz),
    "moe_layer_forward": ([ctypes.POINTER(LayerWeights), _p, _i, _p, ctypes.POINTER(LayerIO), _p, _sz, _p], _i),
    "moe_gather_rows": ([_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "moe_stage_primary": ([_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p], _i),
    "moe_gather_compact_tail": ([_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p], _i),
    "moe_rowcodec_workspace_bytes": ([_i, ctypes.c_int64], _sz),
    "moe_rowcodec_plan": ([_p, _i, ctypes.c_int64, _p, _p, _p, _sz, _p], _i),
    "moe_rowcodec_pack": ([_p, _i, ctypes.c_int64, _p, _p, _p, _sz, _p], _i),
    "moe_tilecodec_pack": ([_p, ctypes.c_int64, _p, _p, _p, _p], _i),
    "moe_tilecodec_compact": ([_p, _p, _p, _i, ctypes.c_int64, _p, ctypes.c_int64, _p, _p, _p, _p], _i),
    "moe_ipc_alloc": ([_sz, ctypes.POINTER(_p), _p], _i),
    "moe_ipc_free": ([_p], _i),
    "moe_ipc_open": ([_p, ctypes.POINTER(_p)], _i),
    "moe_ipc_close": ([_p], _i),
    "moe_ep_p2p_route_workspace_bytes": ([ctypes.POINTER(EpP2P), _i], _sz),
    "moe_ep_p2p_route": ([ctypes.POINTER(EpP2P), _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p], _i),
    "moe_ep_p2p_workspace_bytes": ([ctypes.POINTER(EpP2P), _i], _sz),
    "moe_ep_p2p_experts": ([ctypes.POINTER(EpP2P), _p, _p, _i, _i, _p, _p, _p, _sz, ctypes.POINTER(_p), _p], _i),
    "moe_ep_p2p_finish": ([ctypes.POINTER(EpP2P), _p], _i),
    "moe_ep_dispatch": ([_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _p], _i),
    "moe_ep_unpack": ([_p, _i, _p, _p], _i),
    "moe_ep_combine": ([_p, _p, _p, _p, _p, _i, _i, _i, _p, _p], _i),
    "moe_combine": ([_p, _p, _p, _p, _p, _i, _i, _i, _p, _p], _i),
    "moe_shared_expert_workspace_bytes": ([_i, _i], _sz),
    "moe_shared_expert": ([_p, _p, _p, _p, _p, _i, _i, _i, _p, _p, _p, _sz, _p], _i),
    "moe_grouped_paired": ([_i, _i, _i], _i),
}

EXPORTED = tuple(_SIGNATURES)


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    """Load the in-tree library; raise if it was not built."""
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m lightreason_b200.build` "
                           "(there is no CPU fallback)")
    so = ctypes.CDLL(str(LIB_PATH))
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(so, name)
        fn.argtypes = args
        fn.restype = res
    return so


def check(status: int, what: str) -> None:
    if status == MOE_OK:
        return
    msg = f"{what}: {lib().moe_last_error().decode(errors='replace')}"
    if status == MOE_EINVAL:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _bits(t: torch.Tensor) -> torch.Tensor:
    """A BF16 tensor seen as the int16 bit patterns the ABI takes."""
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def device_check(device: torch.device | int | None = None) -> None:
    index = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    check(lib().moe_device_check(index.index if index.index is not None else torch.cuda.current_device()),
          "moe_device_check")


def _cuda_bf16(t: torch.Tensor, name: str) -> None:
    _require(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous(),
             f"{name} must be a contiguous CUDA BF16 tensor")


# ---------------------------------------------------------------- router ---

def router_topk(x: torch.Tensor, router: torch.Tensor, bias: torch.Tensor | None = None,
                shared_gate_w: torch.Tensor | None = None, top_k: int = 8):
    """Router + top-k (+ sigmoid shared gate).  Returns idx int64 [T,K], scores
    f32 [T,K], scores bf16 [T,K], logits bf16 [T,E], sig bf16 [T] or None."""
    _cuda_bf16(x, "x")
    _cuda_bf16(router, "router")
    tokens, hidden = x.shape
    experts = router.shape[0]
    dev = x.device
    logits = torch.empty((tokens, experts), dtype=torch.bfloat16, device=dev)
    idx = torch.empty((tokens, top_k), dtype=torch.int64, device=dev)
    sf = torch.empty((tokens, top_k), dtype=torch.float32, device=dev)
    sb = torch.empty((tokens, top_k), dtype=torch.bfloat16, device=dev)
    sig = torch.empty(tokens, dtype=torch.bfloat16, device=dev) if shared_gate_w is not None else None
    if bias is not None:
        _require(bias.is_cuda and bias.dtype == torch.float32 and bias.numel() == experts, "bias must be CUDA f32 [E]")
    check(lib().moe_router_topk(_ptr(x), _ptr(router), _ptr(bias), _ptr(shared_gate_w), tokens, hidden, experts, top_k,
                                _ptr(logits), _ptr(idx), _ptr(sf), _ptr(sb), _ptr(sig), _stream(dev)),
          "moe_router_topk")
    return idx, sf, sb, logits, sig


def router_select(logits: torch.Tensor, bias: torch.Tensor | None = None, top_k: int = 8):
    _cuda_bf16(logits, "logits")
    tokens, experts = logits.shape
    dev = logits.device
    idx = torch.empty((tokens, top_k), dtype=torch.int64, device=dev)
    sf = torch.empty((tokens, top_k), dtype=torch.float32, device=dev)
    sb = torch.empty((tokens, top_k), dtype=torch.bfloat16, device=dev)
    check(lib().moe_router_select(_ptr(logits), _ptr(bias), tokens, experts, top_k, _ptr(idx), _ptr(sf), _ptr(sb),
                                  _stream(dev)), "moe_router_select")
    return idx, sf, sb


# --------------------------------------------------------------- permute ---

def permute(idx: torch.Tensor, experts: int, *, wide: bool = False):
    """Eager dispatch order.  Returns offsets [E+1], perm_token [R], perm_slot
    [R], route_pos [T,K], active [E] (first num_active valid), num_active [1],
    bad_routes [1] (int32, on the device)."""
    _require(idx.is_cuda and idx.dtype == torch.int64 and idx.dim() == 2 and idx.is_contiguous(),
             "idx must be a contiguous CUDA int64 [T, K] tensor")
    tokens, top_k = idx.shape
    dev = idx.device
    i32 = dict(dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, **i32)
    ptok = torch.empty(max(tokens * top_k, 1), **i32)
    pslot = torch.empty(max(tokens * top_k, 1), **i32)
    rpos = torch.empty((tokens, top_k), **i32)
    active = torch.empty(experts, **i32)
    counters = torch.zeros(2, **i32)
    if wide:
        hist = torch.empty(max(lib().moe_permute_hist_ints(tokens, top_k, experts), 1), **i32)
        check(lib().moe_permute_wide(_ptr(idx), tokens, top_k, experts, _ptr(offsets), _ptr(ptok), _ptr(pslot),
                                     _ptr(rpos), _ptr(active), counters.data_ptr(), counters.data_ptr() + 4,
                                     hist.data_ptr(), _stream(dev)), "moe_permute_wide")
    else:
        check(lib().moe_permute(_ptr(idx), tokens, top_k, experts, _ptr(offsets), _ptr(ptok), _ptr(pslot),
                                _ptr(rpos), _ptr(active), counters.data_ptr(), counters.data_ptr() + 4,
                                _stream(dev)), "moe_permute")
    return offsets, ptok[:tokens * top_k], pslot[:tokens * top_k], rpos, active, counters[:1], counters[1:]


# ------------------------------------------------- pointer-table experts ---

def expert_block_rows(gate_up: list, down: list, hidden: torch.Tensor, token_ids: list[int] | None = None):
    """GPU counterpart of cpu_experts.c expert_rows / expert_block_rows: the
    BF16 down projection of each (expert weights, token) pair.  gate_up[i] is a
    [2I,H] and down[i] a [H,I] CUDA BF16 tensor; hidden [T,H]."""
    _cuda_bf16(hidden, "hidden")
    pairs = len(gate_up)
    _require(len(down) == pairs, "gate_up and down need one entry per pair")
    for g, d in zip(gate_up, down):
        _cuda_bf16(g, "gate_up row")
        _cuda_bf16(d, "down row")
    out = torch.empty((pairs, hidden.shape[-1]), dtype=torch.bfloat16, device=hidden.device)
    if pairs == 0:
        return out
    work = torch.empty(pairs * 512 * 2, dtype=torch.uint8, device=hidden.device)
    gp = (ctypes.c_void_p * pairs)(*[t.data_ptr() for t in gate_up])
    dp = (ctypes.c_void_p * pairs)(*[t.data_ptr() for t in down])
    if token_ids is None:
        check(lib().moe_expert_rows(ctypes.cast(gp, _p), ctypes.cast(dp, _p), _ptr(hidden), _ptr(out), pairs,
                                    _ptr(work), work.numel(), _stream(hidden.device)), "moe_expert_rows")
    else:
        tid = (ctypes.c_int32 * pairs)(*token_ids)
        check(lib().moe_expert_block_rows(ctypes.cast(gp, _p), ctypes.cast(dp, _p), _ptr(hidden),
                                          ctypes.cast(tid, _p), _ptr(out), hidden.shape[0], pairs, _ptr(work),
                                          work.numel(), _stream(hidden.device)), "moe_expert_block_rows")
    return out


# ----------------------------------------------------------------- layer ---

def layer_workspace_bytes(tokens: int, experts: int, top_k: int, hidden: int, inner: int) -> int:
    return int(lib().moe_layer_workspace_bytes(tokens, experts, top_k, hidden, inner, inner))


class Layer:
    """Device-resident weights of one MoE layer bound to the C ABI structure.

    gate_up [E,2I,H] and down [E,H,I] may instead be host-resident: pass
    host_gate_up/host_down as pinned CPU tensors (mapped with
    moe_host_register) and the forward gathers the selected experts per call.
    """

    def __init__(self, *, router=None, gate_up=None, down=None, bias=None, shared_gate=None, shared_up=None,
                 shared_down=None, shared_gate_w=None, top_k=8, host_gate_up=None, host_down=None,
                 host_packed=None, device=None, cache_slots=None):
        """router may be None for a layer only called with route_in (the
        Qwen3_5MoeExperts.forward form); experts and hidden then come from the
        banks."""
        if router is not None:
            _cuda_bf16(router, "router")
        self.router, self.bias = router, bias
        self.gate_up, self.down = gate_up, down
        self.shared = (shared_gate, shared_up, shared_down, shared_gate_w)
        ref = gate_up if gate_up is not None else host_gate_up
        if router is not None:
            self.experts, self.hidden = router.shape
        elif host_packed is not None:
            self.experts, self.hidden = host_packed.experts, host_packed.hidden
        else:
            _require(ref is not None, "a router or expert banks are required")
            self.experts, self.hidden = ref.shape[0], ref.shape[2]
        self.top_k = top_k
        self.host_gate_up, self.host_down = host_gate_up, host_down
        self.host_packed = host_packed
        if host_packed is not None:
            _require(host_packed.experts == self.experts and host_packed.hidden == self.hidden,
                     "packed host banks do not match the router")
            self.inner = host_packed.inner
        else:
            bank = gate_up if gate_up is not None else host_gate_up
            dbank = down if down is not None else host_down
            _require(bank is not None and dbank is not None, "expert banks are required")
            self.inner = bank.shape[1] // 2
            _require(tuple(bank.shape) == (self.experts, 2 * self.inner, self.hidden), "gate_up must be [E, 2I, H]")
            _require(tuple(dbank.shape) == (self.experts, self.hidden, self.inner), "down must be [E, H, I]")
        if router is not None:
            self.device = router.device
        elif gate_up is not None:
            self.device = gate_up.device
        else:
            self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                         torch.cuda.current_device())
        self._mapped = []
        self._host_dev = (None, None)
        if host_gate_up is not None:
            self._host_dev = (self._map(host_gate_up), self._map(host_down))
        self.w = LayerWeights(
            router=_ptr(router), router_bias=_ptr(bias), gate_up=_ptr(gate_up), down=_ptr(down),
            gate_up_stride=2 * self.inner * self.hidden, down_stride=self.hidden * self.inner,
            shared_gate=_ptr(shared_gate), shared_up=_ptr(shared_up), shared_down=_ptr(shared_down),
            shared_gate_w=_ptr(shared_gate_w), experts=self.experts, hidden=self.hidden, inner=self.inner,
            shared_inner=(shared_gate.shape[0] if shared_gate is not None else self.inner), top_k=top_k)
        self._slots = None
        self._ws = None
        # expert cache over the host banks: cache_slots slot rows kept across calls
        self.cache_slots = cache_slots
        self.cache = None
        if cache_slots is not None:
            _require(host_gate_up is not None or host_packed is not None, "cache_slots needs host banks")
            _require(0 < cache_slots <= 1024, "cache_slots must be in [1, 1024]")
            self.cache = torch.zeros(self.experts + 2 * cache_slots + 3, dtype=torch.int32, device=self.device)
            self.cache[:self.experts + cache_slots] = -1

    def cache_stats(self) -> dict:
        """Calls, routed-expert uses and misses counted by the expert cache."""
        _require(self.cache is not None, "no expert cache")
        calls, uses, misses = self.cache[-3:].tolist()
        return {"calls": calls, "uses": uses, "misses": misses,
                "hit_rate": (uses - misses) / uses if uses else 0.0}

    def _map(self, t: torch.Tensor) -> int:
        _require(t.device.type == "cpu" and t.is_contiguous() and t.dtype == torch.bfloat16,
                 "host banks must be contiguous CPU BF16 tensors")
        dev = ctypes.c_uint64()
        if t.is_pinned():
            # Memory pinned by torch's allocator is already mapped (UVA).
            return t.data_ptr()
        check(lib().moe_host_register(ctypes.c_void_p(t.data_ptr()), t.numel() * 2, ctypes.byref(dev)),
              "moe_host_register")
        self._mapped.append(t)
        return dev.value

    def release(self) -> None:
        for t in self._mapped:
            lib().moe_host_unregister(ctypes.c_void_p(t.data_ptr()))
        self._mapped.clear()

    def set_top_k(self, top_k: int) -> None:
        """Route width of later calls (the workspace and slots are re-sized)."""
        _require(0 < top_k <= self.experts, "top_k must be in [1, experts]")
        self.top_k = self.w.top_k = top_k
        self._ws = self._slots = None

    def workspace(self, tokens: int) -> torch.Tensor:
        need = layer_workspace_bytes(tokens, self.experts, self.top_k, self.hidden, self.inner)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def slots(self, tokens: int):
        n = min(self.experts, tokens * self.top_k)
        if self.cache_slots is not None:
            _require(self.cache_slots >= n, f"cache_slots {self.cache_slots} < min(E, T*top_k) = {n}")
            n = self.cache_slots
        if self._slots is None or self._slots[0].shape[0] < n:
            self._slots = (torch.empty((n, 2 * self.inner, self.hidden), dtype=torch.bfloat16, device=self.device),
                           torch.empty((n, self.hidden, self.inner), dtype=torch.bfloat16, device=self.device))
        return self._slots

    def forward_rows_raw(self, x_ptr: int, tokens: int, route_in: torch.Tensor, out: torch.Tensor,
                         stage_events=None) -> torch.Tensor:
        """Rows-mode forward whose input rows live at a raw device address (a
        symmetric buffer): x [tokens, H] BF16 at x_ptr, route_in CUDA int64
        [tokens, 1], out [tokens, H]."""
        _require(self.top_k == 1, "rows mode needs top_k 1")
        _require(route_in.dtype == torch.int64 and tuple(route_in.shape) == (tokens, 1) and route_in.is_contiguous()
                 and route_in.is_cuda, "route_in must be CUDA int64 [T, 1]")
        _cuda_bf16(out, "out")
        _require(tuple(out.shape) == (tokens, self.hidden), "out must be [T, H]")
        ws = self.workspace(tokens)
        io = LayerIO(route_in=_ptr(route_in), rows_mode=1)
        if stage_events is not None:
            for e in stage_events:
                if e is not None and not e.cuda_event:
                    e.record()
            handles = (_p * len(stage_events))(*[e.cuda_event if e is not None else None for e in stage_events])
            io.stage_events, io.num_stage_events = ctypes.cast(handles, ctypes.POINTER(_p)), len(stage_events)
        check(lib().moe_layer_forward(ctypes.byref(self.w), ctypes.c_void_p(x_ptr), tokens, _ptr(out),
                                      ctypes.byref(io), _ptr(ws), ws.numel(), _stream(out.device)),
              "moe_layer_forward")
        return out

    def forward(self, x: torch.Tensor, *, route_in=None, weights_in=None, out=None, idx_out=None, scores_out=None,
                logits_out=None, stage_events=None, rows_mode=False) -> torch.Tensor:
        """One layer step on the current stream.  stage_events: optional list of
        8 torch.cuda.Event recorded at the stage boundaries (see moe_layer_io).
        rows_mode (route_in with top_k 1): out[t] = token t's unweighted expert
        row, no combine; weights_in may be None."""
        _cuda_bf16(x, "x")
        tokens = x.shape[0]
        _require(x.shape[1] == self.hidden, "x must be [T, H]")
        if route_in is not None:
            _require(route_in.dtype == torch.int64 and tuple(route_in.shape) == (tokens, self.top_k)
                     and route_in.is_contiguous() and route_in.is_cuda, "route_in must be CUDA int64 [T, K]")
            _require(rows_mode or (weights_in is not None and weights_in.dtype == torch.bfloat16
                                   and tuple(weights_in.shape) == (tokens, self.top_k) and weights_in.is_contiguous()),
                     "weights_in must be CUDA BF16 [T, K]")
        _require(not rows_mode or (route_in is not None and self.top_k == 1), "rows_mode needs route_in and top_k 1")
        out = torch.empty_like(x) if out is None else out
        ws = self.workspace(tokens)
        io = LayerIO(route_in=_ptr(route_in), weights_in=_ptr(weights_in), idx_out=_ptr(idx_out),
                     scores_out=_ptr(scores_out), logits_out=_ptr(logits_out), rows_mode=int(rows_mode))
        if stage_events is not None:
            for e in stage_events:
                if e is not None and not e.cuda_event:
                    e.record()  # torch creates the CUDA event lazily on first record
            handles = (_p * len(stage_events))(*[e.cuda_event if e is not None else None for e in stage_events])
            io.stage_events, io.num_stage_events = ctypes.cast(handles, ctypes.POINTER(_p)), len(stage_events)
        if self.host_gate_up is not None or self.host_packed is not None:
            gs, ds = self.slots(tokens)
            if self.host_packed is not None:
                io.host_descriptors = self.host_packed.descriptors.data_ptr()
            else:
                io.host_gate_up, io.host_down = self._host_dev
            io.gate_up_slots, io.down_slots, io.max_slots = gs.data_ptr(), ds.data_ptr(), gs.shape[0]
            if self.cache is not None:
                io.expert_cache = self.cache.data_ptr()
        check(lib().moe_layer_forward(ctypes.byref(self.w), _ptr(x), tokens, _ptr(out), ctypes.byref(io), _ptr(ws),
                                      ws.numel(), _stream(x.device)), "moe_layer_forward")
        return out

    __call__ = forward


# ---------------------------------------------------------------- gather ---

def gather_rows(descriptors, destinations, sizes, src, dst, count, *, max_copies, experts, codec, stripes,
                threads):
    """Launch the descriptor-driven copy on the current stream (tables are CUDA tensors)."""
    for name, t, dt in (("descriptors", descriptors, torch.int64), ("destinations", destinations, torch.int64),
                        ("sizes", sizes, torch.int64), ("src", src, torch.int32), ("dst", dst, torch.int32),
                        ("count", count, torch.int64)):
        _require(t.is_cuda and t.dtype == dt and t.is_contiguous(), f"{name} must be a contiguous CUDA {dt} tensor")
    banks = destinations.numel()
    check(lib().moe_gather_rows(_ptr(descriptors), _ptr(destinations), _ptr(sizes), _ptr(src), _ptr(dst), _ptr(count),
                                experts, banks, max_copies, codec, stripes, threads, _stream(destinations.device)),
          "moe_gather_rows")


def _table(name, t, dtype, dims=None):
    _require(t.is_cuda and t.dtype == dtype and t.is_contiguous() and (dims is None or t.dim() == dims),
             f"{name} must be a contiguous CUDA {dtype} tensor")


def stage_primary(sources, miss_sources, layouts, prefix_tables, plan, count, *, experts, packed_slots):
    """moe_stage_primary on the current stream (all tables CUDA tensors)."""
    for name, t, dt in (("sources", sources, torch.int64), ("miss_sources", miss_sources, torch.int64),
                        ("layouts", layouts, torch.int64), ("prefix_tables", prefix_tables, torch.int64),
                        ("count", count, torch.int32)):
        _table(name, t, dt)
    _table("plan", plan, torch.int32, 2)
    _require(plan.shape[0] == 3, "plan must be int32 [3, rows]")
    banks = layouts.numel() // 5
    _require(banks * 5 == layouts.numel() and sources.numel() == banks * experts * 3
             and miss_sources.numel() == sources.numel(), "tables disagree with experts / banks")
    check(lib().moe_stage_primary(_ptr(sources), _ptr(miss_sources), _ptr(layouts), _ptr(prefix_tables), _ptr(plan),
                                  _ptr(count), experts, packed_slots, plan.shape[1], banks, _stream(plan.device)),
          "moe_stage_primary")


def gather_compact_tail(sources, destinations, sizes, prefix_tables, tail, src, dst, count, entries, resident, *,
                        experts):
    """moe_gather_compact_tail on the current stream (all tables CUDA tensors)."""
    for name, t, dt in (("sources", sources, torch.int64), ("destinations", destinations, torch.int64),
                        ("sizes", sizes, torch.int64), ("prefix_tables", prefix_tables, torch.int64),
                        ("tail", tail, torch.int64), ("src", src, torch.int32), ("dst", dst, torch.int32),
                        ("count", count, torch.int64), ("resident", resident, torch.int64)):
        _table(name, t, dt)
    _table("entries", entries, torch.int32, 2)
    _require(entries.shape[0] == 2, "entries must be int32 [2, rows]")
    banks = destinations.numel()
    check(lib().moe_gather_compact_tail(_ptr(sources), _ptr(destinations), _ptr(sizes), _ptr(prefix_tables),
                                        _ptr(tail), _ptr(src), _ptr(dst), _ptr(count), _ptr(entries), _ptr(resident),
                                        experts, entries.shape[1], banks, _stream(src.device)),
          "moe_gather_compact_tail")


# ---------------------------------------------------- combine, shared expert ---

def combine(y, route_pos, scores, *, shared_rows=None, sig=None, out=None):
    """moe_combine on the current stream: the ordered BF16 combine of route
    rows y [rows, H] for route_pos / scores [T, K] (+ the gated shared rows)."""
    for name, t in (("y", y), ("scores", scores)):
        _bf16_2d(t, name)
    _table("route_pos", route_pos, torch.int32, 2)
    tokens, top_k = route_pos.shape
    _require(tuple(scores.shape) == (tokens, top_k), "scores must be [T, K] like route_pos")
    _require((shared_rows is None) == (sig is None), "shared_rows and sig go together")
    hidden = y.shape[1]
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=y.device)
    check(lib().moe_combine(_ptr(y), _ptr(route_pos), _ptr(scores), _ptr(shared_rows), _ptr(sig), tokens, top_k,
                            hidden, _ptr(out), _stream(y.device)), "moe_combine")
    return out


def shared_expert(x, gate, up, down, gate_w=None):
    """moe_shared_expert on the current stream: (out [T, H], sig [T] or None)."""
    for name, t in (("x", x), ("gate", gate), ("up", up), ("down", down)):
        _bf16_2d(t, name)
    tokens, hidden = x.shape
    inner = gate.shape[0]
    out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=x.device)
    sig = torch.empty(tokens, dtype=torch.bfloat16, device=x.device) if gate_w is not None else None
    ws = torch.empty(max(lib().moe_shared_expert_workspace_bytes(tokens, inner), 16), dtype=torch.uint8,
                     device=x.device)
    check(lib().moe_shared_expert(_ptr(x), _ptr(gate), _ptr(up), _ptr(down), _ptr(gate_w), tokens, hidden, inner,
                                  _ptr(out), _ptr(sig), _ptr(ws), ws.numel(), _stream(x.device)),
          "moe_shared_expert")
    return out, sig


def _bf16_2d(t, name):
    _require(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.dim() == 2,
             f"{name} must be a contiguous CUDA BF16 matrix")


# ---------------------------------------------------------------- codecs ---

def _bits_view(t: "torch.Tensor", name: str) -> "torch.Tensor":
    _require(t.is_cuda and t.is_contiguous() and t.element_size() == 2,
             f"{name} must be a contiguous CUDA tensor of 16-bit values (BF16 bits)")
    return t.view(torch.int16)


def rowcodec_plan(bank: "torch.Tensor"):
    """moe_rowcodec_plan on the current stream: the device version of
    bf16_expert_codec.plan_bank for a CUDA bank [E, ...].  Returns (meta int64
    [E, 3] CUDA tensor of (offset or -1, base, escapes), packed bytes,
    workspace).  Synchronises once to read the packed size."""
    bank = _bits_view(bank, "bank")
    rows = bank.shape[0]
    n = bank.numel() // max(rows, 1)
    ws_bytes = lib().moe_rowcodec_workspace_bytes(rows, n)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=bank.device)
    meta = torch.empty((rows, 3), dtype=torch.int64, device=bank.device)
    total = torch.empty(1, dtype=torch.int64, device=bank.device)
    check(lib().moe_rowcodec_plan(_ptr(bank), rows, n, _ptr(meta), _ptr(total), _ptr(ws), ws.numel(),
                                  _stream(bank.device)), "moe_rowcodec_plan")
    return meta, int(total.item()), ws


def rowcodec_pack(bank: "torch.Tensor", meta=None):
    """Device row-codec encoder of a CUDA bank [E, ...] (16-bit BF16 bits):
    the bytes of bf16_expert_codec.pack_bank.  Returns (packed uint8 CUDA
    tensor of max(size, 16) bytes, plan rows as plan_bank: (offset, base,
    escapes) or None).  `meta` (int64 [E, 3] CUDA) overrides the plan, e.g. to
    pack a row that the 1% rule keeps raw."""
    bank = _bits_view(bank, "bank")
    rows = bank.shape[0]
    n = bank.numel() // max(rows, 1)
    planned, size, ws = rowcodec_plan(bank)
    if meta is None:
        meta = planned
    else:
        _table("meta", meta, torch.int64, 2)
        m = meta.cpu()
        size = max([int(o) + row_bytes(n, int(e)) for o, _, e in m.tolist() if o >= 0] + [0])
    packed = torch.zeros(max(size, 16), dtype=torch.uint8, device=bank.device)
    check(lib().moe_rowcodec_pack(_ptr(bank), rows, n, _ptr(meta), _ptr(packed), _ptr(ws), ws.numel(),
                                  _stream(bank.device)), "moe_rowcodec_pack")
    plan = [None if o < 0 else (int(o), int(b), int(e)) for o, b, e in meta.cpu().tolist()]
    return packed, plan


def row_bytes(n: int, escapes: int) -> int:
    """Packed bytes of a row of n values with `escapes` escapes (unaligned)."""
    return 3 * n // 2 + 6 * escapes


def tilecodec_pack(raw: "torch.Tensor"):
    """Device tile-codec encoder (cpu_bf16_reads.h:16-52 pack_cpu_read_tiles)
    of a CUDA array of 256-value tiles.  Returns (packed uint8 [tiles, 384],
    bases uint8 [tiles] with 255 = raw, encoded tiles); raw tiles pack to 384
    zero bytes."""
    raw = _bits_view(raw, "raw")
    _require(raw.numel() % 256 == 0, "raw must hold whole 256-value tiles")
    tiles = raw.numel() // 256
    packed = torch.empty((tiles, 384), dtype=torch.uint8, device=raw.device)
    bases = torch.empty(tiles, dtype=torch.uint8, device=raw.device)
    encoded = torch.zeros(1, dtype=torch.int64, device=raw.device)
    check(lib().moe_tilecodec_pack(_ptr(raw), tiles, _ptr(packed), _ptr(bases), _ptr(encoded),
                                   _stream(raw.device)), "moe_tilecodec_pack")
    return packed, bases, int(encoded.item())


def tilecodec_compact(raw: "torch.Tensor", packed: "torch.Tensor", bases: "torch.Tensor", arena: "torch.Tensor",
                      data_offsets: "torch.Tensor", header_offsets: "torch.Tensor") -> "torch.Tensor":
    """moe_tilecodec_compact on the current stream: assemble the compact rows of
    the resident tile codec from raw rows [rows, n] (CUDA, 16-bit BF16 bits)
    and their moe_tilecodec_pack output into `arena` (CUDA uint8) at the given
    byte offsets (CUDA int64 [rows]; a negative data offset keeps the row out).
    Returns the per-row data bytes (CUDA int64 [rows]; -1 = did not fit)."""
    raw = _bits_view(raw, "raw")
    _require(raw.dim() == 2 and raw.shape[1] % 256 == 0, "raw must be [rows, n] with n a multiple of 256")
    rows, tiles = raw.shape[0], raw.shape[1] // 256
    _require(packed.is_cuda and packed.dtype == torch.uint8 and packed.numel() == rows * tiles * 384,
             "packed must be the CUDA uint8 output of tilecodec_pack for these rows")
    _require(bases.is_cuda and bases.dtype == torch.uint8 and bases.numel() == rows * tiles,
             "bases must be the CUDA uint8 output of tilecodec_pack for these rows")
    _require(arena.is_cuda and arena.dtype == torch.uint8 and arena.is_contiguous(), "arena must be CUDA uint8")
    for name, t in (("data_offsets", data_offsets), ("header_offsets", header_offsets)):
        _require(t.is_cuda and t.dtype == torch.int64 and t.numel() == rows and t.is_contiguous(),
                 f"{name} must be a CUDA int64 tensor of one entry per row")
    sizes = torch.empty(rows, dtype=torch.int64, device=raw.device)
    check(lib().moe_tilecodec_compact(_ptr(raw), _ptr(packed), _ptr(bases), rows, tiles, _ptr(arena), arena.numel(),
                                      _ptr(data_offsets), _ptr(header_offsets), _ptr(sizes), _stream(raw.device)),
          "moe_tilecodec_compact")
    return sizes


def prefix_table(bases) -> "torch.Tensor":
    """Per (expert, 32 tiles): (raw tiles before the group << 32) | bitmask of
    the group's raw tiles (base 255), from tile bases uint8 [E, tiles] (a
    numpy array; tiles a multiple of 32).  Returns int64 [E, tiles / 32] (CPU)."""
    import numpy as np

    bases = np.asarray(bases, dtype=np.uint8)
    _require(bases.ndim == 2 and bases.shape[1] % 32 == 0, "bases must be [E, tiles] with tiles % 32 == 0")
    fallback = (bases == 255).reshape(bases.shape[0], -1, 32)
    flags = np.packbits(fallback, axis=-1, bitorder="little").view(np.uint32).reshape(bases.shape[0], -1)
    counts = fallback.sum(axis=-1, dtype=np.uint64)
    before = counts.cumsum(axis=-1) - counts
    return torch.from_numpy(((before << np.uint64(32)) | flags.astype(np.uint64)).view(np.int64))


class PackedHostBanks:
    """Expert banks kept in pinned host RAM in the lossless row codec of
    bf16_expert_codec (edge35b/bf16_expert_codec.py), with the device
    descriptor table [2][E][3] that moe_layer_forward decodes from:
    (packed row, base, escapes), or (raw row, -1, 0) for a row that does not
    pack.  gate_up [E, 2I, H] and down [E, H, I] are uint16 BF16 bit arrays.
    encoder "device" packs each bank with the device encoders
    (moe_rowcodec_plan / moe_rowcodec_pack) and "host" with the numpy
    encoder; both give the same bytes."""

    def __init__(self, gate_up, down, device, encoder: str = "device"):
        import numpy as np

        from lightreason_b200 import bf16_expert_codec as codec

        _require(encoder in ("device", "host"), f"unknown encoder {encoder!r}")

        self.experts, two_i, self.hidden = gate_up.shape
        self.inner = two_i // 2
        _require(tuple(down.shape) == (self.experts, self.hidden, self.inner), "down must be [E, H, I]")
        table = np.zeros((2, self.experts, 3), dtype=np.int64)
        self.buffers = []
        self.packed_bytes = []
        for b, bank in enumerate((gate_up, down)):
            if encoder == "device":
                packed, rows = rowcodec_pack(torch.from_numpy(np.ascontiguousarray(bank).view(np.int16)).to(device))
            else:
                packed, rows = codec.pack_bank(bank)
                packed = torch.from_numpy(packed)
            row_bytes = bank[0].nbytes
            raw_rows = [e for e, r in enumerate(rows) if r is None]
            tail = (packed.numel() + 15) & ~15
            total = tail + len(raw_rows) * row_bytes
            host = torch.empty(max(total, 16), dtype=torch.uint8).pin_memory()
            host[:packed.numel()].copy_(packed)
            del packed
            host_np = host.numpy()
            base_ptr = host.data_ptr()
            for e, r in enumerate(rows):
                if r is not None:
                    table[b, e] = (base_ptr + r[0], r[1], r[2])
            for j, e in enumerate(raw_rows):
                off = tail + j * row_bytes
                host_np[off:off + row_bytes] = np.ascontiguousarray(bank[e]).view(np.uint8).reshape(-1)
                table[b, e] = (base_ptr + off, -1, 0)
            self.buffers.append(host)
            self.packed_bytes.append([(bank[0].nbytes if r is None else codec.row_bytes(bank[0].size, r[2]))
                                      for r in rows])
        self.descriptors = torch.from_numpy(table).to(device)

    def expert_bytes(self, e: int) -> int:
        """Bytes that cross the host link to stage expert e."""
        return self.packed_bytes[0][e] + self.packed_bytes[1][e]
