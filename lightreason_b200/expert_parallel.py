"""Expert-parallel MoE layer: one process per GPU, experts sharded by rank.

Two exchanges: PeerExchange (the default), where the expert kernel itself
pulls token rows from their senders over NVLink peer memory and stores the
expert rows back into the senders' memory (no host synchronisation), and
TorchExchange, token dispatch and combine through NCCL all-to-all, whose step
is described below.

Rank r of `world` owns the global experts [r*El, (r+1)*El), El = E / world,
and keeps replicas of the router and the shared expert.  One step on rank r:

  1. moe_router_topk on its own T tokens (logits, top-k, BF16 weights and
     the sigmoid shared gate);
  2. moe_permute over the E global experts (eager order: ascending expert,
     slot-major, token), which also groups the routes by owning rank;
  3. moe_ep_dispatch packs the rows and local expert ids in that order and
     counts the routes per destination;
  4. the counts are all-gathered (the one host read of a step: the split
     sizes of the all-to-all), then all_to_all_single moves rows and ids;
  5. moe_ep_unpack + one moe_layer_forward in rows mode over [own tokens ;
     received rows] with top_k = 1 and El + 1 local experts -- the shared
     expert is local expert El -- giving the unweighted row y of every row;
  6. the rows go back with the transposed splits, in the sender's permuted
     order;
  7. moe_ep_combine runs the layer's ordered combine on them: bf16(acc +
     bf16(y * w)) in ascending position (= ascending global expert, the eager
     index_add order), then + bf16(sig * shared row).

The result equals the single-GPU layer bit for bit: every product and every
rounding point is the same, only the place it runs on changes.  The
reference runs this layer on one GPU; there is no reference interface for
the exchange.
"""

from __future__ import annotations

import ctypes
import math

import torch

from lightreason_b200 import native
from lightreason_b200.native import _ptr, _require, check, lib


# phases of one peer-exchange rank step, in launch order
EP_STAGES = ("route", "experts", "finish", "combine")


def shard(experts: int, world: int, rank: int) -> range:
    _require(world >= 1 and experts % world == 0, f"{experts} experts do not shard evenly over {world} ranks")
    el = experts // world
    return range(rank * el, (rank + 1) * el)


def balanced_placement(loads, world: int) -> list[int]:
    """The owner rank of every expert, each rank owning len(loads) / world
    experts, with the per-rank sums of `loads` (routes per expert, measured on
    a calibration batch) balanced by the longest-processing-time rule:
    experts in descending load (ties: lower id first), each to the least
    loaded rank that still has room (ties: the lower rank)."""
    loads = [int(v) for v in loads]
    experts = len(loads)
    _require(world >= 1 and experts % world == 0, f"{experts} experts do not shard evenly over {world} ranks")
    room = [experts // world] * world
    sums = [0] * world
    owner = [0] * experts
    for e in sorted(range(experts), key=lambda e: (-loads[e], e)):
        r = min((q for q in range(world) if room[q] > 0), key=lambda q: (sums[q], q))
        owner[e] = r
        sums[r] += loads[e]
        room[r] -= 1
    return owner


def placement_experts(owner, rank: int) -> list[int]:
    """The experts rank `rank` owns, ascending (its local order)."""
    return [e for e, r in enumerate(owner) if r == rank]


def placement_table(owner) -> list[int]:
    """moe_ep_p2p.placement: (owner << 16) | index among the owner's experts."""
    seen: dict[int, int] = {}
    table = []
    for r in owner:
        table.append((int(r) << 16) | seen.get(r, 0))
        seen[r] = seen.get(r, 0) + 1
    return table


def expert_loads(router: torch.Tensor, x: torch.Tensor, *, bias=None, top_k: int = 8) -> torch.Tensor:
    """Routes per expert (int64 [E], on the device) of the layer's router over
    the tokens x [T, H]: the load a placement balances."""
    native._cuda_bf16(router, "router")
    native._cuda_bf16(x, "x")
    experts, hidden = router.shape
    tokens = x.shape[0]
    d = x.device
    logits = torch.empty((tokens, experts), dtype=torch.bfloat16, device=d)
    idx = torch.empty((tokens, top_k), dtype=torch.int64, device=d)
    check(lib().moe_router_topk(_ptr(x), _ptr(router), _ptr(bias), None, tokens, hidden, experts, top_k,
                                _ptr(logits), _ptr(idx), None, None, None, native._stream(d)), "moe_router_topk")
    return torch.bincount(idx.view(-1), minlength=experts)


class TorchExchange:
    """The all-to-all steps over a torch.distributed process group (NCCL for
    CUDA tensors, gloo for CPU ones).  Rows travel as int32 views (gloo has
    no 16-bit types)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def splits(self, send_counts: torch.Tensor) -> list[list[int]]:
        """All ranks' per-destination counts as a host matrix m[src][dst]."""
        gathered = torch.empty(self.world * self.world, dtype=send_counts.dtype, device=send_counts.device)
        self.dist.all_gather_into_tensor(gathered, send_counts.contiguous(), group=self.group)
        return gathered.view(self.world, self.world).tolist()

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]):
        """Rows of `inp` (dim 0) split by in_splits to the ranks; `out` receives
        out_splits rows from each rank, in rank order."""
        width = math.prod(inp.shape[1:]) * inp.element_size() // 4
        o = out.view(torch.int32).reshape(out.shape[0], width)
        i = inp.view(torch.int32).reshape(inp.shape[0], width)
        self.dist.all_to_all_single(o, i, out_splits, in_splits, group=self.group)


def exchange_step(state, ex, compute) -> list[list[int]]:
    """The exchange of one rank's step around its local compute.  `state`
    holds the rank's buffers (tokens, rank, world, send_counts, send_rows,
    send_meta, xin, recv_meta, yin, ret) with dispatch already done; rows
    received from rank s land in xin after the own tokens, in rank order, and
    the weighted rows go back in the same order, so ret follows the sender's
    permuted order.  Returns the split matrix m[src][dst]."""
    m = ex.splits(state.send_counts)
    r, t = state.rank, state.tokens
    sends = m[r]
    recvs = [m[src][r] for src in range(state.world)]
    received, routes = sum(recvs), sum(sends)
    ex.all_to_all(state.xin[t:t + received], state.send_rows[:routes], recvs, sends)
    ex.all_to_all(state.recv_meta[:received], state.send_meta[:routes], recvs, sends)
    compute(received)
    ex.all_to_all(state.ret[:routes], state.yin[t:t + received], sends, recvs)
    return m


class ExpertParallelLayer:
    """One rank's share of the expert-parallel layer (device BF16 tensors).

    gate_up [El, 2I, H] and down [El, H, I]: this rank's experts in ascending
    id -- shard(E, world, rank), or with `placement` (owner rank per expert,
    e.g. balanced_placement of measured loads; peer exchange only) the
    experts it assigns to this rank; router [E, H], bias (f32 [E] or None)
    and the shared expert are replicas.  `tokens` bounds the per-step token
    count (it sizes the buffers)."""

    def __init__(self, *, router, gate_up, down, shared_gate, shared_up, shared_down, shared_gate_w, rank, world,
                 tokens, bias=None, top_k=8, exchange=None, placement=None):
        native._cuda_bf16(router, "router")
        self.experts, self.hidden = router.shape
        self.rank, self.world, self.top_k = rank, world, top_k
        self.placement = None
        if placement is not None:
            owner = [int(r) for r in placement]
            _require(len(owner) == self.experts and all(0 <= r < world for r in owner) and
                     all(owner.count(r) == self.experts // world for r in range(world)),
                     "placement must give every rank E / world experts")
            self.placement = owner
        self.expert_ids = (placement_experts(self.placement, rank) if self.placement is not None
                           else list(shard(self.experts, world, rank)))
        self.local_experts = len(self.expert_ids)
        _require(tuple(gate_up.shape[:1]) == (self.local_experts,) and tuple(down.shape[:1]) == (self.local_experts,),
                 "gate_up/down must hold this rank's experts")
        _require(shared_gate.shape[0] == gate_up.shape[1] // 2,
                 "the shared expert runs as a local expert: its inner width must equal the experts'")
        self.router, self.bias, self.shared_gate_w = router, bias, shared_gate_w
        self.dev = router.device
        # Local banks: the rank's experts, then the shared expert as expert El.
        self.gate_up = torch.cat([gate_up, torch.cat([shared_gate, shared_up], 0)[None]], 0).contiguous()
        self.down = torch.cat([down, shared_down[None]], 0).contiguous()
        self.local = native.Layer(gate_up=self.gate_up, down=self.down, top_k=1)
        self.exchange = exchange
        self.max_tokens = tokens
        routes = tokens * top_k
        recv_max = world * routes          # every rank may route everything here
        d = self.dev
        bf = dict(dtype=torch.bfloat16, device=d)
        i32 = dict(dtype=torch.int32, device=d)
        self.logits = torch.empty((tokens, self.experts), **bf)
        self.idx = torch.empty((tokens, top_k), dtype=torch.int64, device=d)
        self.scores = torch.empty((tokens, top_k), **bf)
        self.offsets = torch.empty(self.experts + 1, **i32)
        self.perm_token = torch.empty(max(routes, 1), **i32)
        self.perm_slot = torch.empty(max(routes, 1), **i32)
        self.route_pos = torch.empty((tokens, top_k), **i32)
        self.active = torch.empty(self.experts, **i32)
        self.counters = torch.zeros(2, **i32)
        self.send_rows = torch.empty((max(routes, 1), self.hidden), **bf)
        self.send_meta = torch.empty(max(routes, 1), **i32)
        self.send_counts = torch.zeros(world, dtype=torch.int64, device=d)
        self.sig = torch.empty(tokens, **bf)
        # [own tokens ; received rows] and their one-slot routes.
        self.xin = torch.empty((tokens + recv_max, self.hidden), **bf)
        self.route_in = torch.full((tokens + recv_max, 1), self.local_experts, dtype=torch.int64, device=d)
        self.recv_meta = torch.empty(max(recv_max, 1), **i32)
        self.yin = torch.empty((tokens + recv_max, self.hidden), **bf)
        self.ret = torch.empty((max(routes, 1), self.hidden), **bf)
        self.last_splits = None
        self._own_routes = tokens
        # K-split router partials: at most 4 splits of [T, E] FP32 for any T <= tokens
        self.rsplit = torch.empty(16 * tokens * self.experts + 16, dtype=torch.uint8, device=d)

    # -- phases (split out so that one process can drive several virtual ranks)
    def dispatch(self, x: torch.Tensor) -> None:
        _require(self.placement is None, "an expert placement runs with the peer exchange only")
        native._cuda_bf16(x, "x")
        tokens = x.shape[0]
        _require(tokens <= self.max_tokens and x.shape[1] == self.hidden, "x must be [T <= tokens, H]")
        self.tokens = tokens
        s = native._stream(self.dev)
        if tokens > self._own_routes:
            self.route_in[:tokens].fill_(self.local_experts)   # unpack reuses the rows past the own tokens
        self._own_routes = tokens
        self.xin[:tokens].copy_(x)
        if self.bias is not None:
            _require(self.bias.is_cuda and self.bias.dtype == torch.float32, "bias must be CUDA f32 [E]")
        # the layer's own router (same K splits as moe_layer_forward at this width)
        check(lib().moe_router_topk_ws(_ptr(self.xin), _ptr(self.router), _ptr(self.bias), _ptr(self.shared_gate_w),
                                       tokens, self.hidden, self.experts, self.top_k, _ptr(self.logits),
                                       _ptr(self.idx), None, _ptr(self.scores), _ptr(self.sig), _ptr(self.rsplit),
                                       self.rsplit.numel(), s), "moe_router_topk_ws")
        c = self.counters.data_ptr()
        check(lib().moe_permute(_ptr(self.idx), tokens, self.top_k, self.experts, _ptr(self.offsets),
                                _ptr(self.perm_token), _ptr(self.perm_slot), _ptr(self.route_pos), _ptr(self.active),
                                c, c + 4, s), "moe_permute")
        check(lib().moe_ep_dispatch(_ptr(self.xin), _ptr(self.idx), _ptr(self.offsets),
                                    _ptr(self.perm_token), _ptr(self.perm_slot), tokens, self.top_k, self.experts,
                                    self.hidden, self.world, _ptr(self.send_rows), _ptr(self.send_meta),
                                    _ptr(self.send_counts), s), "moe_ep_dispatch")

    def compute(self, received: int, stage_events=None) -> None:
        """Local experts over [own tokens ; `received` rows already in xin/recv_meta]
        (stage_events: as in native.Layer.forward, for the local layer)."""
        t = self.tokens
        s = native._stream(self.dev)
        check(lib().moe_ep_unpack(_ptr(self.recv_meta), received, self.route_in[t:].data_ptr(), s), "moe_ep_unpack")
        n = t + received
        self.local(self.xin[:n], route_in=self.route_in[:n], out=self.yin[:n], stage_events=stage_events,
                   rows_mode=True)

    def combine(self, out: torch.Tensor) -> torch.Tensor:
        t = self.tokens
        check(lib().moe_ep_combine(_ptr(self.ret), _ptr(self.route_pos), _ptr(self.scores), _ptr(self.yin),
                                   _ptr(self.sig), t, self.top_k, self.hidden, _ptr(out), native._stream(self.dev)),
              "moe_ep_combine")
        return out

    # -- one distributed step
    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stage_events=None,
                ep_events=None) -> torch.Tensor:
        """One rank step.  stage_events: the local layer's stage events (as in
        native.Layer.forward).  ep_events (peer exchange only): None or
        len(EP_STAGES) + 1 torch.cuda.Event recorded on the compute stream at
        the boundaries of the step's phases."""
        _require(self.exchange is not None, "forward needs an exchange (use run_virtual_ranks for one process)")
        if isinstance(self.exchange, PeerExchange):
            return self._forward_peer(x, torch.empty_like(x) if out is None else out, stage_events, ep_events)
        self.dispatch(x)
        self.last_splits = exchange_step(self, self.exchange,
                                         lambda received: self.compute(received, stage_events))
        return self.combine(torch.empty_like(x) if out is None else out)

    __call__ = forward

    # -- the peer-memory step: no host synchronisation, graph-capturable
    def _peer_buffers(self):
        ex = self.exchange
        if getattr(self, "_peer_ready", False):
            return
        _require(ex.capacity >= self.max_tokens * self.top_k and ex.own_rows >= self.max_tokens,
                 "peer exchange sized below tokens * top_k")
        d = self.dev
        rws = lib().moe_ep_p2p_route_workspace_bytes(ctypes.byref(ex.args), self.max_tokens)
        self.p_rsplit = self.rsplit if self.rsplit.numel() >= rws else torch.empty(rws, dtype=torch.uint8, device=d)
        self.p_shared = torch.empty((self.max_tokens, self.hidden), dtype=torch.bfloat16, device=d)
        self.p_stats = torch.zeros(2 + self.world, dtype=torch.int32, device=d)
        inner = self.gate_up.shape[1] // 2
        self.p_inner = inner
        ws = lib().moe_ep_p2p_workspace_bytes(ctypes.byref(ex.args), inner)
        _require(ws > 0, "peer exchange: workspace query failed")
        self.p_ws = torch.empty(ws, dtype=torch.uint8, device=d)
        self.p_place = None
        if self.placement is not None:
            self.p_place = torch.tensor(placement_table(self.placement), dtype=torch.int32, device=d)
        ex.args.placement = self.p_place.data_ptr() if self.p_place is not None else None
        self._peer_ready = True

    def _forward_peer(self, x, out, stage_events, ep_events=None):
        """One rank step over the peer exchange: route (the router over the own
        tokens, which also puts the own rows into the symmetric buffer and one
        entry per route into its owner's, each route's return row ordered by
        expert id within its token), the owner's plan and grouped kernel (rows
        pulled from their senders, expert rows stored into the senders' ret),
        finish (flags), the ordered combine.  stage_events: None or two CUDA
        events recorded around the grouped kernel."""
        ex = self.exchange
        self._peer_buffers()
        native._cuda_bf16(x, "x")
        tokens = x.shape[0]
        _require(tokens <= self.max_tokens and x.shape[1] == self.hidden, "x must be [T <= tokens, H]")
        _require(ep_events is None or len(ep_events) == len(EP_STAGES) + 1,
                 f"ep_events must hold {len(EP_STAGES) + 1} events")
        self.tokens = tokens
        s = native._stream(self.dev)
        a = ctypes.byref(ex.args)

        def mark(i):
            if ep_events is not None:
                ep_events[i].record()
        mark(0)
        check(lib().moe_ep_p2p_route(a, _ptr(x), tokens, _ptr(self.router), _ptr(self.bias),
                                     _ptr(self.shared_gate_w), _ptr(self.logits), _ptr(self.idx), _ptr(self.scores),
                                     _ptr(self.sig), _ptr(self.route_pos), _ptr(self.p_rsplit),
                                     self.p_rsplit.numel(), s), "moe_ep_p2p_route")
        mark(1)
        kev = None
        if stage_events is not None:
            for e in stage_events:
                if not e.cuda_event:
                    e.record()  # torch creates the CUDA event lazily on first record
            kev = (native._p * 2)(*[e.cuda_event for e in stage_events])
        check(lib().moe_ep_p2p_experts(a, _ptr(self.gate_up), _ptr(self.down), self.p_inner, tokens,
                                       _ptr(self.p_shared), _ptr(self.p_stats), _ptr(self.p_ws), self.p_ws.numel(),
                                       kev, s), "moe_ep_p2p_experts")
        mark(2)
        check(lib().moe_ep_p2p_finish(a, s), "moe_ep_p2p_finish")
        mark(3)
        check(lib().moe_ep_combine(ctypes.c_void_p(ex.ret_ptr), _ptr(self.route_pos), _ptr(self.scores),
                                   _ptr(self.p_shared), _ptr(self.sig), tokens, self.top_k, self.hidden, _ptr(out), s),
              "moe_ep_combine")
        mark(4)
        return out

    def peer_stats(self) -> dict:
        """This rank's share of the last peer step (syncs): rows received from
        each sender, local experts with rows."""
        v = self.p_stats.tolist()
        return {"rows_received": v[0], "local_experts_with_rows": v[1], "rows_per_sender": v[2:]}


class PeerExchange:
    """Symmetric buffers over NVLink for ExpertParallelLayer: one CUDA-IPC
    buffer per rank (moe_ipc_alloc), mapped by every peer, laid out as
    moe_ep_p2p describes: flags, counts, one 16-byte meta entry per route a
    sender may send (capacity = tokens * top_k per sender, so no route is ever
    dropped), the rank's own token rows [tokens, H], which the owners of its
    routes read, and the return rows [capacity, H] they write.  Construct it
    on every rank of the process group together; close() before the group
    ends."""

    def __init__(self, *, world, rank, tokens, top_k, hidden, experts, device, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.world, self.rank = world, rank
        self.capacity = tokens * top_k
        self.own_rows = tokens
        cap, h = self.capacity, hidden
        align = lambda v, a: (v + a - 1) // a * a  # noqa: E731
        off_fp, off_fr, off_count, off_meta = 0, 256, 512, 1024
        off_tokens = align(off_meta + world * cap * 16, 4096)
        off_ret = align(off_tokens + tokens * h * 2, 4096)
        total = off_ret + cap * h * 2
        _require(world <= 64, "at most 64 ranks")
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        check(lib().moe_ipc_alloc(total, ctypes.byref(base), handle), "moe_ipc_alloc")
        self._base = base
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        if world > 1:
            every = torch.empty(world * 64, dtype=torch.uint8, device=device)
            dist.all_gather_into_tensor(every, mine, group=group)
            handles = every.view(world, 64).cpu().numpy()
        else:
            handles = mine.view(1, 64).cpu().numpy()
        self._opened = []
        peers = []
        for q in range(world):
            if q == rank:
                peers.append(base.value)
                continue
            h_q = (ctypes.c_uint8 * 64)(*handles[q].tolist())
            p = ctypes.c_void_p()
            check(lib().moe_ipc_open(h_q, ctypes.byref(p)), "moe_ipc_open")
            self._opened.append(p)
            peers.append(p.value)
        i32 = dict(dtype=torch.int32, device=device)
        self.peers = torch.tensor(peers, dtype=torch.int64, device=device)
        self.step = torch.ones(1, **i32)
        self.sync = torch.zeros(2 + 64, **i32)  # two last-CTA counters, a send count per rank
        self.error = torch.zeros(1, **i32)
        self.ret_ptr = base.value + off_ret
        self.args = native.EpP2P(peers=self.peers.data_ptr(), off_flags_publish=off_fp, off_flags_return=off_fr,
                                 off_count=off_count, off_meta=off_meta, off_tokens=off_tokens, off_ret=off_ret,
                                 world=world,
                                 rank=rank, capacity=cap, hidden=hidden, top_k=top_k, experts=experts,
                                 local_experts=experts // world, own_rows=tokens, step=self.step.data_ptr(),
                                 sync=self.sync.data_ptr(), error=self.error.data_ptr())
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier(group=group)  # every mapping exists before any rank's first step

    def check(self) -> None:
        """Raise if a bounded wait of an earlier step gave up (syncs the device)."""
        code = int(self.error.item())
        if code:
            what = {1: "a sender never published its routes", 2: "an owner never returned its rows",
                    3: "the expert kernel gave up waiting",
                    4: "the expert placement table is malformed"}.get(code, "unknown")
            raise RuntimeError(f"expert-parallel exchange failed ({code}): {what}")

    def close(self) -> None:
        torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier(group=self.group)
        for p in self._opened:
            lib().moe_ipc_close(p)
        self._opened.clear()
        if self.world > 1:
            self.dist.barrier(group=self.group)
        if self._base:
            lib().moe_ipc_free(self._base)
            self._base = None


def run_virtual_ranks(layers: list[ExpertParallelLayer], xs: list[torch.Tensor], outs=None,
                      stage_events=None) -> list[torch.Tensor]:
    """One step of `len(layers)` ranks driven from one process on one device:
    the all-to-all becomes device copies between the ranks' buffers.  Same
    kernels and buffers as the distributed step (for parity tests and for
    measuring the layer at a world size larger than the GPUs at hand)."""
    world = len(layers)
    for layer, x in zip(layers, xs):
        layer.dispatch(x)
    m = torch.stack([layer.send_counts for layer in layers]).tolist()
    for dst, layer in enumerate(layers):
        row = layer.tokens
        for src in range(world):
            lo = sum(m[src][:dst])
            n = m[src][dst]
            layer.xin[row:row + n].copy_(layers[src].send_rows[lo:lo + n])
            layer.recv_meta[row - layer.tokens:row - layer.tokens + n].copy_(layers[src].send_meta[lo:lo + n])
            row += n
        layer.compute(row - layer.tokens, stage_events if dst == 0 else None)
    for src, layer in enumerate(layers):
        pos = 0
        for dst in range(world):
            n = m[src][dst]
            start = layers[dst].tokens + sum(m[s][dst] for s in range(src))
            layer.ret[pos:pos + n].copy_(layers[dst].yin[start:start + n])
            pos += n
    outs = outs or [torch.empty_like(x) for x in xs]
    return [layer.combine(o) for layer, o in zip(layers, outs)]


__all__ = ["EP_STAGES", "ExpertParallelLayer", "PeerExchange", "TorchExchange", "balanced_placement",
           "exchange_step", "expert_loads", "placement_experts", "placement_table", "run_virtual_ranks", "shard"]
