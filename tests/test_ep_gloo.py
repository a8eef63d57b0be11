"""Expert parallelism on CPU: two gloo ranks run the exchange of
lightreason_b200.expert_parallel (TorchExchange + exchange_step, the code the
NCCL path runs) around the oracle's arithmetic, and each rank's output must
equal the single-process oracle layer bit for bit.

This pins the decomposition the GPU path relies on: dispatch in the permuted
order, unweighted expert rows computed by the owning rank (the shared expert
as one more local expert of the home rank), and the layer's ordered BF16
combine on the home rank over the returned rows.
"""

from __future__ import annotations

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from lightreason_b200 import synthetic as S

EXPERTS, TOKENS, HIDDEN, INNER = 16, 5, 256, 128


def _rows(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy().view(np.uint16)


def _weights():
    w = S.layer_weights(77, experts=EXPERTS, hidden=HIDDEN, inner=INNER, shared_inner=INNER)
    gu, dn = w.stacked()
    return w, gu, dn


def _rank_main(rank: int, world: int, port: int, failures) -> None:
    import torch.distributed as dist

    from lightreason_b200.expert_parallel import TorchExchange, exchange_step, shard
    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, gu, dn = _weights()
        x = S.hidden_states(900 + rank, TOKENS, hidden=HIDDEN)
        want = O.moe_layer(x, w.router, w.bias, gu, dn, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)[0]

        # dispatch (what router_topk + permute + moe_ep_dispatch produce)
        logits = O.linear_bf16(x, w.router)
        idx, _, scores = O.router_select(logits, w.bias, 8)
        offsets, ptok, pslot, rpos = O.permute(idx, EXPERTS)
        el = EXPERTS // world
        routes = int(offsets[EXPERTS])
        eid = idx[ptok, pslot]
        meta = eid % el
        counts = [int(offsets[min((d + 1) * el, EXPERTS)] - offsets[d * el]) for d in range(world)]
        st = SimpleNamespace(
            rank=rank, world=world, tokens=TOKENS,
            send_counts=torch.tensor(counts, dtype=torch.int64),
            send_rows=_rows(x[ptok]), send_meta=torch.from_numpy(meta.astype(np.int32)),
            xin=torch.empty((TOKENS + world * routes * 2, HIDDEN), dtype=torch.bfloat16),
            recv_meta=torch.empty(world * routes * 2, dtype=torch.int32),
            yin=torch.empty((TOKENS + world * routes * 2, HIDDEN), dtype=torch.bfloat16),
            ret=torch.empty((routes, HIDDEN), dtype=torch.bfloat16))
        mine = shard(EXPERTS, world, rank)

        sh, sig = O.shared_expert(x, w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)

        def compute(received: int) -> None:
            st.yin[:TOKENS] = _rows(sh)                       # the shared expert: local expert El
            if received == 0:
                return
            rows = _bits(st.xin[TOKENS:TOKENS + received])
            local = st.recv_meta[:received].numpy().astype(np.int64).reshape(-1, 1)
            assert local.max() < el
            loc_off, loc_tok, _, _ = O.permute(local, el)
            y = O.experts_by_route(rows, gu[mine.start:mine.stop], dn[mine.start:mine.stop], loc_off, loc_tok, el)
            unweighted = np.empty_like(y)
            unweighted[loc_tok] = y                           # back to the received order
            st.yin[TOKENS:TOKENS + received] = _rows(unweighted)

        m = exchange_step(st, TorchExchange(), compute)
        assert sum(m[rank]) == routes
        got = O.combine(_bits(st.ret), rpos, scores, _bits(st.yin[:TOKENS]), sig)
        if not np.array_equal(got, want):
            failures.put(f"rank {rank}: {int((got != want).sum())} values differ")
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        failures.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_expert_parallel_exchange_matches_single_layer(world):
    ctx = mp.get_context("spawn")
    failures = ctx.SimpleQueue()
    mp.start_processes(_rank_main, args=(world, _free_port(), failures), nprocs=world, start_method="spawn")
    errs = []
    while not failures.empty():
        errs.append(failures.get())
    assert not errs, errs


def test_balanced_placement_rule():
    """Expert placement by the longest-processing-time rule: every rank owns
    E / world experts, every expert exactly one owner, the heaviest experts
    land on distinct ranks, and the per-rank load is within one expert's load
    of the mean (the rule's bound when every rank has the same room)."""
    from lightreason_b200.expert_parallel import balanced_placement, placement_experts, placement_table

    rng = np.random.default_rng(3)
    loads = (1000 / np.arange(1, 257) ** 1.1 * rng.uniform(0.5, 1.5, 256)).astype(np.int64)
    rng.shuffle(loads)
    for world in (2, 4, 8):
        owner = balanced_placement(loads, world)
        assert sorted(set(owner)) == list(range(world))
        assert all(owner.count(r) == 256 // world for r in range(world))
        sums = np.bincount(owner, weights=loads, minlength=world)
        assert sums.max() - sums.mean() <= loads.max(), (world, sums)
        top = np.argsort(-loads, kind="stable")[:world]
        assert len({owner[e] for e in top}) == world
        # the table the kernels read: (owner << 16) | index among the owner's experts, ascending ids
        table = placement_table(owner)
        for r in range(world):
            mine = placement_experts(owner, r)
            assert mine == sorted(mine)
            assert [table[e] for e in mine] == [(r << 16) | j for j in range(len(mine))]
    # equal loads: ties go to the lower rank, i.e. round robin
    assert balanced_placement([5] * 8, 4) == [0, 1, 2, 3, 0, 1, 2, 3]
