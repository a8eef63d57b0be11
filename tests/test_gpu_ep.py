"""Expert-parallel layer on the GPU.

* Virtual ranks (one device, the exchange as device copies): every rank's
  output equals the single-GPU layer on the same tokens bit for bit, for
  world sizes 1, 2, 4 and 8 at the 35B shapes with Zipf-skewed routing.
* Real ranks (NCCL, one process per GPU; skipped with fewer than 2 GPUs): the
  same equality across processes.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from lightreason_b200 import build, native
from lightreason_b200 import synthetic as S
from lightreason_b200.expert_parallel import ExpertParallelLayer, run_virtual_ranks, shard
from oracle import oracle as O
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


def to_dev(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


class Weights:
    def __init__(self, seed: int, dev):
        self.w = S.layer_weights(seed, bias="zipf")
        self.gu, self.dn = self.w.stacked()
        d = lambda a: to_dev(a, dev)  # noqa: E731
        self.router, self.gu_dev, self.dn_dev = d(self.w.router), d(self.gu), d(self.dn)
        self.sh = [d(self.w.sh_gate), d(self.w.sh_up), d(self.w.sh_down), d(self.w.sh_gate_w)]
        self.bias = torch.from_numpy(self.w.bias).to(dev)
        self.single = native.Layer(router=self.router, gate_up=self.gu_dev, down=self.dn_dev, bias=self.bias,
                                   shared_gate=self.sh[0], shared_up=self.sh[1], shared_down=self.sh[2],
                                   shared_gate_w=self.sh[3])

    def rank_layer(self, rank: int, world: int, tokens: int, exchange=None, device=None, placement=None):
        from lightreason_b200.expert_parallel import placement_experts

        mine = placement_experts(placement, rank) if placement is not None else list(shard(256, world, rank))
        sel = torch.tensor(mine, dtype=torch.int64, device=self.gu_dev.device)
        mv = (lambda t: t.to(device)) if device is not None else (lambda t: t)  # noqa: E731
        return ExpertParallelLayer(router=mv(self.router), gate_up=mv(self.gu_dev.index_select(0, sel)),
                                   down=mv(self.dn_dev.index_select(0, sel)), shared_gate=mv(self.sh[0]),
                                   shared_up=mv(self.sh[1]), shared_down=mv(self.sh[2]), shared_gate_w=mv(self.sh[3]),
                                   bias=mv(self.bias), rank=rank, world=world, tokens=tokens, exchange=exchange,
                                   placement=placement)


@pytest.fixture(scope="module")
def dev():
    build.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    native.device_check(0)
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def weights(dev):
    return Weights(41, dev)


@pytest.mark.parametrize("world,tokens", [(1, 48), (2, 64), (4, 40), (8, 512)])
def test_virtual_ranks_equal_single_gpu_layer(dev, weights, world, tokens):
    layers = [weights.rank_layer(r, world, tokens) for r in range(world)]
    xs = [to_dev(S.hidden_states(1000 + 10 * world + r, tokens), dev) for r in range(world)]
    outs = run_virtual_ranks(layers, xs)
    for r, (x, out) in enumerate(zip(xs, outs)):
        want = weights.single(x)
        torch.cuda.synchronize()
        assert np.array_equal(bits(out), bits(want)), f"rank {r} of {world}"
    # a second step on the same buffers with other tokens
    xs = [to_dev(S.hidden_states(2000 + 10 * world + r, tokens // 2 + 1), dev) for r in range(world)]
    outs = run_virtual_ranks(layers, xs)
    for x, out in zip(xs, outs):
        assert np.array_equal(bits(out), bits(weights.single(x)))


def test_virtual_ranks_against_oracle(dev, weights):
    world, tokens = 4, 16
    layers = [weights.rank_layer(r, world, tokens) for r in range(world)]
    x_bits = [S.hidden_states(3000 + r, tokens) for r in range(world)]
    outs = run_virtual_ranks(layers, [to_dev(x, dev) for x in x_bits])
    w = weights.w
    for r in (0, 3):
        idx = layers[r].idx[:tokens].cpu().numpy()
        sc = bits(layers[r].scores[:tokens])
        offsets, ptok, _, rpos = O.permute(idx, 256)
        y = O.experts_by_route(x_bits[r], weights.gu, weights.dn, offsets, ptok, 256)
        sh, sig = O.shared_expert(x_bits[r], w.sh_gate, w.sh_up, w.sh_down, w.sh_gate_w)
        assert_close(bits(outs[r]), O.combine(y, rpos, sc, sh, sig), what=f"expert-parallel rank {r}")


def _nccl_rank(rank: int, world: int, port: int, tokens: int, failures) -> None:
    import torch.distributed as dist

    from lightreason_b200.expert_parallel import TorchExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        w = Weights(41, dev)
        layer = w.rank_layer(rank, world, tokens, exchange=TorchExchange())
        for step in range(2):
            x = to_dev(S.hidden_states(4000 + 10 * step + rank, tokens), dev)
            out = layer(x)
            want = w.single(x)
            torch.cuda.synchronize()
            if not np.array_equal(bits(out), bits(want)):
                failures.put(f"rank {rank} step {step}: output differs from the single-GPU layer")
        dist.barrier()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        failures.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_ranks_equal_single_gpu_layer():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    failures = ctx.SimpleQueue()
    mp.start_processes(_nccl_rank, args=(world, _free_port(), 128, failures), nprocs=world, start_method="spawn")
    errs = []
    while not failures.empty():
        errs.append(failures.get())
    assert not errs, errs


def test_peer_exchange_one_rank_equals_single_gpu_layer(dev, weights):
    """The peer-memory step at world 1 (its own buffer as the only peer; every
    wait is on a kernel that already finished earlier in the stream): kernels
    and buffer layout, bit-exact against the single-GPU layer, twice in a row,
    and replayed from a CUDA graph."""
    from lightreason_b200.expert_parallel import PeerExchange

    tokens = 96
    ex = PeerExchange(world=1, rank=0, tokens=tokens, top_k=8, hidden=2048, experts=256, device=dev)
    try:
        layer = weights.rank_layer(0, 1, tokens, exchange=ex)
        for step in range(2):
            x = to_dev(S.hidden_states(5000 + step, tokens - 7 * step), dev)
            out = layer(x)
            ex.check()
            assert np.array_equal(bits(out), bits(weights.single(x))), step
        x = to_dev(S.hidden_states(5100, tokens), dev)
        out = torch.empty_like(x)
        layer(x, out=out)                                    # warm every buffer before capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer(x, out=out)
        for seed in (5200, 5300):
            x.copy_(to_dev(S.hidden_states(seed, tokens), dev))
            g.replay()
            torch.cuda.synchronize()
            ex.check()
            assert np.array_equal(bits(out), bits(weights.single(x))), seed
        del g
    finally:
        ex.close()


def _peer_rank(rank: int, world: int, port: int, tokens: int, failures, balanced: bool = False) -> None:
    import torch.distributed as dist

    from lightreason_b200.expert_parallel import PeerExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    ex = None
    try:
        w = Weights(41, dev)
        placement = None
        if balanced:
            from lightreason_b200.expert_parallel import balanced_placement, expert_loads

            loads = expert_loads(w.router, to_dev(S.hidden_states(6900 + rank, tokens), dev), bias=w.bias)
            dist.all_reduce(loads)
            placement = balanced_placement(loads.cpu().tolist(), world)
            if placement == [e * world // 256 for e in range(256)]:
                failures.put(f"rank {rank}: the balanced placement is the contiguous one; the test needs another")
        ex = PeerExchange(world=world, rank=rank, tokens=tokens, top_k=8, hidden=2048, experts=256, device=dev)
        layer = w.rank_layer(rank, world, tokens, exchange=ex, placement=placement)
        for step in range(3):
            x = to_dev(S.hidden_states(6000 + 10 * step + rank, tokens - step), dev)
            out = layer(x)
            want = w.single(x)
            torch.cuda.synchronize()
            ex.check()
            if not np.array_equal(bits(out), bits(want)):
                failures.put(f"rank {rank} step {step}: peer-exchange output differs from the single-GPU layer")
        dist.barrier()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        failures.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("balanced", [False, True], ids=["contiguous", "balanced"])
def test_peer_exchange_ranks_equal_single_gpu_layer(balanced):
    """Real ranks over NVLink peer memory, bit-exact against the single-GPU
    layer: contiguous expert ranges, and a placement balanced on measured
    routes (experts of one rank scattered over the id range)."""
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    failures = ctx.SimpleQueue()
    mp.start_processes(_peer_rank, args=(world, _free_port(), 128, failures, balanced), nprocs=world,
                       start_method="spawn")
    errs = []
    while not failures.empty():
        errs.append(failures.get())
    assert not errs, errs
